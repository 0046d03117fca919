// The decode step and its helpers (decode.cu).
#pragma once
#include "gdn_common.cuh"

namespace gdn {

// Scratch of a decode step: for any layer of these dims, and for this layer
// (the out_proj split-K partials only when its out_proj splits).
size_t decode_workspace_bytes(const gdn_dims& d, int64_t batch);
size_t decode_workspace_bytes_for(const gdn_layer& L, int64_t batch, int flags = 0,
                                  int x_dtype = GDN_DTYPE_F32);
int validate_layer(const gdn_layer* L);
// flags: 0 or GDN_DECODE_REF_PROJECTIONS
int decode_step(const gdn_layer* L, int64_t B, const void* x, int x_dtype, float* out, float* S, float* conv_buf,
                int32_t* conv_pos, void* ws, size_t ws_bytes, cudaStream_t s, int flags = 0);
int profile_enable(int on);
// Records phase event i (0..4) on s when phase timing is enabled; no-op otherwise.
int phase_mark(int i, cudaStream_t s);
int phase_ms(float* ms, int n);

}  // namespace gdn
