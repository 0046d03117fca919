// Chunked prefill (prefill.cu).
#pragma once
#include "gdn_common.cuh"

namespace gdn {

size_t prefill_workspace_bytes(const gdn_dims& d, int64_t T);

// A highest-priority side stream of the calling host thread on the current
// device, with a fork and a join event (created on first use, kept).
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
int side_stream(SideStream** out);
// out [T][hidden] fp32 after out_proj, or (out == NULL) the gated head outputs
// before out_proj: token t's [Hv*128] fp16 row goes to gated_out->row(t) (see RowDest).
int prefill(const gdn_layer* L, int64_t T, const void* x, int x_dtype, float* out, const RowDest* gated_out,
            float* S, float* conv_buf, int32_t* conv_pos, void* ws, size_t ws_bytes, cudaStream_t s);
int validate_layer(const gdn_layer* L);

}  // namespace gdn
