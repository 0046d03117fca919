// The chunked recurrence's tensor-core (tcgen05 / TMEM) kernels (chunk_tc.cu).
#pragma once
#include <cuda_bf16.h>
#include "gdn_common.cuh"

namespace gdn {

// Bytes of one chunk's tile images: [64][128] (W', Q), [128][64] (E^T, U'^T,
// D^T), [128][128] (S^T), bf16 in the layout of img_off (ptx_sm100.cuh).
size_t chunk_img_w_bytes();
size_t chunk_img_e_bytes();
size_t chunk_img_s_bytes();

// State passing over the nc chunks of every head (grid = hv CTAs): reads the
// W', E^T and U'^T images [hv][nc] and the chunks' decays gchunk [hv][nc],
// updates S [hv][128][128] (fp32, row = k, col = v) in place, and writes each
// chunk's start state (simg, S^T images) and deltas (dimg, D^T images).
int launch_chunk_scan_tc(const uint8_t* wimg, const uint8_t* eimg, const uint8_t* uimg, const float* gchunk, float* S,
                         uint8_t* simg, uint8_t* dimg, int hv, int64_t nc, cudaStream_t s);

// Outputs of every (chunk, head), RMSNorm, SiLU(z) gate -> fp16 rows of
// `gated` [T][hv * 128] or, with gated == NULL, the rows of `dst`.
int launch_chunk_out_tc(const __nv_bfloat16* qn, const __nv_bfloat16* kn, const uint8_t* simg, const uint8_t* dimg,
                        const float* gcum, const float* proj, int64_t ldp, const float* head_norm, __half* gated,
                        const RowDest& dst, int64_t T, int64_t Tp, int hk, int hv, int qkv, int head_map,
                        cudaStream_t s);

}  // namespace gdn
