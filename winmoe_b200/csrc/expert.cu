// The expert FFN of the MoE layers on the device (the fused GPU route of the
// reference, engine/runtime/gpu_offload.cu:718-751, gpu_expert_ffn_fused, and
// its batched accumulation, :766-793): for m tokens,
//     g = W_gate x, u = W_up x            (hidden -> inter, Q4_K or Q5_K)
//     a = (g * sigmoid(g)) * u            (swiglu_kernel, :460-466)
//     y = W_down a                        (inter -> hidden, Q4_K or Q5_K)
//     out = y, or out += weight * y       (weighted_add_kernel, :469-471)
// The projections are the streamed GEMVs of gemv_stream.cu (fp32 arithmetic up
// to summation order, as the reference's fp32-activation GPU kernels); the
// expert cache that owns the weights stays the reference's.
#include "gdn_common.cuh"
#include "quant.cuh"

namespace gdn {
namespace {

// a = (g * sigmoid(g)) * u with sigmoid(g) = 1 / (1 + expf(-g)), in the
// reference kernel's order of operations.
__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ a,
                              int64_t n) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float gv = g[i];
    const float sig = 1.0f / (1.0f + expf(-gv));
    a[i] = (gv * sig) * u[i];
}

// out[i] += weight * y[i].
__global__ void weighted_add_kernel(float* __restrict__ out, const float* __restrict__ y, float weight, int64_t n) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = fmaf(weight, y[i], out[i]);
}

int gemv(int type, const void* w, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
         cudaStream_t s) {
    return type == GDN_GGML_Q4_K ? launch_q4_k_gemv(w, n, k, x, dt, m, y, n, s)
                                 : launch_q5_k_gemv(w, n, k, x, dt, m, y, n, s);
}

}  // namespace

size_t expert_ffn_workspace_bytes(int64_t m, int64_t hidden, int64_t inter) {
    // g, u, a: [m][inter] fp32 each; y: [m][hidden] fp32; 256-byte aligned pieces
    return 3 * round_up((size_t)m * inter * 4, 256) + round_up((size_t)m * hidden * 4, 256);
}

int launch_expert_ffn(const void* w_gate, const void* w_up, const void* w_down, int gate_type, int down_type,
                      int64_t hidden, int64_t inter, const void* x, int x_dtype, int64_t m, float* out, float weight,
                      int accumulate, void* workspace, size_t workspace_bytes, cudaStream_t s) {
    if (m <= 0) return GDN_OK;
    if (workspace_bytes < expert_ffn_workspace_bytes(m, hidden, inter))
        return fail(GDN_ERR_ARG, "expert ffn: workspace of %zu bytes, %zu needed", workspace_bytes,
                    expert_ffn_workspace_bytes(m, hidden, inter));
    uint8_t* p = static_cast<uint8_t*>(workspace);
    const size_t piece = round_up((size_t)m * inter * 4, 256);
    float* g = reinterpret_cast<float*>(p);
    float* u = reinterpret_cast<float*>(p + piece);
    float* a = reinterpret_cast<float*>(p + 2 * piece);
    float* y = reinterpret_cast<float*>(p + 3 * piece);
    int st;
    if ((st = gemv(gate_type, w_gate, inter, hidden, x, x_dtype, m, g, s))) return st;
    if ((st = gemv(gate_type, w_up, inter, hidden, x, x_dtype, m, u, s))) return st;
    const int64_t na = m * inter;
    if ((st = launch_pdl("swiglu_kernel", swiglu_kernel, dim3((unsigned)((na + 255) / 256)), dim3(256), 0, s, g, u, a,
                         na)))
        return st;
    if (!accumulate) return gemv(down_type, w_down, hidden, inter, a, GDN_DTYPE_F32, m, out, s);
    if ((st = gemv(down_type, w_down, hidden, inter, a, GDN_DTYPE_F32, m, y, s))) return st;
    const int64_t ny = m * hidden;
    return launch_pdl("weighted_add_kernel", weighted_add_kernel, dim3((unsigned)((ny + 255) / 256)), dim3(256), 0, s,
                      out, y, weight, ny);
}

}  // namespace gdn
