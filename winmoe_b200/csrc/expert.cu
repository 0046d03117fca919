// The expert FFN of the MoE layers on the device (the fused GPU route of the
// reference, engine/runtime/gpu_offload.cu:718-751, gpu_expert_ffn_fused, and
// its batched accumulation, :766-793): for m tokens,
//     g = W_gate x, u = W_up x            (hidden -> inter, Q4_K or Q5_K)
//     a = (g * sigmoid(g)) * u            (swiglu_kernel, :460-466)
//     y = W_down a                        (inter -> hidden, Q4_K or Q5_K)
//     out = y, or out += weight * y       (weighted_add_kernel, :469-471)
// The projections are the streamed GEMVs of gemv_stream.cu (fp32 arithmetic up
// to summation order, as the reference's fp32-activation GPU kernels), with the
// SwiGLU and the weighted accumulation folded into the down projection; the
// expert cache that owns the weights stays the reference's.
#include "gdn_common.cuh"
#include "quant.cuh"

namespace gdn {
namespace {

int fmt_of(int type) { return type == GDN_GGML_Q4_K ? 1 : 2; }

}  // namespace

size_t expert_ffn_workspace_bytes(int64_t m, int64_t hidden, int64_t inter) {
    (void)hidden;
    return round_up((size_t)m * 2 * inter * 4, 256);  // [m][gate | up] fp32
}

// Two launches: gate and up as one streamed GEMV over both matrices (half the
// CTAs each, rows written as [m][gate | up]), then the down projection, whose
// activation staging forms (g * sigmoid(g)) * u from those rows and whose
// output is stored or, accumulating, added as weight * y.
int launch_expert_ffn(const void* w_gate, const void* w_up, const void* w_down, int gate_type, int down_type,
                      int64_t hidden, int64_t inter, const void* x, int x_dtype, int64_t m, float* out, float weight,
                      int accumulate, void* workspace, size_t workspace_bytes, cudaStream_t s) {
    if (m <= 0) return GDN_OK;
    if (workspace_bytes < expert_ffn_workspace_bytes(m, hidden, inter))
        return fail(GDN_ERR_ARG, "expert ffn: workspace of %zu bytes, %zu needed", workspace_bytes,
                    expert_ffn_workspace_bytes(m, hidden, inter));
    float* gu = static_cast<float*>(workspace);
    GemvOpts both;
    both.wq2 = static_cast<const uint8_t*>(w_up);
    both.n1 = inter;
    int st = launch_gemv_stream(fmt_of(gate_type), w_gate, nullptr, 2 * inter, hidden, x, x_dtype, m, gu, 2 * inter, s,
                                both);
    if (st) return st < 0 ? fail(st, "expert ffn: gate / up projection (hidden %lld)", (long long)hidden) : st;
    GemvOpts down;
    down.swiglu = 1;
    down.accumulate = accumulate;
    down.alpha = weight;
    st = launch_gemv_stream(fmt_of(down_type), w_down, nullptr, hidden, inter, gu, GDN_DTYPE_F32, m, out, hidden, s,
                            down);
    return st < 0 ? fail(st, "expert ffn: down projection (inter %lld)", (long long)inter) : st;
}

}  // namespace gdn
