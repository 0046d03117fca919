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

size_t experts_ffn_workspace_bytes(int n_experts, int64_t m, int64_t hidden, int64_t inter) {
    (void)hidden;
    return round_up((size_t)m * n_experts * 2 * inter * 4, 256);  // [m][n_experts][gate | up] fp32
}

// out = sum_e weight_e * y_e, or with accumulate out += sum_e weight_e * y_e
// (weights NULL: all 1), in two launches: the gate and up rows of every expert
// as one streamed GEMV over a table of 2 n matrices (rows written as
// [m][e][gate | up]), then the down projections of all experts as one GEMV
// along a k axis of n inter values -- the experts' down matrices side by side,
// expert e's inputs its SwiGLU (g * sigmoid(g)) * u times weight_e -- which
// forms the weighted sum in its own accumulators.  One expert: the weight
// scales the output instead (out = weight y, or out += weight y).
int launch_experts_ffn(int ne, const void* const* w_gate, const void* const* w_up, const void* const* w_down,
                       int gate_type, int down_type, int64_t hidden, int64_t inter, const void* x, int x_dtype,
                       int64_t m, const float* weights, float* out, int accumulate, void* workspace,
                       size_t workspace_bytes, cudaStream_t s) {
    if (m <= 0 || ne <= 0) return GDN_OK;
    if (ne > kMaxExpertsPerCall) return fail(GDN_ERR_ARG, "experts ffn: at most %d experts per call", kMaxExpertsPerCall);
    if (workspace_bytes < experts_ffn_workspace_bytes(ne, m, hidden, inter))
        return fail(GDN_ERR_ARG, "expert ffn: workspace of %zu bytes, %zu needed", workspace_bytes,
                    experts_ffn_workspace_bytes(ne, m, hidden, inter));
    float* gu = static_cast<float*>(workspace);
    GemvOpts up;
    up.nseg = 2 * ne;
    up.seg_rows = inter;
    for (int e = 0; e < ne; e++) {
        up.seg[2 * e] = static_cast<const uint8_t*>(w_gate[e]);
        up.seg[2 * e + 1] = static_cast<const uint8_t*>(w_up[e]);
    }
    int st = launch_gemv_stream(fmt_of(gate_type), w_gate[0], nullptr, 2 * ne * inter, hidden, x, x_dtype, m, gu,
                                2 * ne * inter, s, up);
    if (st) return st < 0 ? fail(st, "expert ffn: gate / up projections (hidden %lld)", (long long)hidden) : st;
    GemvOpts dn;
    dn.swiglu = 1;
    dn.accumulate = accumulate;
    if (ne == 1) {
        dn.alpha = weights ? weights[0] : 1.0f;
    } else {
        dn.kseg = ne;
        for (int e = 0; e < ne; e++) {
            dn.seg[e] = static_cast<const uint8_t*>(w_down[e]);
            dn.kscale[e] = weights ? weights[e] : 1.0f;
        }
    }
    st = launch_gemv_stream(fmt_of(down_type), w_down[0], nullptr, hidden, ne * inter, gu, GDN_DTYPE_F32, m, out,
                            hidden, s, dn);
    return st < 0 ? fail(st, "expert ffn: down projection (inter %lld)", (long long)inter) : st;
}

}  // namespace gdn
