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

struct ExpertWeights {
    float w[kMaxExpertsPerCall];
};

// out[j][i] (+)= sum_e w_e * y[j][e * hidden + i], the experts in order.
__global__ void experts_sum_kernel(const float* __restrict__ y, float* __restrict__ out, ExpertWeights wts, int ne,
                                   int64_t hidden, int64_t total, int accumulate) {
    pdl_trigger();
    pdl_wait();
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const int64_t j = t / hidden, i = t - j * hidden;
    const float* yr = y + j * ne * hidden + i;
    float acc = accumulate ? out[t] : 0.0f;
    for (int e = 0; e < ne; e++) acc = fmaf(wts.w[e], yr[(int64_t)e * hidden], acc);
    out[t] = acc;
}

}  // namespace

size_t experts_ffn_workspace_bytes(int n_experts, int64_t m, int64_t hidden, int64_t inter) {
    // [m][n_experts][gate | up] and, with more than one expert, [m][n_experts][hidden], fp32
    const size_t gu = round_up((size_t)m * n_experts * 2 * inter * 4, 256);
    return n_experts > 1 ? gu + round_up((size_t)m * n_experts * hidden * 4, 256) : gu;
}

// out = sum_e weight_e * y_e, or with accumulate out += sum_e weight_e * y_e
// (weights NULL: all 1).  One expert: two launches -- gate and up as one
// streamed GEMV over both matrices (rows written as [m][gate | up]), then the
// down projection, whose activation staging forms (g * sigmoid(g)) * u and
// whose output is weight * y, stored or added.  n experts: three launches -- the gate and
// up rows of all of them as one GEMV over 2 n matrices, the n down projections
// as one GEMV over n matrices (each reading its expert's [gate | up] slice,
// each expert's result in its own columns), then their weighted sum in expert
// order.
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
    if (ne == 1) {
        dn.accumulate = accumulate;
        dn.alpha = weights ? weights[0] : 1.0f;
        st = launch_gemv_stream(fmt_of(down_type), w_down[0], nullptr, hidden, inter, gu, GDN_DTYPE_F32, m, out,
                                hidden, s, dn);
        return st < 0 ? fail(st, "expert ffn: down projection (inter %lld)", (long long)inter) : st;
    }
    float* yd = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         round_up((size_t)m * ne * 2 * inter * 4, 256));
    dn.nseg = ne;
    dn.seg_rows = hidden;
    dn.x_seg = 2 * inter;
    dn.ldx = 2 * ne * inter;
    for (int e = 0; e < ne; e++) dn.seg[e] = static_cast<const uint8_t*>(w_down[e]);
    st = launch_gemv_stream(fmt_of(down_type), w_down[0], nullptr, ne * hidden, inter, gu, GDN_DTYPE_F32, m, yd,
                            ne * hidden, s, dn);
    if (st) return st < 0 ? fail(st, "expert ffn: down projections (inter %lld)", (long long)inter) : st;
    ExpertWeights wts;
    for (int e = 0; e < kMaxExpertsPerCall; e++) wts.w[e] = e < ne ? (weights ? weights[e] : 1.0f) : 0.0f;
    const int64_t total = m * hidden;
    return launch_pdl("experts_sum_kernel", experts_sum_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, s,
                      (const float*)yd, out, wts, ne, hidden, total, accumulate);
}

}  // namespace gdn
