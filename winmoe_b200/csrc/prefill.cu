// Chunked prefill of the Gated DeltaNet layer: T tokens of one sequence.
//
// The reference has no prefill path: prompt tokens go one at a time through
// deltanet_forward (engine/runtime/winmoe_inference.c:2286-2291 drives
// engine/runtime/deltanet_impl.h:145-377).  This computes the same recurrence
//   S_t = a_t S_{t-1} + k_t d_t^T,  d_t = b_t (v_t - a_t S_{t-1}^T k_t),
//   o_t = S_t^T q_t / sqrt(d)
// chunk by chunk (C = 64 tokens).  With G_i the inclusive cumulative log decay
// inside a chunk, gam_i = exp(G_i), e_i = exp(G_63 - G_i) and
// L[i][j] = b_i exp(G_i - G_j) (k_i . k_j) for j < i, the chunk's deltas are
//   D = U' - W' S0,   (I + L) W' = diag(b gam) K,   (I + L) U' = diag(b) V,
// its outputs
//   O = scale * (diag(gam) Q S0 + P D),   P[i][j] = exp(G_i - G_j) (q_i . k_j), j <= i,
// and the state it hands on
//   S_end = gam_63 S0 + (diag(e) K)^T D.
// Every exponent is a difference G_i - G_j with i >= j (<= 0): no division by
// a cumulative decay.  Log decays are clamped at -110, below which exp() is 0
// in fp32 whatever the rest of the sum, so a decay that underflows to 0 in the
// reference (expf, deltanet_impl.h:251) zeroes the same products here.
//
// Per-element exponentials (the exp(G_i - G_j) factors) use the __expf
// intrinsic, and SiLU (conv output, output gate) one hardware tanh:
// x sigmoid(x) = h + h tanh(h), h = x / 2, absolute error <= 2^-12 |x|.  These
// errors sit below the bf16 / fp16 rounding every one of these values goes
// through next; with IEEE expf and division the output kernel spent ~3/4 of its
// time there, and with exp + divide per SiLU the prep kernel was bound by the
// special-function pipe.
//
// Kernels: prep (conv1d + SiLU + L2 norm, gates and the window hand-off,
// token-parallel), K1 chunk_local (W', U', e*K, cumulative G; (I + L)^-1 by blocked
// fp32 inversion, then W' and U' as tensor-core products), K2 chunk_scan (state passing, sequential over chunks,
// parallel over heads x 16-column slabs), K3 chunk_out (outputs, per-head
// RMSNorm and SiLU(z) gate).  The in/out projections are the tensor-core
// GEMMs of gemm_tc.cu.
#include <algorithm>

#include "gdn_common.cuh"
#include "quant.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "ptx_sm100.cuh"
#include "warp_mma.cuh"
#include "chunk_tc.cuh"

namespace gdn {

using wmma16::bf16;

namespace {

constexpr int HD = 128;                 // head dim
constexpr int CH = 64;                  // chunk length
constexpr float kLogDecayMin = -110.0f;  // exp() of anything <= this is 0 in fp32
constexpr int LDH = HD + 8;             // padded smem row (bf16 elements) of 128-wide tiles

struct PDims {
    int hk, hv, key, inner, qkv;
    int64_t np, ldp, T, Tp, nc;
};

PDims pdims(const gdn_dims& d, int64_t T) {
    PDims r;
    r.hk = d.num_k_heads;
    r.hv = d.num_v_heads;
    r.key = r.hk * HD;
    r.inner = r.hv * HD;
    r.qkv = 2 * r.key + r.inner;
    r.np = (int64_t)r.qkv + r.inner + 2 * r.hv;
    r.ldp = (r.np + 3) / 4 * 4;
    r.T = T;
    r.nc = (T + CH - 1) / CH;
    r.Tp = r.nc * CH;
    return r;
}

struct PWork {
    float* proj;      // [T][ldp] raw projections
    void* xconv;      // [T][hidden] fp16 operand copy of x
    float* partial;   // split-K partials of the gate rows
    size_t partial_bytes;
    bf16 *qn, *kn;    // [Hk][Tp][128] conv'd, SiLU'd, L2-normalised
    bf16* vb;         // [Hv][Tp][128] conv'd, SiLU'd
    float *glog, *beta, *gcum;  // [Hv][Tp]
    float* gchunk;    // [Hv][nc] gam_63 of every chunk
    // per (head, chunk) tile images (img_off): W' [64 t][128 k], E^T [128 k][64 t],
    // U'^T [128 v][64 t] from chunk_local; the chunk's start state S^T [128 v][128 k]
    // and deltas D^T [128 v][64 t] from the scan
    uint8_t *wimg, *eimg, *uimg, *simg, *dimg;
    __half* gated;    // [T][inner] out_proj operand
    float* edge;      // [ceil(T / 128)][6][qkv] raw rows at the M-tile edges (fused preprocessing)
    float* win;       // [4][qkv] raw rows T-4..T-1 (fused preprocessing)
    size_t total;
};

constexpr int kGateSplits = 4;

PWork pcarve(const gdn_dims& d, int64_t T, void* base) {
    const PDims D = pdims(d, T);
    PWork w;
    char* p = static_cast<char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p ? p + off : nullptr;
        off += round_up(bytes, 256);
        return r;
    };
    w.proj = reinterpret_cast<float*>(take((size_t)T * D.ldp * 4));
    w.xconv = take((size_t)T * d.hidden * 2);
    w.partial_bytes = gemm_tc_workspace_bytes(T, 2 * D.hv, kGateSplits);
    w.partial = reinterpret_cast<float*>(take(w.partial_bytes));
    const size_t kv = (size_t)D.Tp * HD * 2;
    w.qn = reinterpret_cast<bf16*>(take(kv * D.hk));
    w.kn = reinterpret_cast<bf16*>(take(kv * D.hk));
    w.vb = reinterpret_cast<bf16*>(take(kv * D.hv));
    w.glog = reinterpret_cast<float*>(take((size_t)D.Tp * D.hv * 4));
    w.beta = reinterpret_cast<float*>(take((size_t)D.Tp * D.hv * 4));
    w.gcum = reinterpret_cast<float*>(take((size_t)D.Tp * D.hv * 4));
    w.gchunk = reinterpret_cast<float*>(take((size_t)D.nc * D.hv * 4));
    const size_t tiles = (size_t)D.nc * D.hv;
    w.wimg = reinterpret_cast<uint8_t*>(take(tiles * chunk_img_w_bytes()));
    w.eimg = reinterpret_cast<uint8_t*>(take(tiles * chunk_img_e_bytes()));
    w.uimg = reinterpret_cast<uint8_t*>(take(tiles * chunk_img_e_bytes()));
    w.simg = reinterpret_cast<uint8_t*>(take(tiles * chunk_img_s_bytes()));
    w.dimg = reinterpret_cast<uint8_t*>(take(tiles * chunk_img_e_bytes()));
    w.gated = reinterpret_cast<__half*>(take((size_t)T * D.inner * 2));
    w.edge = reinterpret_cast<float*>(take((size_t)((T + 127) / 128) * 6 * D.qkv * 4));
    w.win = reinterpret_cast<float*>(take((size_t)4 * D.qkv * 4));
    w.total = off;
    return w;
}

// ------------------------------------------------------------------ prep
//
// One kernel for everything between the input projection and the chunked
// recurrence.  Warps per block of kTokBlock tokens: one per 128-channel chunk
// hc of qkv, plus one gate warp.
//
// Chunk warps: lane l owns channels 4l..4l+3.  All kTokBlock raw projection
// rows are loaded up front (16 loads in flight per lane), then the causal
// conv1d over tokens t-3..t (taps k = 0 oldest .. 3 = t) runs from the last
// token down, in place; tokens before the prompt come from the conv window of
// the state: token -j (j = 1..3) sits in slot (p0 - j) mod 4
// (deltanet_impl.h:220-230).  Then SiLU; q/k chunks are L2-normalised
// (deltanet_impl.h:85-91), the sixteen butterflies interleaved.  The outputs
// are rounded to bf16 next, so the conv taps contract to FMAs and the sum of
// squares is fp32 (the reference's double sum and separate roundings move
// these values by ~1e-7 relative, far below bf16's 2^-9).
// Padding tokens (t >= T) are written as zeros.  The warp of token block 0
// also writes the conv window after the prompt -- slot (p0 + i) mod 4 <- raw
// projection of token i for the last min(T, 4) tokens -- after it has read the
// old window: no other warp touches those channels' window.  (conv_pos is
// advanced by the next kernel, once every warp here has read it.)
//
// Gate warp: lane = value head; per token the log decay log(a) = ssm_a *
// softplus(alpha + dt_bias) with the reference's clamps (a in [0, 1], NaN ->
// 0.99, no ssm_a/dt_bias -> 0.99; deltanet_impl.h:247-257) kept in log space,
// and beta = stable sigmoid (260).
constexpr int kTokBlock = 16;

// Log decay and beta of one (token, head) from its raw projections, with the
// reference's clamps (deltanet_impl.h:247-260) in log space.
__device__ __forceinline__ void gate_values(float beta_raw, float alpha_raw, float sa, float db, bool have_a,
                                            float& gl_out, float& beta_out) {
    float gl = logf(0.99f);
    if (have_a) {
        const float x = alpha_raw + db;
        gl = sa * (log1pf(expf(-fabsf(x))) + fmaxf(x, 0.0f));
        if (isnan(gl)) gl = logf(0.99f);
        gl = fminf(gl, 0.0f);
    }
    gl_out = fmaxf(gl, kLogDecayMin);
    if (beta_raw >= 0.0f) {
        beta_out = 1.0f / (1.0f + expf(-beta_raw));
    } else {
        const float z = expf(beta_raw);
        beta_out = z / (1.0f + z);
    }
}

// Gates of all value heads for tokens tb .. tb + ntok - 1 (one warp; lane = head).
template <int ntok>
__device__ __forceinline__ void gate_block(const float* __restrict__ proj, int64_t ldp, int64_t T, int64_t tb,
                                           int64_t Tp, const float* __restrict__ ssm_a,
                                           const float* __restrict__ dt_bias, float* __restrict__ glog,
                                           float* __restrict__ beta, int qkv, int hv, int lane) {
    const int64_t gate0 = (int64_t)qkv + (int64_t)hv * HD;
    for (int h = lane; h < hv; h += 32) {
        const float sa = ssm_a != nullptr ? ssm_a[h] : 0.0f;
        const float db = dt_bias != nullptr ? dt_bias[h] : 0.0f;
#pragma unroll 4
        for (int64_t t = tb; t < tb + ntok; t++) {
            const int64_t i = (int64_t)h * Tp + t;
            if (t >= T) {
                glog[i] = 0.0f;
                beta[i] = 0.0f;
                continue;
            }
            const float* pr = proj + t * ldp + gate0;
            gate_values(pr[h], pr[hv + h], sa, db, ssm_a != nullptr && dt_bias != nullptr, glog[i], beta[i]);
        }
    }
}


__global__ void __launch_bounds__(256, 2) prefill_prep_kernel(const float* __restrict__ proj, int64_t ldp, int64_t T,
                                                           int64_t Tp, float* __restrict__ conv_buf,
                                                           const int32_t* __restrict__ conv_pos,
                                                           const float* __restrict__ conv_w, bf16* __restrict__ qn,
                                                           bf16* __restrict__ kn, bf16* __restrict__ vb,
                                                           const float* __restrict__ ssm_a,
                                                           const float* __restrict__ dt_bias, float* __restrict__ glog,
                                                           float* __restrict__ beta, int qkv, int hk, int hv) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int nchunk = qkv / HD + 1;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nblk = Tp / kTokBlock;
    if (gw >= nblk * nchunk) return;
    const int hc = (int)(gw % nchunk);
    const int64_t tb = (gw / nchunk) * kTokBlock;

    if (hc == nchunk - 1) {  // ---- gates of all heads for this token block
        gate_block<kTokBlock>(proj, ldp, T, tb, Tp, ssm_a, dt_bias, glog, beta, qkv, hv, lane);
        return;
    }

    bf16* dst;
    if (hc < hk) dst = qn + (int64_t)hc * Tp * HD;
    else if (hc < 2 * hk) dst = kn + (int64_t)(hc - hk) * Tp * HD;
    else dst = vb + (int64_t)(hc - 2 * hk) * Tp * HD;
    dst += 4 * lane;
    const int ch = hc * HD + 4 * lane;
    const bool conv = conv_buf != nullptr && conv_w != nullptr;

    float4 x[kTokBlock];  // raw projections, then (in place) the outputs
#pragma unroll
    for (int j = 0; j < kTokBlock; j++)
        x[j] = tb + j < T ? *reinterpret_cast<const float4*>(proj + (tb + j) * ldp + ch) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (conv) {
        float4 wv[4];
#pragma unroll
        for (int c = 0; c < 4; c++) wv[c] = reinterpret_cast<const float4*>(conv_w)[ch + c];
        float4 hist[3];  // raw projections of tokens tb-3, tb-2, tb-1
        const int p0 = *conv_pos;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            const int64_t tt = tb - 3 + j;
            hist[j] = tt >= 0 ? *reinterpret_cast<const float4*>(proj + tt * ldp + ch)
                              : *reinterpret_cast<const float4*>(conv_buf + (int64_t)((p0 + (int)tt) & 3) * qkv + ch);
        }
        if (tb == 0) {  // the window after the prompt (the old one is read above, in program order)
            for (int64_t i = (T > 4 ? T - 4 : 0); i < T; i++)
                *reinterpret_cast<float4*>(conv_buf + (int64_t)((p0 + (int)i) & 3) * qkv + ch) =
                    *reinterpret_cast<const float4*>(proj + i * ldp + ch);
        }
#pragma unroll
        for (int j = kTokBlock - 1; j >= 0; j--) {  // x[j] needs raw x[j-3..j]: run from the top down
            const float4 r0 = j >= 3 ? x[j - 3] : hist[j];
            const float4 r1 = j >= 2 ? x[j - 2] : hist[j + 1];
            const float4 r2 = j >= 1 ? x[j - 1] : hist[j + 2];
            const float h0[4] = {r0.x, r0.y, r0.z, r0.w}, h1[4] = {r1.x, r1.y, r1.z, r1.w};
            const float h2[4] = {r2.x, r2.y, r2.z, r2.w}, in[4] = {x[j].x, x[j].y, x[j].z, x[j].w};
            float o[4];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float4 w = wv[c];
                float sum = w.x * h0[c];
                sum = fmaf(w.y, h1[c], sum);
                sum = fmaf(w.z, h2[c], sum);
                sum = fmaf(w.w, in[c], sum);
                o[c] = silu_fast(sum);
            }
            x[j] = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
    if (hc < 2 * hk) {
        float ss[kTokBlock];
#pragma unroll
        for (int j = 0; j < kTokBlock; j++)
            ss[j] = fmaf(x[j].x, x[j].x, fmaf(x[j].y, x[j].y, fmaf(x[j].z, x[j].z, x[j].w * x[j].w)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int j = 0; j < kTokBlock; j++) ss[j] += __shfl_xor_sync(0xffffffffu, ss[j], o);
#pragma unroll
        for (int j = 0; j < kTokBlock; j++) {
            // 1 / (sqrt(ss) + 1e-6) (deltanet_impl.h:89): the epsilon shifts the result by
            // 1e-6 / sqrt(ss) relative, so above ss = 1e-4 one rsqrt is as good
            const float inv = inv_l2(ss[j]);
            x[j] = make_float4(x[j].x * inv, x[j].y * inv, x[j].z * inv, x[j].w * inv);
        }
    }
#pragma unroll
    for (int j = 0; j < kTokBlock; j++) {
        const int64_t t = tb + j;
        const uint2 v = t < T ? make_uint2(wmma16::pack_bf16(x[j].x, x[j].y), wmma16::pack_bf16(x[j].z, x[j].w))
                              : make_uint2(0u, 0u);
        *reinterpret_cast<uint2*>(dst + t * HD) = v;
    }
}

// ----------------------------------------------------------------- gates
//
// The gate rows' split-K partials part[z][t][2 Hv] (beta rows, then alpha rows)
// summed in split order -- the additions of splitk_reduce_kernel -- and turned
// into the log decay and beta of every (head, token) at once: thread per
// (token, head), zeros for the padding tokens T .. Tp-1.
__global__ void __launch_bounds__(256) prefill_gate_kernel(const float* __restrict__ part, int splits, int64_t T,
                                                           int64_t Tp, int hv, const float* __restrict__ ssm_a,
                                                           const float* __restrict__ dt_bias,
                                                           float* __restrict__ glog, float* __restrict__ beta) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= Tp * hv) return;
    const int64_t t = i / hv;
    const int h = (int)(i % hv);
    const int64_t o = (int64_t)h * Tp + t;
    if (t >= T) {
        glog[o] = 0.0f;
        beta[o] = 0.0f;
        return;
    }
    const int64_t slice = T * 2 * (int64_t)hv;
    float braw = 0.0f, araw = 0.0f;
    for (int z = 0; z < splits; z++) {
        braw += part[z * slice + t * 2 * hv + h];
        araw += part[z * slice + t * 2 * hv + hv + h];
    }
    const bool have_a = ssm_a != nullptr && dt_bias != nullptr;
    gate_values(braw, araw, have_a ? ssm_a[h] : 0.0f, have_a ? dt_bias[h] : 0.0f, have_a, glog[o], beta[o]);
}

// ----------------------------------------------------------------- edges
//
// The prep kernel's remainder when the input projection's epilogue has done
// conv1d + SiLU + L2 for rows 3.. of every M tile (PrepEpilogue): warps per
// (tile j, 128-channel chunk hc) finish the tile's rows 0..2 -- their conv
// reads the raw rows above them from the previous tile's edge rows, or for
// tile 0 from the conv window of the state -- and the warps of tile 0 then
// write the window after the prompt from `win`; plus one gate warp per
// kGateTok tokens.  Same arithmetic as the prep kernel, row for row.
constexpr int kGateTok = 4;
__global__ void __launch_bounds__(256) prefill_edge_kernel(const float* __restrict__ edge,
                                                           const float* __restrict__ win, int rows, int64_t ntiles,
                                                           const float* __restrict__ proj, int64_t ldp, int64_t T,
                                                           int64_t Tp, float* __restrict__ conv_buf,
                                                           const int32_t* __restrict__ conv_pos,
                                                           const float* __restrict__ conv_w, bf16* __restrict__ qn,
                                                           bf16* __restrict__ kn, bf16* __restrict__ vb,
                                                           const float* __restrict__ ssm_a,
                                                           const float* __restrict__ dt_bias,
                                                           float* __restrict__ glog, float* __restrict__ beta,
                                                           int qkv, int hk, int hv, int with_gates) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int nchunk = qkv / HD;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_gate = with_gates ? Tp / kGateTok : 0;  // gate warps first: theirs is the longest chain
    if (gw < n_gate) {
        gate_block<kGateTok>(proj, ldp, T, gw * kGateTok, Tp, ssm_a, dt_bias, glog, beta, qkv, hv, lane);
        return;
    }
    if (gw >= n_gate + ntiles * nchunk) return;
    const int64_t j = (gw - n_gate) / nchunk;
    const int hc = (int)((gw - n_gate) % nchunk);
    const int ch = hc * HD + 4 * lane;
    const int64_t t0 = j * rows;
    const bool conv = conv_buf != nullptr && conv_w != nullptr;
    float4 x[3], hist[3];
#pragma unroll
    for (int i = 0; i < 3; i++) {
        x[i] = t0 + i < T ? *reinterpret_cast<const float4*>(edge + (j * 6 + i) * qkv + ch) : make_float4(0.f, 0.f, 0.f, 0.f);
        hist[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (conv) {
        const int p0 = *conv_pos;
#pragma unroll
        for (int i = 0; i < 3; i++)
            hist[i] = j > 0 ? *reinterpret_cast<const float4*>(edge + ((j - 1) * 6 + 3 + i) * qkv + ch)
                            : *reinterpret_cast<const float4*>(conv_buf + (int64_t)((p0 + i - 3) & 3) * qkv + ch);
        if (j == 0) {  // the window after the prompt (the old one is read above, in program order)
            for (int64_t i = (T > 4 ? T - 4 : 0); i < T; i++)
                *reinterpret_cast<float4*>(conv_buf + (int64_t)((p0 + (int)i) & 3) * qkv + ch) =
                    *reinterpret_cast<const float4*>(win + (i - (T - 4)) * qkv + ch);
        }
        float4 wv[4];
#pragma unroll
        for (int c = 0; c < 4; c++) wv[c] = reinterpret_cast<const float4*>(conv_w)[ch + c];
        float4 o[3];
#pragma unroll
        for (int i = 0; i < 3; i++) {
            const float4 r0 = i >= 3 ? x[0] : hist[i];
            const float4 r1 = i >= 2 ? x[i - 2] : hist[i + 1];
            const float4 r2 = i >= 1 ? x[i - 1] : hist[i + 2];
            const float h0[4] = {r0.x, r0.y, r0.z, r0.w}, h1[4] = {r1.x, r1.y, r1.z, r1.w};
            const float h2[4] = {r2.x, r2.y, r2.z, r2.w}, in[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float4 w = wv[c];
                float sum = w.x * h0[c];
                sum = fmaf(w.y, h1[c], sum);
                sum = fmaf(w.z, h2[c], sum);
                sum = fmaf(w.w, in[c], sum);
                v[c] = silu_fast(sum);
            }
            o[i] = make_float4(v[0], v[1], v[2], v[3]);
        }
#pragma unroll
        for (int i = 0; i < 3; i++) x[i] = o[i];
    }
    if (hc < 2 * hk) {
#pragma unroll
        for (int i = 0; i < 3; i++) {
            float ss = fmaf(x[i].x, x[i].x, fmaf(x[i].y, x[i].y, fmaf(x[i].z, x[i].z, x[i].w * x[i].w)));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = inv_l2(ss);
            x[i] = make_float4(x[i].x * inv, x[i].y * inv, x[i].z * inv, x[i].w * inv);
        }
    }
    bf16* dst;
    if (hc < hk) dst = qn + (int64_t)hc * Tp * HD;
    else if (hc < 2 * hk) dst = kn + (int64_t)(hc - hk) * Tp * HD;
    else dst = vb + (int64_t)(hc - 2 * hk) * Tp * HD;
    dst += 4 * lane;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int64_t t = t0 + i;
        if (t >= Tp) break;
        const uint2 v = t < T ? make_uint2(wmma16::pack_bf16(x[i].x, x[i].y), wmma16::pack_bf16(x[i].z, x[i].w))
                              : make_uint2(0u, 0u);
        *reinterpret_cast<uint2*>(dst + t * HD) = v;
    }
}

// -------------------------------------------------------- K1: chunk_local
//
// grid (nc, Hv), 256 threads.  L = strictly lower b_i exp(G_i - G_j) K K^T from
// a bf16 tensor-core product; T = (I + L)^-1 blocked by 16 (fp32 substitution
// on the diagonal blocks, hi + lo bf16 MMAs below them); W' = T diag(b gam) K,
// U'^T = (T diag(b) V)^T and E^T = (diag(e) K)^T, staged in shared memory as the
// tile images the tensor-core scan reads (img_off) and written by bulk copies;
// the chunk's cumulative G and gam_63 go to HBM.
struct LocalSmem {
    bf16 k[CH][LDH];
    bf16 v[CH][LDH];
    float L[CH][CH + 1];  // strictly lower part: b_i exp(G_i - G_j) k_i . k_j
    float T[CH][CH + 1];  // (I + L)^-1, unit lower triangular
    float M[4][16][17];   // block products of the inversion stages
    float G[CH], beta[CH];
    float sc[2][CH];      // column scales of T: b_j gam_j (for W') and b_j (for U')
};
// The products leave through shared regions that are dead by then, each
// staged as its 16 KB image: U'^T through V, W' through T, E^T through L.
constexpr uint32_t kImgW = CH * HD * 2, kImgE = HD * CH * 2;
static_assert(sizeof(LocalSmem::v) >= kImgE && sizeof(LocalSmem::T) >= kImgW && sizeof(LocalSmem::L) >= kImgE,
              "images fit their staging regions");
static_assert(offsetof(LocalSmem, v) % 16 == 0 && offsetof(LocalSmem, T) % 16 == 0 &&
              offsetof(LocalSmem, L) % 16 == 0, "bulk sources aligned");

__global__ void __launch_bounds__(256, 3) chunk_local_kernel(const bf16* __restrict__ kn, const bf16* __restrict__ vb,
                                                          const float* __restrict__ glog,
                                                          const float* __restrict__ beta,
                                                          uint8_t* __restrict__ wimg, uint8_t* __restrict__ uimg,
                                                          uint8_t* __restrict__ eimg,
                                                          float* __restrict__ gcum, float* __restrict__ gchunk,
                                                          int64_t Tp, int hk, int hv, int head_map,
                                                          int32_t* __restrict__ conv_pos, int64_t T) {
    pdl_trigger();
    pdl_wait();
    // The prep kernel has read conv_pos and written the new window: advance it.
    if (conv_pos != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *conv_pos += (int32_t)T;
    extern __shared__ uint8_t smem_raw[];
    LocalSmem& sm = *reinterpret_cast<LocalSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int c = blockIdx.x, h = blockIdx.y;
    const int g = head_map ? (h % hk) : (h / (hv / hk));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t t0 = (int64_t)c * CH;
    const bf16* kc = kn + ((int64_t)g * Tp + t0) * HD;
    const bf16* vcg = vb + ((int64_t)h * Tp + t0) * HD;
    for (int i = tid; i < CH * HD / 8; i += 256) {
        const int r = i / (HD / 8), q = i % (HD / 8);
        wmma16::cp_async16(&sm.k[r][q * 8], kc + r * HD + q * 8);
        wmma16::cp_async16(&sm.v[r][q * 8], vcg + r * HD + q * 8);
    }
    wmma16::cp_async_commit();
    if (warp == 0) {  // inclusive cumulative log decay, 2 tokens per lane
        const float* gl = glog + (int64_t)h * Tp + t0;
        const float a = gl[2 * lane], b = gl[2 * lane + 1];
        float s = a + b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        float excl = __shfl_up_sync(0xffffffffu, s, 1);
        if (lane == 0) excl = 0.0f;
        sm.G[2 * lane] = excl + a;
        sm.G[2 * lane + 1] = (excl + a) + b;
    } else if (warp == 1) {
        sm.beta[2 * lane] = beta[(int64_t)h * Tp + t0 + 2 * lane];
        sm.beta[2 * lane + 1] = beta[(int64_t)h * Tp + t0 + 2 * lane + 1];
    }
    wmma16::cp_async_wait<0>();
    __syncthreads();

    // ---- L = mask(b_i exp(G_i - G_j) K K^T), the 20 n8 tiles on or below the
    // diagonal blocks only (nothing reads the upper blocks): warp w takes m tile
    // mt(w) and n8 tiles n0(w) .. n0(w) + cnt(w) - 1 (nibble w of the constants),
    // at most three each -- 3,3,2 of m tile 3, 3,3 of m tile 2, 2,2 of 1, 2 of 0.
    {
        const int mt = (0x01122333 >> (4 * warp)) & 15;
        const int nt0 = (0x02030630 >> (4 * warp)) & 15;
        const int cnt = (0x22233233 >> (4 * warp)) & 15;
        float acc[3][4] = {};
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            uint32_t a[4];
            wmma16::load_a(a, &sm.k[0][0], LDH, 16 * mt, 16 * kk);
#pragma unroll
            for (int pr = 0; pr < 2; pr++) {  // n8 tiles nt0 + 2 pr, nt0 + 2 pr + 1 (within 0..7)
                if (2 * pr >= cnt) break;
                uint32_t b[4];
                wmma16::load_b_nk(b, &sm.k[0][0], LDH, 16 * kk, 8 * (nt0 + 2 * pr));
                wmma16::mma(acc[2 * pr], a, b[0], b[1]);
                if (2 * pr + 1 < cnt) wmma16::mma(acc[2 * pr + 1], a, b[2], b[3]);
            }
        }
        const int gq = lane >> 2, qq = lane & 3;
#pragma unroll
        for (int n = 0; n < 3; n++) {
            if (n >= cnt) break;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = 16 * mt + gq + ((e >> 1) << 3);
                const int j = 8 * (nt0 + n) + 2 * qq + (e & 1);
                sm.L[i][j] = (j < i) ? sm.beta[i] * __expf(sm.G[i] - sm.G[j]) * acc[n][e] : 0.0f;
            }
        }
    }
    __syncthreads();

    // ---- T = (I + L)^-1 (fp32), blocked by 16: the four diagonal blocks by
    // forward substitution (one thread per block column), then the lower
    // off-diagonal blocks through the 2 x 2 split into 32-row halves (below).
    // (T's upper 16-blocks are never read: nothing clears them.)
    if (tid < CH) {
        // column jc of the block's inverse: col[i] = -sum_{kk<i} L_i,kk col[kk], the
        // sums accumulated column-wise (each step's FMAs independent of each
        // other; the same terms in the same order as a row-wise dot product)
        const int o = (tid >> 4) * 16, jc = tid & 15;
        float col[16];
#pragma unroll
        for (int i = 0; i < 16; i++) col[i] = i == jc ? 1.0f : 0.0f;
#pragma unroll
        for (int kk = 0; kk < 15; kk++) {
            if (kk < jc) continue;
            const float ck = col[kk];
#pragma unroll
            for (int i = kk + 1; i < 16; i++) col[i] = fmaf(-sm.L[o + i][o + kk], ck, col[i]);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) sm.T[o + i][o + jc] = col[i];
    } else if (tid < 2 * CH) {
        const int j = tid - CH;
        sm.sc[0][j] = sm.beta[j] * __expf(sm.G[j]);
        sm.sc[1][j] = sm.beta[j];
    }
    __syncthreads();
    // Off-diagonal blocks on the tensor cores, one warp per output block: each
    // 16x16x16 product takes its fp32 operands as hi + lo bf16 pairs (three MMAs:
    // hi.hi + hi.lo + lo.hi, relative error ~2^-17 -- T then enters W' and U' as a
    // 16-bit hi + lo pair itself).  Fragments follow the m16n8k16 layout.
    {
        const int gq = lane >> 2, qq = lane & 3;
        auto split2 = [](float x0, float x1, uint32_t& hi, uint32_t& lo) {
            const bf16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
            hi = wmma16::pack_bf16(__bfloat162float(h0), __bfloat162float(h1));
            lo = wmma16::pack_bf16(x0 - __bfloat162float(h0), x1 - __bfloat162float(h1));
        };
        // A: rows r0..r0+15, cols c0..c0+15 of a row-major fp32 tile (pitch ld)
        auto frag_a = [&](const float* X, int ld, int r0, int c0, uint32_t (&hi)[4], uint32_t (&lo)[4]) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float* p = X + (r0 + gq + 8 * (i & 1)) * ld + c0 + 2 * qq + 8 * (i >> 1);
                split2(p[0], p[1], hi[i], lo[i]);
            }
        };
        // B (16 x 8): B[k][n] = X[k0 + k][n0 + n]
        auto frag_b = [&](const float* X, int ld, int k0, int n0, uint32_t (&hi)[2], uint32_t (&lo)[2]) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const float* p = X + (k0 + 2 * qq + 8 * i) * ld + n0 + gq;
                split2(p[0], p[ld], hi[i], lo[i]);
            }
        };
        auto mma3 = [](float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], const uint32_t (&bh)[2],
                       const uint32_t (&bl)[2]) {
            wmma16::mma(c, ah, bh[0], bh[1]);
            wmma16::mma(c, ah, bl[0], bl[1]);
            wmma16::mma(c, al, bh[0], bh[1]);
        };
        // T as 2 x 2 blocks of 32: [[A, 0], [C, B]]^-1 = [[A^-1, 0], [-B^-1 C A^-1, B^-1]].
        // Stage 1 completes A^-1 and B^-1 (blocks (1,0) and (3,2), one warp each);
        // stage 2 forms X = C A^-1 (four warps, into M); stage 3 T_C = -B^-1 X (four
        // warps).  Dependent chains of two block products per stage.
        auto store_m = [&](int idx, const float (&m)[2][4]) {
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                sm.M[idx][gq][8 * nt + 2 * qq] = m[nt][0];
                sm.M[idx][gq][8 * nt + 2 * qq + 1] = m[nt][1];
                sm.M[idx][gq + 8][8 * nt + 2 * qq] = m[nt][2];
                sm.M[idx][gq + 8][8 * nt + 2 * qq + 1] = m[nt][3];
            }
        };
        auto store_t_neg = [&](int bi, int bj, const float (&t)[2][4]) {
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                sm.T[16 * bi + gq][16 * bj + 8 * nt + 2 * qq] = -t[nt][0];
                sm.T[16 * bi + gq][16 * bj + 8 * nt + 2 * qq + 1] = -t[nt][1];
                sm.T[16 * bi + gq + 8][16 * bj + 8 * nt + 2 * qq] = -t[nt][2];
                sm.T[16 * bi + gq + 8][16 * bj + 8 * nt + 2 * qq + 1] = -t[nt][3];
            }
        };
        // the block product acc += X1[r1 / 16, c1 / 16] X2[k0 / 16, n0 / 16] (16 x 16 x 16)
        auto block_mma = [&](float (&acc)[2][4], const float* X1, int ld1, int r1, int c1, const float* X2, int ld2,
                             int k0, int n0) {
            uint32_t ah[4], al[4];
            frag_a(X1, ld1, r1, c1, ah, al);
#pragma unroll
            for (int nt = 0; nt < 2; nt++) {
                uint32_t bh[2], bl[2];
                frag_b(X2, ld2, k0, n0 + 8 * nt, bh, bl);
                mma3(acc[nt], ah, al, bh, bl);
            }
        };
        const float* Lp = &sm.L[0][0];
        const float* Tp_ = &sm.T[0][0];
        if (warp < 2) {  // T_{bi,bj} = -T_{bi,bi} L_{bi,bj} T_{bj,bj}, (bi, bj) = (1,0), (3,2)
            const int bi = 2 * warp + 1, bj = 2 * warp;
            float m[2][4] = {};
            block_mma(m, Lp, CH + 1, 16 * bi, 16 * bj, Tp_, CH + 1, 16 * bj, 16 * bj);
            store_m(warp, m);
            __syncwarp();
            float t[2][4] = {};
            block_mma(t, Tp_, CH + 1, 16 * bi, 16 * bi, &sm.M[warp][0][0], 17, 0, 0);
            store_t_neg(bi, bj, t);
        }
        __syncthreads();
        const int xi = 2 + (warp >> 1), xj = warp & 1;
        if (warp < 4) {  // X_{i,j} = sum_{k=j}^{1} L_{i,k} T_{k,j} -> M[warp]
            float m[2][4] = {};
            for (int k = xj; k < 2; k++) block_mma(m, Lp, CH + 1, 16 * xi, 16 * k, Tp_, CH + 1, 16 * k, 16 * xj);
            store_m(warp, m);
        }
        __syncthreads();
        if (warp < 4) {  // T_{i,j} = -sum_{k=2}^{i} T_{i,k} X_{k,j}
            float t[2][4] = {};
            for (int k = 2; k <= xi; k++)
                block_mma(t, Tp_, CH + 1, 16 * xi, 16 * k, &sm.M[2 * (k - 2) + xj][0][0], 17, 0, 0);
            store_t_neg(xi, xj, t);
        }
        __syncthreads();
    }

    // ---- U' = (T diag(b)) V, then W' = (T diag(b gam)) K, on the tensor cores:
    // V and K exact bf16; the scaled T enters as hi + lo bf16 fragments built in
    // registers from the fp32 T (register i: row gq + 8 (i & 1), columns
    // 2 qq + 8 (i >> 1) + {0, 1}).  T is block lower triangular, so row block rb
    // takes k-blocks 0..rb only.  Each result is staged as its tile image in a
    // shared region that is dead by then and leaves as one bulk copy: U'^T
    // through V, W' through T (E^T follows, through L).
    {
        const int gq = lane >> 2, qq = lane & 3;
        const int rb = warp & 3, r0 = 16 * rb, n0 = 64 * (warp >> 2);
        float acc[8][4];
        auto product = [&](const bf16* rhs, const float* scale) {
#pragma unroll
            for (int n = 0; n < 8; n++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[n][e] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < CH / 16; kk++) {
                if (kk > rb) break;
                uint32_t ah[4], al[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int row = r0 + gq + 8 * (i & 1), col = 16 * kk + 2 * qq + 8 * (i >> 1);
                    const float x0 = sm.T[row][col] * scale[col];
                    const float x1 = sm.T[row][col + 1] * scale[col + 1];
                    const bf16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
                    ah[i] = wmma16::pack_bf16(__bfloat162float(h0), __bfloat162float(h1));
                    al[i] = wmma16::pack_bf16(x0 - __bfloat162float(h0), x1 - __bfloat162float(h1));
                }
#pragma unroll
                for (int np2 = 0; np2 < 4; np2++) {
                    uint32_t b[4];
                    wmma16::load_b_kn(b, rhs, LDH, 16 * kk, n0 + 16 * np2);
                    wmma16::mma(acc[2 * np2], ah, b[0], b[1]);
                    wmma16::mma(acc[2 * np2 + 1], ah, b[2], b[3]);
                    wmma16::mma(acc[2 * np2], al, b[0], b[1]);
                    wmma16::mma(acc[2 * np2 + 1], al, b[2], b[3]);
                }
            }
        };
        product(&sm.v[0][0], sm.sc[1]);
        __syncthreads();  // V read by every warp: U'^T takes its place (rows v, as the scan reads it)
        uint8_t* ustage = reinterpret_cast<uint8_t*>(&sm.v[0][0]);
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const int cl = n0 + 8 * n + 2 * qq;
#pragma unroll
            for (int e = 0; e < 4; e++)
                *reinterpret_cast<bf16*>(ustage + sm100::img_off(HD, cl + (e & 1), r0 + gq + 8 * (e >> 1))) =
                    __float2bfloat16_rn(acc[n][e]);
        }
        sm100::fence_proxy_async_smem();  // the staged U'^T leaves by bulk copy
        product(&sm.k[0][0], sm.sc[0]);
        __syncthreads();  // T and K read by every warp: W' takes T's place
        if (tid == 0)  // U'^T is complete: its copy runs while W' and E^T are staged
            sm100::bulk_store(uimg + ((int64_t)h * (Tp / CH) + c) * kImgE, sm100::smem_u32(&sm.v[0][0]), kImgE);
        uint8_t* wstage = reinterpret_cast<uint8_t*>(&sm.T[0][0]);
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const int cl = n0 + 8 * n + 2 * qq;
            *reinterpret_cast<uint32_t*>(wstage + sm100::img_off(CH, r0 + gq, cl)) =
                wmma16::pack_bf16(acc[n][0], acc[n][1]);
            *reinterpret_cast<uint32_t*>(wstage + sm100::img_off(CH, r0 + gq + 8, cl)) =
                wmma16::pack_bf16(acc[n][2], acc[n][3]);
        }
    }

    // ---- E^T [k][t] = e_t K[t][k], e_t = exp(G_63 - G_t), into its image in L's place
    // (L is dead since the inversion): thread per (k, 8 tokens), consecutive
    // threads consecutive k -- conflict-free column reads of K
    const float G63 = sm.G[CH - 1];
    uint8_t* estage = reinterpret_cast<uint8_t*>(&sm.L[0][0]);
    for (int e = tid; e < HD * (CH / 8); e += 256) {
        const int kc = e % HD, j = e / HD;
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = __expf(G63 - sm.G[8 * j + i]) * __bfloat162float(sm.k[8 * j + i][kc]);
        *reinterpret_cast<uint4*>(estage + sm100::img_off(HD, kc, 8 * j)) =
            make_uint4(wmma16::pack_bf16(f[0], f[1]), wmma16::pack_bf16(f[2], f[3]), wmma16::pack_bf16(f[4], f[5]),
                       wmma16::pack_bf16(f[6], f[7]));
    }
    if (tid < CH) gcum[(int64_t)h * Tp + t0 + tid] = sm.G[tid];
    if (tid == 0) gchunk[(int64_t)h * (Tp / CH) + c] = expf(G63);
    sm100::fence_proxy_async_smem();  // the staged tiles, written by the generic proxy, leave by bulk copy
    __syncthreads();
    if (tid == 0) {
        const int64_t i = (int64_t)h * (Tp / CH) + c;
        sm100::bulk_store(wimg + i * kImgW, sm100::smem_u32(&sm.T[0][0]), kImgW);
        sm100::bulk_store(eimg + i * kImgE, sm100::smem_u32(&sm.L[0][0]), kImgE);
        sm100::bulk_commit();
        sm100::bulk_wait_read_all();
    }
}

template <typename K>
int set_smem(K kern, size_t bytes) {
    GDN_CUDA(cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return GDN_OK;
}

}  // namespace

size_t prefill_workspace_bytes(const gdn_dims& d, int64_t T) { return pcarve(d, T, nullptr).total; }

// A highest-priority stream per host thread and device, with fork / join events.
// The prefill's input projection (hundreds of one-per-SM CTAs, a partly empty
// last wave) runs there; the gate rows, on the caller's stream meanwhile, get
// only the SMs it leaves idle -- its last wave -- instead of running after it.
// The decode step's input projection does the same.
int side_stream(SideStream** out) {
    thread_local SideStream tls[16];
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 16) return fail(GDN_ERR_CUDA, "device index %d out of range", dev);
    SideStream& r = tls[dev];
    if (r.s == nullptr) {
        int least = 0, greatest = 0;
        GDN_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
        GDN_CUDA(cudaEventCreateWithFlags(&r.fork, cudaEventDisableTiming));
        GDN_CUDA(cudaEventCreateWithFlags(&r.join, cudaEventDisableTiming));
        GDN_CUDA(cudaStreamCreateWithPriority(&r.s, cudaStreamNonBlocking, greatest));
    }
    *out = &r;
    return GDN_OK;
}

int prefill(const gdn_layer* L, int64_t T, const void* x, int x_dtype, float* out, const RowDest* gated_out,
            float* S, float* conv_buf, int32_t* conv_pos, void* wsp, size_t ws_bytes, cudaStream_t s) {
    int st = validate_layer(L);
    if (st) return st;
    if (T <= 0 || T > (int64_t)1 << 26) return fail(GDN_ERR_SHAPE, "T must be in [1, 2^26] (got %lld)", (long long)T);
    if (!x || (!out && !gated_out) || !S || !conv_pos)
        return fail(GDN_ERR_ARG, "x, the output, S and conv_pos must be non-NULL");
    if (x_dtype != GDN_DTYPE_F32 && x_dtype != GDN_DTYPE_BF16 && x_dtype != GDN_DTYPE_F16)
        return fail(GDN_ERR_TYPE, "x_dtype %d is not supported", x_dtype);
    if ((out && !aligned(out, 16)) || !aligned(S, 16))
        return fail(GDN_ERR_ARG, "the output and S must be 16-byte aligned");
    const gdn_dims& d = L->dims;
    if (gated_out) {
        const RowDest& g = *gated_out;
        if (g.n < 1 || g.n > kMaxRowDest || g.rows < 1 || g.rows * g.n != T || g.col0 < 0 ||
            g.ld < g.col0 + (int64_t)d.num_v_heads * 128 || (g.ld | g.col0) % 2 != 0)
            return fail(GDN_ERR_SHAPE, "gated destinations: %d x %lld rows must cover T=%lld, pitch %lld >= "
                        "column %lld + %lld, both even", g.n, (long long)g.rows, (long long)T, (long long)g.ld,
                        (long long)g.col0, (long long)d.num_v_heads * 128);
        for (int r = 0; r < g.n; r++)
            if (!aligned(g.ptr[r], 16)) return fail(GDN_ERR_ARG, "gated destination %d is NULL or misaligned", r);
    }
    const size_t need = prefill_workspace_bytes(d, T);
    if (wsp == nullptr || ws_bytes < need || !aligned(wsp, 256))
        return fail(GDN_ERR_ARG, "workspace must be 256-aligned and hold %zu bytes (got %zu)", need, ws_bytes);
    const PDims D = pdims(d, T);
    const PWork W = pcarve(d, T, wsp);
    const bool conv = (L->conv1d_w != nullptr && conv_buf != nullptr);
    const int64_t hidden = d.hidden;

    // ---- input projection -> proj [T][ldp]
    if ((st = phase_mark(0, s))) return st;
    PrepEpilogue prep;  // Q8_0: the preprocessing runs in the projection's epilogue
    bool gates_done = false;
    if (L->weight_type == GDN_GGML_Q4_K) {
        if (T >= 8 && x_dtype != GDN_DTYPE_F32) {  // tensor cores, exact weights, fp16 x (bf16 converts exactly)
            const void* a = x;
            if (x_dtype != GDN_DTYPE_F16 || !aligned(x, 16)) {
                if ((st = launch_convert(x, x_dtype, W.xconv, false, T * hidden, s))) return st;
                a = W.xconv;
            }
            st = launch_q4_k_gemm_tc(L->in_blocks, D.np, hidden, a, T, W.proj, D.ldp, TcOptions(), s);
        } else {
            st = launch_q4_k_gemv(L->in_blocks, D.np, hidden, x, x_dtype, T, W.proj, D.ldp, s);
        }
        if (st) return st;
    } else {
        const void* a = x;
        if (x_dtype != GDN_DTYPE_F16 || !aligned(x, 16)) {
            if ((st = launch_convert(x, x_dtype, W.xconv, false, T * hidden, s))) return st;
            a = W.xconv;
        }
        const int64_t n_main = (int64_t)D.qkv + D.inner;
        TcOptions fast;  // q, k, v, z rows: one fp16 weight operand; conv1d, SiLU, L2 in its epilogue
        prep.enabled = 1;
        prep.qkv = D.qkv;
        prep.hk = D.hk;
        prep.T = T;
        prep.Tp = D.Tp;
        prep.conv_w = conv ? L->conv1d_w : nullptr;
        prep.qn = W.qn;
        prep.kn = W.kn;
        prep.vb = W.vb;
        prep.edge = W.edge;
        prep.win = W.win;
        fast.prep = &prep;
        SideStream* side = nullptr;
        if ((st = side_stream(&side))) return st;
        GDN_CUDA(cudaEventRecord(side->fork, s));
        GDN_CUDA(cudaStreamWaitEvent(side->s, side->fork, 0));
        st = launch_q8_0_gemm_tc(L->in_qs, L->in_d, n_main, hidden, a, false, T, W.proj, D.ldp, fast, side->s);
        GDN_CUDA(cudaEventRecord(side->join, side->s));
        if (st) {
            (void)cudaStreamWaitEvent(s, side->join, 0);
            return st;
        }
        const int8_t* gq = L->in_qs + n_main * hidden;
        const uint16_t* gd = L->in_d + n_main * (hidden / 32);
        if (x_dtype == GDN_DTYPE_F32) {
            // the fp16 copy of fp32 x is rounded: the gate rows stay on fp32 CUDA cores
            st = launch_q8_0_gemv(gq, gd, 2 * D.hv, hidden, x, x_dtype, T, W.proj + n_main, D.ldp, s);
        } else {
            // beta/alpha rows: exact hi + lo weights (exp(ssm_a * softplus(alpha)) is sensitive);
            // their partials summed straight into the gates, still beside the projection's last wave
            TcOptions exact;
            exact.split_precision = true;
            exact.splits = kGateSplits;
            exact.workspace = W.partial;
            exact.workspace_bytes = W.partial_bytes;
            exact.partials_only = true;
            int used = 0;
            exact.splits_used = &used;
            st = launch_q8_0_gemm_tc(gq, gd, 2 * D.hv, hidden, a, false, T, W.partial, 2 * D.hv, exact, s);
            if (!st) {
                const int64_t n = D.Tp * D.hv;
                st = launch_pdl("prefill_gate_kernel", prefill_gate_kernel, dim3((unsigned)((n + 255) / 256)),
                                dim3(256), 0, s, (const float*)W.partial, used, T, D.Tp, D.hv, L->ssm_a, L->dt_bias,
                                W.glog, W.beta);
                gates_done = true;
            }
        }
        const cudaError_t ej = cudaStreamWaitEvent(s, side->join, 0);  // joined on every path
        if (st) return st;
        if (ej != cudaSuccess) return cuda_status(ej, "prefill: join of the input projection");
    }

    // ---- conv1d + SiLU + L2 norm, gates, window hand-off
    if ((st = phase_mark(1, s))) return st;
    if (prep.enabled) {
        const int64_t ntiles = (T + prep.rows - 1) / prep.rows;
        const int64_t warps = ntiles * (D.qkv / HD) + (gates_done ? 0 : D.Tp / kGateTok);
        st = launch_pdl("prefill_edge_kernel", prefill_edge_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s,
                        (const float*)W.edge, (const float*)W.win, prep.rows, ntiles, (const float*)W.proj, D.ldp, T,
                        D.Tp, conv ? conv_buf : nullptr, (const int32_t*)conv_pos, conv ? L->conv1d_w : nullptr,
                        W.qn, W.kn, W.vb, L->ssm_a, L->dt_bias, W.glog, W.beta, D.qkv, D.hk, D.hv,
                        gates_done ? 0 : 1);
        if (st) return st;
    } else {
        const int64_t warps = (D.Tp / kTokBlock) * (D.qkv / HD + 1);
        st = launch_pdl("prefill_prep_kernel", prefill_prep_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0,
                        s, W.proj, D.ldp, T, D.Tp, conv ? conv_buf : nullptr, conv_pos,
                        conv ? L->conv1d_w : nullptr, W.qn, W.kn, W.vb, L->ssm_a, L->dt_bias, W.glog, W.beta, D.qkv,
                        D.hk, D.hv);
        if (st) return st;
    }

    // ---- chunked recurrence
    if ((st = phase_mark(2, s))) return st;
    {
        const size_t sm1 = sizeof(LocalSmem) + 128;
        if ((st = set_smem(chunk_local_kernel, sm1))) return st;
        st = launch_pdl("chunk_local_kernel", chunk_local_kernel, dim3((unsigned)D.nc, (unsigned)D.hv), dim3(256),
                        sm1, s, W.kn, W.vb, W.glog, W.beta, W.wimg, W.uimg, W.eimg, W.gcum, W.gchunk, D.Tp, D.hk,
                        D.hv, L->head_map, conv ? conv_pos : nullptr, T);
        if (st) return st;
        if ((st = launch_chunk_scan_tc(W.wimg, W.eimg, W.uimg, W.gchunk, S, W.simg, W.dimg, D.hv, D.nc, s))) return st;
        st = launch_chunk_out_tc(W.qn, W.kn, W.simg, W.dimg, W.gcum, W.proj, D.ldp, L->head_norm,
                                 gated_out ? nullptr : W.gated, gated_out ? *gated_out : RowDest{}, T, D.Tp, D.hk,
                                 D.hv, D.qkv, L->head_map, s);
        if (st) return st;
    }

    // ---- output projection (the caller takes the gated heads instead when it shards them)
    if ((st = phase_mark(3, s))) return st;
    if (gated_out) return phase_mark(4, s);
    if (L->weight_type == GDN_GGML_Q4_K) {
        if (T >= 8)  // the fp16 gated heads on the tensor cores, exact weights
            st = launch_q4_k_gemm_tc(L->out_blocks, hidden, D.inner, W.gated, T, out, hidden, TcOptions(), s);
        else
            st = launch_q4_k_gemv(L->out_blocks, hidden, D.inner, W.gated, GDN_DTYPE_F16, T, out, hidden, s);
    } else if (T >= 64) {
        TcOptions fast;
        st = launch_q8_0_gemm_tc(L->out_qs, L->out_d, hidden, D.inner, W.gated, false, T, out, hidden, fast, s);
    } else {
        st = launch_q8_0_gemv(L->out_qs, L->out_d, hidden, D.inner, W.gated, GDN_DTYPE_F16, T, out, hidden, s);
    }
    if (st) return st;
    return phase_mark(4, s);
}

}  // namespace gdn
