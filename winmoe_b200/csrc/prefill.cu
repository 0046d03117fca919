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

namespace gdn {

using wmma16::bf16;

namespace {

constexpr int HD = 128;                 // head dim
constexpr int CH = 64;                  // chunk length
constexpr int BV = 16;                  // state columns per scan CTA
constexpr float kLogDecayMin = -110.0f;  // exp() of anything <= this is 0 in fp32
constexpr int LDH = HD + 8;             // padded smem row (bf16 elements) of 128-wide tiles
constexpr int LDV = BV + 8;             // ... of BV-wide tiles

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
    bf16 *wp, *ek;    // [Hv][Tp][LDH] W', e*K, rows padded as the scan's shared-memory tiles
    bf16* up;         // [Hv][nc][128 / BV][CH][LDV] U', one padded tile per chunk and slab
    bf16* sc;         // [Hv][nc][128][128] state at each chunk start
    bf16* dl;         // [Hv][Tp][128] chunk deltas D
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
    w.wp = reinterpret_cast<bf16*>(take((size_t)D.Tp * LDH * 2 * D.hv));
    w.up = reinterpret_cast<bf16*>(take((size_t)D.nc * (HD / BV) * CH * LDV * 2 * D.hv));
    w.ek = reinterpret_cast<bf16*>(take((size_t)D.Tp * LDH * 2 * D.hv));
    w.sc = reinterpret_cast<bf16*>(take((size_t)D.nc * D.hv * HD * HD * 2));
    w.dl = reinterpret_cast<bf16*>(take(kv * D.hv));
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
// U' = T diag(b) V and e*K, staged in shared memory in the scan's tile layouts
// and written by bulk copies; the chunk's cumulative G and gam_63 go to HBM.
struct LocalSmem {
    bf16 k[CH][LDH];
    bf16 v[CH][LDH];
    float L[CH][CH + 1];  // strictly lower part: b_i exp(G_i - G_j) k_i . k_j
    float T[CH][CH + 1];  // (I + L)^-1, unit lower triangular
    float M[4][16][17];   // block products of the inversion stages
    float G[CH], beta[CH];
    float sc[2][CH];      // column scales of T: b_j gam_j (for W') and b_j (for U')
};
// The products leave through shared regions that are dead by then: U' through
// V + L, W' through T + M (each staged in its HBM layout).
static_assert(offsetof(LocalSmem, L) == offsetof(LocalSmem, v) + sizeof(LocalSmem::v), "V, L adjacent");
static_assert(offsetof(LocalSmem, M) == offsetof(LocalSmem, T) + sizeof(LocalSmem::T), "T, M adjacent");
static_assert(sizeof(LocalSmem::v) + sizeof(LocalSmem::L) >= (HD / BV) * CH * LDV * 2, "U' staging fits");
static_assert(sizeof(LocalSmem::T) + sizeof(LocalSmem::M) >= CH * LDH * 2, "W' staging fits");
static_assert(offsetof(LocalSmem, v) % 16 == 0 && offsetof(LocalSmem, T) % 16 == 0, "bulk sources aligned");

__global__ void __launch_bounds__(256, 3) chunk_local_kernel(const bf16* __restrict__ kn, const bf16* __restrict__ vb,
                                                          const float* __restrict__ glog,
                                                          const float* __restrict__ beta, bf16* __restrict__ wp,
                                                          bf16* __restrict__ up, bf16* __restrict__ ek,
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
    // takes k-blocks 0..rb only.  Each result is staged in its HBM layout in a
    // shared region that is dead by then and leaves as one bulk copy: U' through
    // V + L (slab-major [HD / BV][CH][LDV]), W' through T + M ([CH][LDH]), e*K
    // in place in the K tile.
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
        __syncthreads();  // V (and L) read by every warp: U' takes their place
        bf16* ustage = &sm.v[0][0];
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const int cl = n0 + 8 * n + 2 * qq;
            bf16* d0 = ustage + (cl / BV) * (CH * LDV) + cl % BV;
            *reinterpret_cast<uint32_t*>(d0 + (r0 + gq) * LDV) = wmma16::pack_bf16(acc[n][0], acc[n][1]);
            *reinterpret_cast<uint32_t*>(d0 + (r0 + gq + 8) * LDV) = wmma16::pack_bf16(acc[n][2], acc[n][3]);
        }
        sm100::fence_proxy_async_smem();  // the staged U' leaves by bulk copy
        product(&sm.k[0][0], sm.sc[0]);
        __syncthreads();  // T and K read by every warp: W' takes T's place, e*K K's
        if (tid == 0)  // U' is complete: its copy runs while W' and e*K are staged
            sm100::bulk_store(up + ((int64_t)h * (Tp / CH) + c) * (HD / BV) * (CH * LDV),
                              sm100::smem_u32(&sm.v[0][0]), (HD / BV) * CH * LDV * 2);
        bf16* wstage = reinterpret_cast<bf16*>(&sm.T[0][0]);
#pragma unroll
        for (int n = 0; n < 8; n++) {
            bf16* d0 = wstage + n0 + 8 * n + 2 * qq;
            *reinterpret_cast<uint32_t*>(d0 + (r0 + gq) * LDH) = wmma16::pack_bf16(acc[n][0], acc[n][1]);
            *reinterpret_cast<uint32_t*>(d0 + (r0 + gq + 8) * LDH) = wmma16::pack_bf16(acc[n][2], acc[n][3]);
        }
    }

    // ---- e K with e_i = exp(G_63 - G_i), 8 bf16 per thread, in place
    const float G63 = sm.G[CH - 1];
    for (int e = tid; e < CH * HD / 8; e += 256) {
        const int i = e / (HD / 8), c8 = (e % (HD / 8)) * 8;
        const float ei = __expf(G63 - sm.G[i]);
        uint4* p = reinterpret_cast<uint4*>(&sm.k[i][c8]);
        const uint4 kv = *p;
        const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
        uint32_t ow[4];
#pragma unroll
        for (int w4 = 0; w4 < 4; w4++) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kw[w4]));
            ow[w4] = wmma16::pack_bf16(ei * f.x, ei * f.y);
        }
        *p = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    if (tid < CH) gcum[(int64_t)h * Tp + t0 + tid] = sm.G[tid];
    if (tid == 0) gchunk[(int64_t)h * (Tp / CH) + c] = expf(G63);
    sm100::fence_proxy_async_smem();  // the staged tiles, written by the generic proxy, leave by bulk copy
    __syncthreads();
    if (tid == 0) {
        sm100::bulk_store(wp + ((int64_t)h * Tp + t0) * LDH, sm100::smem_u32(&sm.T[0][0]), CH * LDH * 2);
        sm100::bulk_store(ek + ((int64_t)h * Tp + t0) * LDH, sm100::smem_u32(&sm.k[0][0]), CH * LDH * 2);
        sm100::bulk_commit();
        sm100::bulk_wait_read_all();
    }
}

// --------------------------------------------------------- K2: chunk_scan
//
// grid (128 / BV, Hv), 128 threads; sequential over the chunks of the prompt.
// The state slab S[:, BV columns] lives in fp32 mma accumulators (warp w owns
// key rows 32w..32w+31).  Per chunk: S -> bf16 (smem, and HBM as the chunk's
// start state), D = U' - W' S (warp w: token rows 16w..16w+15), then
// S = gam_63 S + (e K)^T D.  The next chunk's W', e*K and U' stream in (three
// bulk copies, one mbarrier per buffer) while this one is computed; the stores
// of the start state and the deltas are issued behind this chunk's MMAs, off
// the chain of dependent steps.
constexpr int kMaxChunksInSmem = 2048;  // per-chunk decays staged in smem (T up to 128K tokens)

struct ScanSmem {
    bf16 w[2][CH][LDH];
    bf16 e[2][CH][LDH];
    bf16 u[2][CH][LDV];
    bf16 s[HD][LDV];
    bf16 d[CH][LDV];
    float gc[kMaxChunksInSmem];
    uint64_t full[2];  // one mbarrier per buffer: the chunk's three bulk copies landed
};
constexpr uint32_t kScanWBytes = CH * LDH * 2, kScanUBytes = CH * LDV * 2;

__global__ void __launch_bounds__(128) chunk_scan_kernel(const bf16* __restrict__ wp, const bf16* __restrict__ up,
                                                         const bf16* __restrict__ ek,
                                                         const float* __restrict__ gchunk, float* __restrict__ S,
                                                         bf16* __restrict__ sc, bf16* __restrict__ dl, int64_t Tp,
                                                         int64_t nc, uint32_t* __restrict__ err) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    ScanSmem& sm = *reinterpret_cast<ScanSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int slab = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, qq = lane & 3;
    const int v0 = slab * BV;
    float* Sh = S + (int64_t)h * HD * HD;

    // state slab -> accumulators: acc[mt][n][e] = S[32w + 16mt + gq + 8(e>>1)][v0 + 8n + 2qq + (e&1)]
    float acc[2][BV / 8][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int n = 0; n < BV / 8; n++)
#pragma unroll
            for (int e = 0; e < 4; e++)
                acc[mt][n][e] =
                    Sh[(int64_t)(32 * warp + 16 * mt + gq + ((e >> 1) << 3)) * HD + v0 + 8 * n + 2 * qq + (e & 1)];

    // The chunk's W', e*K and U' slab are stored in global memory exactly as the
    // padded shared-memory tiles: one thread brings them with three bulk copies.
    auto prefetch = [&](int64_t c, int buf) {
        const uint32_t bar = sm100::smem_u32(&sm.full[buf]);
        const int64_t base = ((int64_t)h * Tp + c * CH) * LDH;
        sm100::mbar_arrive_expect_tx(bar, 2 * kScanWBytes + kScanUBytes);
        sm100::bulk_load(sm100::smem_u32(&sm.w[buf][0][0]), wp + base, kScanWBytes, bar);
        sm100::bulk_load(sm100::smem_u32(&sm.e[buf][0][0]), ek + base, kScanWBytes, bar);
        sm100::bulk_load(sm100::smem_u32(&sm.u[buf][0][0]), up + ((h * nc + c) * (HD / BV) + slab) * (CH * LDV),
                         kScanUBytes, bar);
    };
    if (tid == 0) {
        sm100::mbar_init(sm100::smem_u32(&sm.full[0]), 1);
        sm100::mbar_init(sm100::smem_u32(&sm.full[1]), 1);
        sm100::fence_barrier_init();
        prefetch(0, 0);
    }
    const bool gc_smem = nc <= kMaxChunksInSmem;
    if (gc_smem)
        for (int64_t i = tid; i < nc; i += 128) sm.gc[i] = gchunk[(int64_t)h * nc + i];
    __syncthreads();  // barriers initialised, decays staged

    for (int64_t c = 0; c < nc; c++) {
        const int buf = (int)(c & 1);
        // ---- chunk start state: bf16 copy in smem (B operand) and in HBM (for the output kernel)
        bf16* scc = sc + (((int64_t)h * nc + c) * HD) * HD;
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int n = 0; n < BV / 8; n++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int r = 32 * warp + 16 * mt + gq + 8 * hf;
                    const int cl = 8 * n + 2 * qq;
                    *reinterpret_cast<uint32_t*>(&sm.s[r][cl]) =
                        wmma16::pack_bf16(acc[mt][n][2 * hf], acc[mt][n][2 * hf + 1]);
                }
        // buf ^ 1 was last read in the previous chunk, before its closing barrier
        if (tid == 0 && c + 1 < nc) prefetch(c + 1, buf ^ 1);
        const bool landed = sm100::mbar_wait(sm100::smem_u32(&sm.full[buf]), (uint32_t)((c >> 1) & 1), err);
        if (!__syncthreads_and(landed)) {  // timed out (error word set): stop, let the copies drain
            if (c + 1 < nc) sm100::mbar_wait(sm100::smem_u32(&sm.full[buf ^ 1]), (uint32_t)(((c + 1) >> 1) & 1), err);
            return;
        }

        // ---- D = U' - W' S   (token rows 16w..16w+15, all BV columns)
        float dacc[BV / 8][4] = {};
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            uint32_t a[4];
            wmma16::load_a(a, &sm.w[buf][0][0], LDH, 16 * warp, 16 * kk);
#pragma unroll
            for (int np2 = 0; np2 < BV / 16; np2++) {
                uint32_t b[4];
                wmma16::load_b_kn(b, &sm.s[0][0], LDV, 16 * kk, 16 * np2);
                wmma16::mma(dacc[2 * np2], a, b[0], b[1]);
                wmma16::mma(dacc[2 * np2 + 1], a, b[2], b[3]);
            }
        }
        // chunk start state -> HBM (16-byte stores issued behind the MMAs above; sm.s
        // is next written after this chunk's last barrier)
        for (int i = tid; i < HD * BV / 8; i += 128) {
            const int r = i / (BV / 8), q = i % (BV / 8);
            *reinterpret_cast<uint4*>(scc + (int64_t)r * HD + v0 + q * 8) = *reinterpret_cast<const uint4*>(&sm.s[r][q * 8]);
        }
        bf16* dlc = dl + ((int64_t)h * Tp + c * CH) * HD + v0;
#pragma unroll
        for (int n = 0; n < BV / 8; n++)
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                const int r = 16 * warp + gq + 8 * hf;
                const int cl = 8 * n + 2 * qq;
                const __nv_bfloat162 u2 = *reinterpret_cast<const __nv_bfloat162*>(&sm.u[buf][r][cl]);
                const float2 uf = __bfloat1622float2(u2);
                *reinterpret_cast<uint32_t*>(&sm.d[r][cl]) =
                    wmma16::pack_bf16(uf.x - dacc[n][2 * hf], uf.y - dacc[n][2 * hf + 1]);
            }
        __syncthreads();

        // ---- S = gam_63 S + (e K)^T D   (key rows 32w..32w+31)
        const float gC = gc_smem ? sm.gc[c] : gchunk[(int64_t)h * nc + c];
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int n = 0; n < BV / 8; n++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[mt][n][e] *= gC;
#pragma unroll
        for (int kk = 0; kk < CH / 16; kk++) {
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                uint32_t a[4];
                wmma16::load_a_t(a, &sm.e[buf][0][0], LDH, 32 * warp + 16 * mt, 16 * kk);
#pragma unroll
                for (int np2 = 0; np2 < BV / 16; np2++) {
                    uint32_t b[4];
                    wmma16::load_b_kn(b, &sm.d[0][0], LDV, 16 * kk, 16 * np2);
                    wmma16::mma(acc[mt][2 * np2], a, b[0], b[1]);
                    wmma16::mma(acc[mt][2 * np2 + 1], a, b[2], b[3]);
                }
            }
        }
        for (int i = tid; i < CH * BV / 8; i += 128) {  // deltas -> HBM, behind the MMAs above
            const int r = i / (BV / 8), q = i % (BV / 8);
            *reinterpret_cast<uint4*>(dlc + (int64_t)r * HD + q * 8) = *reinterpret_cast<const uint4*>(&sm.d[r][q * 8]);
        }
        // sm.s, sm.d and this buffer are rewritten next chunk, the buffer by a bulk
        // copy (async proxy): order this thread's reads of it before that
        sm100::fence_proxy_async_smem();
        __syncthreads();
    }
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int n = 0; n < BV / 8; n++)
#pragma unroll
            for (int e = 0; e < 4; e++)
                Sh[(int64_t)(32 * warp + 16 * mt + gq + ((e >> 1) << 3)) * HD + v0 + 8 * n + 2 * qq + (e & 1)] =
                    acc[mt][n][e];
}

// ---------------------------------------------------------- K3: chunk_out
//
// grid (nc, Hv), 128 threads; warp w owns token rows 16w..16w+15 of the chunk.
//   P = mask(exp(G_i - G_j) Q K^T)                      (bf16, smem)
//   O = scale * (diag(gam) Q S0 + P D)                   (fp32 accumulators)
// then per token: RMSNorm over the head's 128 values times the norm weight
// (deltanet_impl.h:350-361) and the SiLU(z) gate (364-371) -> fp16 out_proj operand.
struct OutSmem {
    bf16 q[CH][LDH];
    bf16 kd[CH][LDH];  // K for P, then the chunk's deltas D
    bf16 s[HD][LDH];
    float G[CH];
    float hn[HD];
};

__global__ void __launch_bounds__(128, 3) chunk_out_kernel(const bf16* __restrict__ qn, const bf16* __restrict__ kn,
                                                        const bf16* __restrict__ sc, const bf16* __restrict__ dl,
                                                        const float* __restrict__ gcum,
                                                        const float* __restrict__ proj, int64_t ldp,
                                                        const float* __restrict__ head_norm,
                                                        __half* __restrict__ gated, const RowDest dst,
                                                        int64_t T, int64_t Tp, int hk,
                                                        int hv, int qkv, int head_map) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    OutSmem& sm = *reinterpret_cast<OutSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int c = blockIdx.x, h = blockIdx.y;
    const int g = head_map ? (h % hk) : (h / (hv / hk));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, qq = lane & 3;
    const int64_t t0 = (int64_t)c * CH;
    const int64_t nc = Tp / CH;
    {
        const bf16* qc = qn + ((int64_t)g * Tp + t0) * HD;
        const bf16* kc = kn + ((int64_t)g * Tp + t0) * HD;
        const bf16* s0 = sc + (((int64_t)h * nc + c) * HD) * HD;
        for (int i = tid; i < CH * HD / 8; i += 128) {
            const int r = i / (HD / 8), q = i % (HD / 8);
            wmma16::cp_async16(&sm.q[r][q * 8], qc + r * HD + q * 8);
            wmma16::cp_async16(&sm.kd[r][q * 8], kc + r * HD + q * 8);
        }
        for (int i = tid; i < HD * HD / 8; i += 128) {
            const int r = i / (HD / 8), q = i % (HD / 8);
            wmma16::cp_async16(&sm.s[r][q * 8], s0 + r * HD + q * 8);
        }
        wmma16::cp_async_commit();
        if (tid < CH) sm.G[tid] = gcum[(int64_t)h * Tp + t0 + tid];
        sm.hn[tid] = head_norm != nullptr ? head_norm[tid] : 1.0f;
    }
    const int rA = 16 * warp + gq, rB = rA + 8;  // this thread's two token rows
    // The gate inputs z of this thread's two rows and 32 columns, fetched now so
    // the loads are in flight during the products below.
    float2 zr[2][HD / 8];
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        const int64_t t = t0 + (hf ? rB : rA);
        const float* z = proj + min(t, T - 1) * ldp + qkv + h * HD;
#pragma unroll
        for (int n = 0; n < HD / 8; n++) zr[hf][n] = *reinterpret_cast<const float2*>(z + 8 * n + 2 * qq);
    }
    wmma16::cp_async_wait<0>();
    __syncthreads();
    // ---- P = mask(exp(G_i - G_j) Q K^T), only this warp's rows, kept in registers
    // as the A fragments of P D: the accumulators of n-tiles 2kk and 2kk+1 are,
    // packed to bf16, the m16k16 fragment of k-block kk.
    uint32_t pa[CH / 16][4];
    {
        float pacc[CH / 8][4] = {};
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            uint32_t a[4];
            wmma16::load_a(a, &sm.q[0][0], LDH, 16 * warp, 16 * kk);
#pragma unroll
            for (int np2 = 0; np2 < CH / 16; np2++) {
                uint32_t b[4];
                wmma16::load_b_nk(b, &sm.kd[0][0], LDH, 16 * kk, 16 * np2);
                wmma16::mma(pacc[2 * np2], a, b[0], b[1]);
                wmma16::mma(pacc[2 * np2 + 1], a, b[2], b[3]);
            }
        }
#pragma unroll
        for (int n = 0; n < CH / 8; n++) {
            const int j = 8 * n + 2 * qq;
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = (e >> 1) ? rB : rA, jj = j + (e & 1);
                v[e] = (jj <= i) ? __expf(sm.G[i] - sm.G[jj]) * pacc[n][e] : 0.0f;
            }
            pa[n >> 1][2 * (n & 1)] = wmma16::pack_bf16(v[0], v[1]);
            pa[n >> 1][2 * (n & 1) + 1] = wmma16::pack_bf16(v[2], v[3]);
        }
    }
    __syncthreads();  // every warp is done with K: the deltas take its place, loaded behind Q S0
    {
        const bf16* dc = dl + ((int64_t)h * Tp + t0) * HD;
        for (int i = tid; i < CH * HD / 8; i += 128) {
            const int r = i / (HD / 8), q = i % (HD / 8);
            wmma16::cp_async16(&sm.kd[r][q * 8], dc + r * HD + q * 8);
        }
        wmma16::cp_async_commit();
    }
    // ---- O = diag(gam) Q S0 + P D
    float o[HD / 8][4] = {};
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++) {
        uint32_t a[4];
        wmma16::load_a(a, &sm.q[0][0], LDH, 16 * warp, 16 * kk);
#pragma unroll
        for (int np2 = 0; np2 < HD / 16; np2++) {
            uint32_t b[4];
            wmma16::load_b_kn(b, &sm.s[0][0], LDH, 16 * kk, 16 * np2);
            wmma16::mma(o[2 * np2], a, b[0], b[1]);
            wmma16::mma(o[2 * np2 + 1], a, b[2], b[3]);
        }
    }
    const float gamA = expf(sm.G[rA]), gamB = expf(sm.G[rB]);
#pragma unroll
    for (int n = 0; n < HD / 8; n++) {
        o[n][0] *= gamA;
        o[n][1] *= gamA;
        o[n][2] *= gamB;
        o[n][3] *= gamB;
    }
    wmma16::cp_async_wait<0>();
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < CH / 16; kk++) {
#pragma unroll
        for (int np2 = 0; np2 < HD / 16; np2++) {
            uint32_t b[4];
            wmma16::load_b_kn(b, &sm.kd[0][0], LDH, 16 * kk, 16 * np2);
            wmma16::mma(o[2 * np2], pa[kk], b[0], b[1]);
            wmma16::mma(o[2 * np2 + 1], pa[kk], b[2], b[3]);
        }
    }
    // ---- scale, per-token RMSNorm over the head, SiLU(z) gate
    const float scale = 1.0f / sqrtf((float)HD);
    double ssA = 0.0, ssB = 0.0;
#pragma unroll
    for (int n = 0; n < HD / 8; n++) {
#pragma unroll
        for (int e = 0; e < 4; e++) o[n][e] = __fmul_rn(o[n][e], scale);
        ssA += (double)o[n][0] * o[n][0] + (double)o[n][1] * o[n][1];
        ssB += (double)o[n][2] * o[n][2] + (double)o[n][3] * o[n][3];
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        ssA += __shfl_xor_sync(0xffffffffu, ssA, off);
        ssB += __shfl_xor_sync(0xffffffffu, ssB, off);
    }
    const float invA = 1.0f / sqrtf((float)(ssA / HD) + 1e-6f);
    const float invB = 1.0f / sqrtf((float)(ssB / HD) + 1e-6f);
    const int inner = hv * HD;
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        const int64_t t = t0 + (hf ? rB : rA);
        if (t >= T) continue;
        const float inv = hf ? invB : invA;
        __half* gout = (gated != nullptr ? gated + t * inner : dst.row<__half>(t)) + h * HD;
#pragma unroll
        for (int n = 0; n < HD / 8; n++) {
            const int v = 8 * n + 2 * qq;
            const float2 zz = zr[hf][n];
            float r2[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                float nv = __fmul_rn(o[n][2 * hf + e], inv);
                if (head_norm != nullptr) nv = __fmul_rn(nv, sm.hn[v + e]);
                float zv = e ? zz.y : zz.x;
                zv = fminf(fmaxf(zv, -88.0f), 88.0f);
                r2[e] = __fmul_rn(nv, silu_fast(zv));
            }
            *reinterpret_cast<__half2*>(gout + v) = __floats2half2_rn(r2[0], r2[1]);
        }
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
                        sm1, s, W.kn, W.vb, W.glog, W.beta, W.wp, W.up, W.ek, W.gcum, W.gchunk, D.Tp, D.hk, D.hv,
                        L->head_map, conv ? conv_pos : nullptr, T);
        if (st) return st;
        const size_t sm2 = sizeof(ScanSmem) + 128;
        if ((st = set_smem(chunk_scan_kernel, sm2))) return st;
        st = launch_pdl("chunk_scan_kernel", chunk_scan_kernel, dim3(HD / BV, (unsigned)D.hv), dim3(128), sm2, s,
                        W.wp, W.up, W.ek, W.gchunk, S, W.sc, W.dl, D.Tp, D.nc, device_error_word());
        if (st) return st;
        const size_t sm3 = sizeof(OutSmem) + 128;
        if ((st = set_smem(chunk_out_kernel, sm3))) return st;
        st = launch_pdl("chunk_out_kernel", chunk_out_kernel, dim3((unsigned)D.nc, (unsigned)D.hv), dim3(128), sm3, s,
                        W.qn, W.kn, W.sc, W.dl, W.gcum, W.proj, D.ldp, L->head_norm,
                        gated_out ? nullptr : W.gated, gated_out ? *gated_out : RowDest{}, T, D.Tp, D.hk, D.hv,
                        D.qkv, L->head_map);
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
