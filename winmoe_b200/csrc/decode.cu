// Decode step of the Gated DeltaNet layer for a batch of independent sequences.
//
//   proj  = in_proj(x)                   [B][QKV | inner | Hv (beta) | Hv (alpha)]
//   state : conv1d window + SiLU, L2-norm of q/k, decay/beta gates, then
//           S <- decay*S; r = S^T k; delta = beta (v - r); S += k delta^T;
//           o = S^T q / sqrt(d); per-head RMSNorm * w; * SiLU(z)  -> gated
//   out   = out_proj(gated)
//
// Reference: deltanet_forward, engine/runtime/deltanet_impl.h:145-377
// (conv 218-236, gates 247-261, L2 264-267, recurrence 279-348, norm 350-361,
// gate 364-371, out_proj 374).
//
// Kernels per step: the input projection (tensor-core GEMM for B >= 64,
// CUDA-core GEMV below), gdn_prep_kernel (conv1d, SiLU, L2 norms, gates),
// gdn_state_kernel (recurrence, RMSNorm, output gate), out_proj.
// The state kernel is the HBM-bound part: every (sequence, value head) owns a
// 128x128 fp32 state (64 KiB) that is read once and written once per token.
#include <algorithm>

#include "gdn_common.cuh"
#include "ptx_sm100.cuh"
#include "quant.cuh"
#include "decode.cuh"
#include "prefill.cuh"

namespace gdn {

constexpr int HD = 128;  // head_dim (the reference's AVX loops assume 128 too)

// -------------------------------------------------------------- prep kernel
//
// One warp per (sequence b, 128-channel chunk hc of the qkv vector): chunk hc
// is q head hc (hc < Hk), k head hc-Hk (hc < 2Hk) or v head hc-2Hk.  Lane l
// owns channels 4l..4l+3 (16-byte loads and stores):
//   window slot p%4 <- raw projection; out = sum_k w[c][k] * window[(p+1-4+k)%4]
//   (k = 0 oldest, k = 3 the value just stored), then SiLU (deltanet_impl.h:218-236);
//   q/k heads are L2-normalised with a double-precision sum (85-91, 264-267).
// One extra warp per sequence (hc = QKV/128) computes the gates of all heads
// (247-261) into gates[b][h] = {decay, beta, 0, 0}.
__global__ void __launch_bounds__(256) gdn_prep_kernel(const float* __restrict__ proj, int64_t np,
                                                       float* __restrict__ act, float4* __restrict__ gates,
                                                       float* __restrict__ conv_buf,
                                                       const int32_t* __restrict__ conv_pos,
                                                       const float* __restrict__ conv_w,
                                                       const float* __restrict__ ssm_a,
                                                       const float* __restrict__ dt_bias, int64_t B, int qkv,
                                                       int key_dim, int hv) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int nchunk = qkv / HD + 1;
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (gw >= B * nchunk) return;
    const int64_t b = gw / nchunk;
    const int hc = (int)(gw % nchunk);
    const float* pr = proj + b * np;
    if (hc == nchunk - 1) {
        const int inner = hv * HD;
        for (int h = lane; h < hv; h += 32) {
            const float beta_raw = pr[qkv + inner + h];
            const float alpha_raw = pr[qkv + inner + hv + h];
            float a = 0.99f;
            if (ssm_a != nullptr && dt_bias != nullptr) {
                const float x = alpha_raw + dt_bias[h];
                const float sp = log1pf(expf(-fabsf(x))) + fmaxf(x, 0.0f);
                a = expf(ssm_a[h] * sp);
            }
            a = (a > 1.0f) ? 1.0f : a;
            a = (a < 0.0f) ? 0.0f : a;
            if (isnan(a)) a = 0.99f;
            float bt;
            if (beta_raw >= 0.0f) {
                bt = 1.0f / (1.0f + expf(-beta_raw));
            } else {
                const float z = expf(beta_raw);
                bt = z / (1.0f + z);
            }
            gates[b * hv + h] = make_float4(a, bt, 0.0f, 0.0f);
        }
        return;
    }
    const int ch = hc * HD + 4 * lane;
    float4 xv = *reinterpret_cast<const float4*>(pr + ch);
    if (conv_buf != nullptr && conv_w != nullptr) {
        const int p = conv_pos[b];
        float* win = conv_buf + b * 4 * (int64_t)qkv;
        const float4 o0 = *reinterpret_cast<const float4*>(win + (int64_t)((p - 3) & 3) * qkv + ch);
        const float4 o1 = *reinterpret_cast<const float4*>(win + (int64_t)((p - 2) & 3) * qkv + ch);
        const float4 o2 = *reinterpret_cast<const float4*>(win + (int64_t)((p - 1) & 3) * qkv + ch);
        *reinterpret_cast<float4*>(win + (int64_t)(p & 3) * qkv + ch) = xv;
        const float4* wv = reinterpret_cast<const float4*>(conv_w) + ch;  // 4 channels x 4 taps
        float in[4] = {xv.x, xv.y, xv.z, xv.w};
        const float h0[4] = {o0.x, o0.y, o0.z, o0.w}, h1[4] = {o1.x, o1.y, o1.z, o1.w};
        const float h2[4] = {o2.x, o2.y, o2.z, o2.w};
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const float4 w = wv[c];
            float sum = 0.0f;
            sum = __fadd_rn(sum, __fmul_rn(w.x, h0[c]));
            sum = __fadd_rn(sum, __fmul_rn(w.y, h1[c]));
            sum = __fadd_rn(sum, __fmul_rn(w.z, h2[c]));
            sum = __fadd_rn(sum, __fmul_rn(w.w, in[c]));
            const float sig = 1.0f / (1.0f + expf(-sum));
            in[c] = __fmul_rn(sum, sig);
        }
        xv = make_float4(in[0], in[1], in[2], in[3]);
    }
    if (ch < 2 * key_dim) {
        double ss = (double)xv.x * xv.x + (double)xv.y * xv.y + (double)xv.z * xv.z + (double)xv.w * xv.w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / (sqrtf((float)ss) + 1e-6f);
        xv = make_float4(__fmul_rn(xv.x, inv), __fmul_rn(xv.y, inv), __fmul_rn(xv.z, inv), __fmul_rn(xv.w, inv));
    }
    *reinterpret_cast<float4*>(act + b * qkv + ch) = xv;
}

// ------------------------------------------------------------- state kernel
//
// Persistent: one CTA (256 threads) per SM walks a contiguous range of tiles
// (sequence b, value head h).  Everything a tile reads -- its 64 KiB fp32
// state, the conv'd q and k of its key group, v and z of head h, and its
// gates -- is brought into a kStateBufs-deep shared-memory ring by
// cp.async.bulk with one mbarrier per slot, so the loop itself issues no
// global loads and HBM always has the next tiles in flight.  The updated
// state goes back to HBM with coalesced 16-byte stores straight from
// registers.  Recurrence: warp w owns state rows [16w, 16w+16), lane l
// columns [4l, 4l+4) (16 float4 registers per thread; one warp access = one
// 512-byte row).  The CTA holding head 0 of sequence b advances conv_pos[b]
// (the prep kernel, which read it, has finished).
constexpr int kStateBufs = 3;
constexpr int kTileFloats = HD * HD;
constexpr uint32_t kTileBytes = kTileFloats * 4;
constexpr uint32_t kVecBytes = HD * 4;

struct StateSlot {
    float S[kTileFloats];
    float q[HD], k[HD], v[HD], z[HD];
    float4 gate;
};

struct StateSmem {
    StateSlot slot[kStateBufs];
    float red[8][HD];   // retrieve partials, one row per warp
    float red2[8][HD];  // output partials
    uint64_t full[kStateBufs];
};

__global__ void __launch_bounds__(256, 1) gdn_state_kernel(
    const float* __restrict__ act, const float4* __restrict__ gates, const float* __restrict__ proj, int64_t np,
    float* __restrict__ S, const float* __restrict__ head_norm, float* __restrict__ gated,
    __half* __restrict__ gated_h, int32_t* __restrict__ conv_pos, int qkv, int key_dim, int hv, int hk,
    int head_map, int64_t n_tiles, int64_t tiles_per_cta, uint32_t* __restrict__ err) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    StateSmem& sm = *reinterpret_cast<StateSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int t = threadIdx.x, w = t >> 5, l = t & 31;
    const int hpg = hv / hk;
    const int inner = hv * HD;
    const int64_t first = (int64_t)blockIdx.x * tiles_per_cta;
    const int64_t last = min(first + tiles_per_cta, n_tiles);
    const int count = (int)max((int64_t)0, last - first);

    // tile -> (b, h); tiles run over the heads of a sequence in order
    auto issue = [&](int i) {
        const int64_t tile = first + i;
        const int64_t b = tile / hv;
        const int h = (int)(tile % hv);
        const int g = head_map ? (h % hk) : (h / hpg);
        StateSlot& sl = sm.slot[i % kStateBufs];
        const uint32_t bar = sm100::smem_u32(&sm.full[i % kStateBufs]);
        const float* a = act + b * qkv;
        sm100::mbar_arrive_expect_tx(bar, kTileBytes + 4 * kVecBytes + 16);
        sm100::bulk_load(sm100::smem_u32(sl.S), S + (b * hv + h) * (int64_t)kTileFloats, kTileBytes, bar);
        sm100::bulk_load(sm100::smem_u32(sl.q), a + g * HD, kVecBytes, bar);
        sm100::bulk_load(sm100::smem_u32(sl.k), a + key_dim + g * HD, kVecBytes, bar);
        sm100::bulk_load(sm100::smem_u32(sl.v), a + 2 * key_dim + h * HD, kVecBytes, bar);
        sm100::bulk_load(sm100::smem_u32(sl.z), proj + b * np + qkv + h * HD, kVecBytes, bar);
        sm100::bulk_load(sm100::smem_u32(&sl.gate), gates + b * hv + h, 16, bar);
    };

    if (t == 0) {
        for (int i = 0; i < kStateBufs; i++) sm100::mbar_init(sm100::smem_u32(&sm.full[i]), 1);
        sm100::fence_barrier_init();
        for (int i = 0; i < kStateBufs && i < count; i++) issue(i);
    }
    __syncthreads();

    // Lane l owns value columns 4l..4l+3; warp w owns key rows 16w..16w+15.  Per
    // tile two block barriers: (A) after the retrieve partials, from which every
    // thread forms the delta of its own columns, and (B) after the output partials,
    // from which every warp forms the whole output row (the RMSNorm needs all 128).
    const float4 hn = head_norm != nullptr ? reinterpret_cast<const float4*>(head_norm)[l]
                                           : make_float4(1.f, 1.f, 1.f, 1.f);
    for (int i = 0; i < count; i++) {
        const int64_t tile = first + i;
        const int64_t b = tile / hv;
        const int h = (int)(tile % hv);
        StateSlot& sl = sm.slot[i % kStateBufs];
        const bool landed =
            sm100::mbar_wait(sm100::smem_u32(&sm.full[i % kStateBufs]), (uint32_t)((i / kStateBufs) & 1), err);
        const float4* Sv = reinterpret_cast<const float4*>(sl.S);
        float4 s[16];
#pragma unroll
        for (int r = 0; r < 16; r++) s[r] = Sv[(16 * w + r) * (HD / 4) + l];
        const float dg = sl.gate.x, bt = sl.gate.y;
        const float4 vv = reinterpret_cast<const float4*>(sl.v)[l];
        const float4 zz = reinterpret_cast<const float4*>(sl.z)[l];
        float kr[16], qr[16];
#pragma unroll
        for (int r = 0; r < 16; r += 4) {
            const float4 k4 = reinterpret_cast<const float4*>(sl.k + 16 * w)[r / 4];
            const float4 q4 = reinterpret_cast<const float4*>(sl.q + 16 * w)[r / 4];
            kr[r] = k4.x; kr[r + 1] = k4.y; kr[r + 2] = k4.z; kr[r + 3] = k4.w;
            qr[r] = q4.x; qr[r + 1] = q4.y; qr[r + 2] = q4.z; qr[r + 3] = q4.w;
        }

        // ---- decay + retrieve (deltanet_impl.h:298-307)
        float4 rp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < 16; r++) {
            s[r].x = __fmul_rn(s[r].x, dg);
            s[r].y = __fmul_rn(s[r].y, dg);
            s[r].z = __fmul_rn(s[r].z, dg);
            s[r].w = __fmul_rn(s[r].w, dg);
            rp.x = fmaf(kr[r], s[r].x, rp.x);
            rp.y = fmaf(kr[r], s[r].y, rp.y);
            rp.z = fmaf(kr[r], s[r].z, rp.z);
            rp.w = fmaf(kr[r], s[r].w, rp.w);
        }
        reinterpret_cast<float4*>(sm.red[w])[l] = rp;
        // (A).  A timed-out copy (error word set) stops the CTA here, before this
        // tile's state or outputs are stored: this tile and the CTA's later ones
        // keep their state of before the step instead of taking stale slot data.
        // The decision is block-uniform; thread 0 then waits (bounded) for the
        // copies still in flight into this CTA's slots before the CTA exits.
        if (!__syncthreads_and(landed)) {
            if (t == 0)
                for (int j = i; j < i + kStateBufs && j < count; j++)
                    sm100::mbar_wait(sm100::smem_u32(&sm.full[j % kStateBufs]), (uint32_t)((j / kStateBufs) & 1), err);
            __syncthreads();
            return;
        }
        float4 rr = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int ww = 0; ww < 8; ww++) {
            const float4 p = reinterpret_cast<const float4*>(sm.red[ww])[l];
            rr.x += p.x;
            rr.y += p.y;
            rr.z += p.z;
            rr.w += p.w;
        }
        // delta = beta (v - S^T k)  (deltanet_impl.h:311-317)
        const float4 dl = make_float4(__fmul_rn(bt, __fsub_rn(vv.x, rr.x)), __fmul_rn(bt, __fsub_rn(vv.y, rr.y)),
                                      __fmul_rn(bt, __fsub_rn(vv.z, rr.z)), __fmul_rn(bt, __fsub_rn(vv.w, rr.w)));

        // ---- update + output read (deltanet_impl.h:320-347); the state goes back to HBM
        float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
        float4* So = reinterpret_cast<float4*>(S + (b * hv + h) * (int64_t)kTileFloats);
#pragma unroll
        for (int r = 0; r < 16; r++) {
            s[r].x = fmaf(kr[r], dl.x, s[r].x);
            s[r].y = fmaf(kr[r], dl.y, s[r].y);
            s[r].z = fmaf(kr[r], dl.z, s[r].z);
            s[r].w = fmaf(kr[r], dl.w, s[r].w);
            op.x = fmaf(qr[r], s[r].x, op.x);
            op.y = fmaf(qr[r], s[r].y, op.y);
            op.z = fmaf(qr[r], s[r].z, op.z);
            op.w = fmaf(qr[r], s[r].w, op.w);
            So[(16 * w + r) * (HD / 4) + l] = s[r];
        }
        reinterpret_cast<float4*>(sm.red2[w])[l] = op;
        // The slot's last generic read is above: order them before the bulk copy
        // that refills it (async proxy); barrier (B) hands the slot over.  (Handing
        // it back before the update measured slower: more reads in flight against
        // the write-back.)
        sm100::fence_proxy_async_smem();
        __syncthreads();  // (B)
        if (t == 0 && i + kStateBufs < count) issue(i + kStateBufs);

        // ---- output, per-head RMSNorm (deltanet_impl.h:350-361) and SiLU(z) gate (364-371)
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int ww = 0; ww < 8; ww++) {
            const float4 p = reinterpret_cast<const float4*>(sm.red2[ww])[l];
            o.x += p.x;
            o.y += p.y;
            o.z += p.z;
            o.w += p.w;
        }
        const float sc = 1.0f / sqrtf((float)HD);
        o = make_float4(__fmul_rn(o.x, sc), __fmul_rn(o.y, sc), __fmul_rn(o.z, sc), __fmul_rn(o.w, sc));
        double so = (double)o.x * o.x + (double)o.y * o.y + (double)o.z * o.z + (double)o.w * o.w;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) so += __shfl_xor_sync(0xffffffffu, so, off);
        if ((l >> 2) == w) {  // each warp writes 16 of the 128 columns
            const float inv = 1.0f / sqrtf((float)(so / HD) + 1e-6f);
            const float ov[4] = {o.x, o.y, o.z, o.w}, zv4[4] = {zz.x, zz.y, zz.z, zz.w};
            const float hv4[4] = {hn.x, hn.y, hn.z, hn.w};
            float gv[4];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                float nv = __fmul_rn(ov[c], inv);
                if (head_norm != nullptr) nv = __fmul_rn(nv, hv4[c]);
                const float zv = fminf(fmaxf(zv4[c], -88.0f), 88.0f);
                gv[c] = __fmul_rn(nv, zv / (1.0f + expf(-zv)));
            }
            const int64_t idx = b * inner + h * HD + 4 * l;
            if (gated != nullptr) *reinterpret_cast<float4*>(gated + idx) = make_float4(gv[0], gv[1], gv[2], gv[3]);
            if (gated_h != nullptr) {
                const __half2 h01 = __floats2half2_rn(gv[0], gv[1]), h23 = __floats2half2_rn(gv[2], gv[3]);
                *reinterpret_cast<uint2*>(gated_h + idx) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
            }
        }
        if (t == 0 && h == 0 && conv_pos != nullptr) conv_pos[b] += 1;
    }
}

size_t state_kernel_smem() { return sizeof(StateSmem) + 128; }

// ----------------------------------------------------------- phase timing

namespace {
constexpr int kPhases = 4;
struct PhaseEvents {
    bool on = false;
    bool created = false;
    cudaEvent_t ev[kPhases + 1];
};
PhaseEvents g_phase[64];

PhaseEvents* phase_events() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    return g_phase[dev].on ? &g_phase[dev] : nullptr;
}

inline int mark(PhaseEvents* pe, int i, cudaStream_t s) {
    if (pe) GDN_CUDA(cudaEventRecord(pe->ev[i], s));
    return GDN_OK;
}

// Tensor-core projections.  Q8_0 with 16-bit x from 5 sequences: with one M
// tile the GEMM streams the 35B layer's weights over 128 CTAs, a nearly fixed
// cost, while the int8-MMA GEMV costs ~4.3 us per row and steps up past 4 rows
// (device-paced step at B = 4 / 5 / 8: GEMV 33.7 / 50.8 / 51.7 us, GEMM 42.9 /
// 46.4 / 45.2 us; at 16 / 32 / 63 the GEMM's 55 / 69 / 93 us against 100 / 179
// / 340 us); with fp32 x, whose exact activations the GEMV keeps, from 64.  Q4_K from 32 rows (below, the fp16-MMA GEMV is faster:
// the 35B layer's input projection 15 / 21 us at 8 / 16 rows against 29 us).
constexpr int64_t kTcMinBatch = 64;
constexpr int64_t kTcMinBatch16 = 5;
constexpr int64_t kTcMinBatchQ4k = 32;

bool q8_tc(int64_t B, int x_dtype) { return B >= kTcMinBatch || (B >= kTcMinBatch16 && x_dtype != GDN_DTYPE_F32); }
// Split-K factor of the tensor-core out_proj (K = inner is long, N = hidden short).
constexpr int kOutSplits = 8;
// Split-K factor of the 2 Hv gate rows' exact tensor-core GEMM (one column tile).
constexpr int kGateSplits = 8;

struct Dims {
    int hv, hk, key, inner, qkv;
    int64_t np;   // projection width: QKV + inner + 2 Hv
    int64_t ldp;  // its row stride in the workspace, a multiple of 4 floats (16-byte rows)
};

Dims dims_of(const gdn_dims& d) {
    Dims r;
    r.hv = d.num_v_heads;
    r.hk = d.num_k_heads;
    r.key = r.hk * HD;
    r.inner = r.hv * HD;
    r.qkv = 2 * r.key + r.inner;
    r.np = (int64_t)r.qkv + r.inner + 2 * r.hv;
    r.ldp = (r.np + 3) / 4 * 4;
    return r;
}

struct Workspace {
    float* proj = nullptr;      // [B][np]
    float* act = nullptr;       // [B][QKV] conv'd, SiLU'd, q/k L2-normalised
    float4* gates = nullptr;    // [B][Hv] {decay, beta, 0, 0}
    float* gated = nullptr;     // [B][inner] fp32 (CUDA-core out_proj)
    __half* gated_h = nullptr;  // [B][inner] fp16 (tensor-core out_proj)
    void* xconv = nullptr;      // [B][hidden] 2-byte operand copy of x
    float* partial = nullptr;   // split-K partials of out_proj
    size_t partial_bytes = 0;
    float* gpartial = nullptr;  // split-K partials of the gate rows (tensor-core in_proj)
    size_t gpartial_bytes = 0;
    size_t total = 0;
};

// out_proj runs on the tensor cores with split K (partials in the workspace)
// from these batches on: Q8_0 as q8_tc, Q4_K from kTcMinBatchQ4k.
bool out_proj_splits(int weight_type, int64_t B, int x_dtype) {
    return weight_type == GDN_GGML_Q8_0 ? q8_tc(B, x_dtype) : B >= kTcMinBatchQ4k;
}

// split_out: reserve the split-K partials of out_proj (only used when it splits);
// tc_in: those of the gate rows of a tensor-core input projection.
Workspace carve(const gdn_dims& d, int64_t B, void* base, bool split_out, bool tc_in) {
    const Dims D = dims_of(d);
    Workspace w;
    char* p = static_cast<char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char* r = p ? p + off : nullptr;
        off += round_up(bytes, 256);
        return r;
    };
    w.proj = reinterpret_cast<float*>(take((size_t)B * D.ldp * 4));
    w.act = reinterpret_cast<float*>(take((size_t)B * D.qkv * 4));
    w.gates = reinterpret_cast<float4*>(take((size_t)B * D.hv * 16));
    w.gated = reinterpret_cast<float*>(take((size_t)B * D.inner * 4));
    w.gated_h = reinterpret_cast<__half*>(take((size_t)B * D.inner * 2));
    w.xconv = take((size_t)B * d.hidden * 2);
    if (split_out) {
        w.partial_bytes = gemm_tc_workspace_bytes(B, d.hidden, kOutSplits);
        w.partial = reinterpret_cast<float*>(take(w.partial_bytes));
    }
    if (tc_in) {
        w.gpartial_bytes = gemm_tc_workspace_bytes(B, 2 * (int64_t)D.hv, kGateSplits);
        w.gpartial = reinterpret_cast<float*>(take(w.gpartial_bytes));
    }
    w.total = off;
    return w;
}
}  // namespace

int phase_mark(int i, cudaStream_t s) { return mark(phase_events(), i, s); }

int profile_enable(int on) {
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(GDN_ERR_ARG, "device %d out of range", dev);
    PhaseEvents& pe = g_phase[dev];
    if (on && !pe.created) {
        for (int i = 0; i <= kPhases; i++) GDN_CUDA(cudaEventCreate(&pe.ev[i]));
        pe.created = true;
    }
    pe.on = on != 0;
    return GDN_OK;
}

int phase_ms(float* ms, int n) {
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !g_phase[dev].created) return fail(GDN_ERR_STATE, "profiling was never enabled");
    PhaseEvents& pe = g_phase[dev];
    GDN_CUDA(cudaEventSynchronize(pe.ev[kPhases]));
    int w = 0;
    for (int i = 0; i < kPhases && i < n; i++, w++) GDN_CUDA(cudaEventElapsedTime(&ms[i], pe.ev[i], pe.ev[i + 1]));
    return w;
}

// Covers both weight types and every activation type (the split-K buffers from
// the smallest batch that may take them).
size_t decode_workspace_bytes(const gdn_dims& d, int64_t batch) {
    return carve(d, batch, nullptr, batch >= std::min(kTcMinBatch16, kTcMinBatchQ4k), batch >= kTcMinBatch16).total;
}

// The input projection runs on the tensor cores (Q8_0 weights, q8_tc).
bool in_proj_tc(int weight_type, int64_t B, int x_dtype) {
    return weight_type == GDN_GGML_Q8_0 && q8_tc(B, x_dtype);
}

size_t decode_workspace_bytes_for(const gdn_layer& L, int64_t batch, int flags, int x_dtype) {
    const bool ref = (flags & GDN_DECODE_REF_PROJECTIONS) != 0;
    return carve(L.dims, batch, nullptr, !ref && out_proj_splits(L.weight_type, batch, x_dtype),
                 !ref && in_proj_tc(L.weight_type, batch, x_dtype)).total;
}

int validate_layer(const gdn_layer* L) {
    if (L == nullptr) return fail(GDN_ERR_ARG, "layer is NULL");
    const gdn_dims& d = L->dims;
    if (d.head_dim != HD) return fail(GDN_ERR_SHAPE, "head_dim must be 128 (got %d)", d.head_dim);
    if (d.num_k_heads <= 0 || d.num_v_heads <= 0 || d.num_v_heads % d.num_k_heads != 0)
        return fail(GDN_ERR_SHAPE, "num_v_heads (%d) must be a positive multiple of num_k_heads (%d)",
                    d.num_v_heads, d.num_k_heads);
    if (d.hidden <= 0 || d.hidden % 256 != 0)
        return fail(GDN_ERR_SHAPE, "hidden must be a positive multiple of 256 (got %d)", d.hidden);
    if (L->head_map != GDN_HEAD_MAP_GROUPED && L->head_map != GDN_HEAD_MAP_INTERLEAVED)
        return fail(GDN_ERR_ARG, "head_map must be 0 or 1 (got %d)", L->head_map);
    if (L->weight_type == GDN_GGML_Q8_0) {
        if (!L->in_qs || !L->in_d || !L->out_qs || !L->out_d) return fail(GDN_ERR_ARG, "Q8_0 weight planes are NULL");
        if (!aligned(L->in_qs, 16) || !aligned(L->out_qs, 16) || !aligned(L->in_d, 16) || !aligned(L->out_d, 16))
            return fail(GDN_ERR_ARG, "Q8_0 planes must be 16-byte aligned");
    } else if (L->weight_type == GDN_GGML_Q4_K) {
        if (!L->in_blocks || !L->out_blocks) return fail(GDN_ERR_ARG, "Q4_K weight blocks are NULL");
        if (!aligned(L->in_blocks, 16) || !aligned(L->out_blocks, 16))
            return fail(GDN_ERR_ARG, "Q4_K blocks must be 16-byte aligned");
    } else {
        return fail(GDN_ERR_TYPE, "weight_type %d is not supported (8 = Q8_0, 12 = Q4_K)", L->weight_type);
    }
    if (L->conv1d_w && !aligned(L->conv1d_w, 16)) return fail(GDN_ERR_ARG, "conv1d_w must be 16-byte aligned");
    return GDN_OK;
}

// Input projection: proj[B][np] = x . in_proj^T.
// Q8_0, B >= 64: tensor cores with fp16 activations (bf16 / fp16 x converts
// exactly).  The q, k, v and z rows take one fp16 weight operand (each weight
// d*q rounded once, ~2^-12 relative: ~1e-4 of a projection); the 2 Hv gate
// rows take exact hi + lo weights, since exp(ssm_a * softplus(alpha))
// magnifies any rounding of alpha, split K on the caller's stream beside the
// main GEMM (on the side stream, 96 of 148 SMs at the 35B dims).  fp32 x is
// rounded by the fp16 conversion: then the gate rows run on fp32 CUDA cores
// from the unrounded x.  Otherwise one CUDA-core GEMV over all rows.
static int in_projection(const gdn_layer* L, const Dims& D, int64_t B, const void* x, int x_dtype,
                         const Workspace& ws, cudaStream_t s) {
    const int64_t hidden = L->dims.hidden;
    if (L->weight_type == GDN_GGML_Q4_K) {
        // fp16 x (bf16 / fp16 convert exactly; fp32 would be rounded: CUDA cores then)
        if (B < kTcMinBatchQ4k || x_dtype == GDN_DTYPE_F32)
            return launch_q4_k_gemv(L->in_blocks, D.np, hidden, x, x_dtype, B, ws.proj, D.ldp, s);
        const void* a = x;
        if (x_dtype != GDN_DTYPE_F16 || !aligned(x, 16)) {
            const int st = launch_convert(x, x_dtype, ws.xconv, false, B * hidden, s);
            if (st) return st;
            a = ws.xconv;
        }
        return launch_q4_k_gemm_tc(L->in_blocks, D.np, hidden, a, B, ws.proj, D.ldp, TcOptions(), s);
    }
    if (!q8_tc(B, x_dtype)) return launch_q8_0_gemv(L->in_qs, L->in_d, D.np, hidden, x, x_dtype, B, ws.proj, D.ldp, s);
    const void* a = x;
    int st;
    if (x_dtype != GDN_DTYPE_F16 || !aligned(x, 16)) {
        if ((st = launch_convert(x, x_dtype, ws.xconv, false, B * hidden, s))) return st;
        a = ws.xconv;
    }
    const int64_t n_main = (int64_t)D.qkv + D.inner;
    SideStream* side = nullptr;
    if ((st = side_stream(&side))) return st;
    GDN_CUDA(cudaEventRecord(side->fork, s));
    GDN_CUDA(cudaStreamWaitEvent(side->s, side->fork, 0));
    st = launch_q8_0_gemm_tc(L->in_qs, L->in_d, n_main, hidden, a, false, B, ws.proj, D.ldp, TcOptions(), side->s);
    GDN_CUDA(cudaEventRecord(side->join, side->s));
    if (!st) {
        const int8_t* gq = L->in_qs + n_main * hidden;
        const uint16_t* gd = L->in_d + n_main * (hidden / 32);
        if (x_dtype == GDN_DTYPE_F32) {
            st = launch_q8_0_gemv(gq, gd, D.np - n_main, hidden, x, x_dtype, B, ws.proj + n_main, D.ldp, s);
        } else {
            TcOptions exact;
            exact.split_precision = true;
            exact.splits = kGateSplits;
            exact.workspace = ws.gpartial;
            exact.workspace_bytes = ws.gpartial_bytes;
            st = launch_q8_0_gemm_tc(gq, gd, D.np - n_main, hidden, a, false, B, ws.proj + n_main, D.ldp, exact, s);
        }
    }
    const cudaError_t ej = cudaStreamWaitEvent(s, side->join, 0);  // joined on every path
    if (st) return st;
    if (ej != cudaSuccess) return cuda_status(ej, "decode: join of the input projection");
    return GDN_OK;
}

// The projections as the reference's CPU computes them (quant_matvec per
// tensor, engine/runtime/deltanet_impl.h:275-278 and 374): each of attn_qkv,
// attn_gate, ssm_beta, ssm_alpha and ssm_out takes its own Q8_K or fp32
// branch by its row count, bit for bit (launch_q8_0_gemv_ref).
static int in_projection_ref(const gdn_layer* L, const Dims& D, int64_t B, const float* x, const Workspace& ws,
                             cudaStream_t s) {
    const int64_t hidden = L->dims.hidden, kb = hidden / 32;
    const int64_t seg[4][2] = {{0, D.qkv}, {D.qkv, D.inner}, {(int64_t)D.qkv + D.inner, D.hv},
                               {(int64_t)D.qkv + D.inner + D.hv, D.hv}};
    for (const auto& g : seg) {
        const int st = launch_q8_0_gemv_ref(L->in_qs + g[0] * hidden, L->in_d + g[0] * kb, g[1], hidden, x, B,
                                            ws.proj + g[0], D.ldp, s);
        if (st) return st;
    }
    return GDN_OK;
}

int decode_step(const gdn_layer* L, int64_t B, const void* x, int x_dtype, float* out, float* S, float* conv_buf,
                int32_t* conv_pos, void* wsp, size_t ws_bytes, cudaStream_t s, int flags) {
    int st = validate_layer(L);
    if (st) return st;
    const bool ref = (flags & GDN_DECODE_REF_PROJECTIONS) != 0;
    if (flags & ~GDN_DECODE_REF_PROJECTIONS) return fail(GDN_ERR_ARG, "decode: unknown flags 0x%x", flags);
    if (ref && (L->weight_type != GDN_GGML_Q8_0 || x_dtype != GDN_DTYPE_F32 || !aligned(x, 16)))
        return fail(GDN_ERR_TYPE, "reference projections take a Q8_0 layer and 16-byte aligned fp32 x");
    if (B <= 0 || B > 65535) return fail(GDN_ERR_SHAPE, "batch must be in [1, 65535] (got %lld)", (long long)B);
    if (!x || !out || !S || !conv_pos) return fail(GDN_ERR_ARG, "x, out, S and conv_pos must be non-NULL");
    if (x_dtype != GDN_DTYPE_F32 && x_dtype != GDN_DTYPE_BF16 && x_dtype != GDN_DTYPE_F16)
        return fail(GDN_ERR_TYPE, "x_dtype %d is not supported", x_dtype);
    if (!aligned(S, 16)) return fail(GDN_ERR_ARG, "S must be 16-byte aligned");
    const gdn_dims& d = L->dims;
    const bool tc_out = !ref && out_proj_splits(L->weight_type, B, x_dtype);
    const size_t need = decode_workspace_bytes_for(*L, B, flags, x_dtype);
    if (wsp == nullptr || ws_bytes < need || !aligned(wsp, 256))
        return fail(GDN_ERR_ARG, "workspace must be 256-aligned and hold %zu bytes (got %zu)", need, ws_bytes);
    const Dims D = dims_of(d);
    const Workspace ws = carve(d, B, wsp, tc_out, !ref && in_proj_tc(L->weight_type, B, x_dtype));
    const bool conv = (L->conv1d_w != nullptr && conv_buf != nullptr);
    PhaseEvents* pe = phase_events();

    if ((st = mark(pe, 0, s))) return st;
    if ((st = ref ? in_projection_ref(L, D, B, static_cast<const float*>(x), ws, s)
                  : in_projection(L, D, B, x, x_dtype, ws, s)))
        return st;
    if ((st = mark(pe, 1, s))) return st;
    {
        const int64_t warps = B * (D.qkv / HD + 1);
        st = launch_pdl("gdn_prep_kernel", gdn_prep_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s,
                        ws.proj, D.ldp, ws.act, ws.gates, conv ? conv_buf : nullptr, conv_pos,
                        conv ? L->conv1d_w : nullptr, L->ssm_a, L->dt_bias, B, D.qkv, D.key, D.hv);
        if (st) return st;
    }
    if ((st = mark(pe, 2, s))) return st;
    {
        const int64_t n_tiles = B * D.hv;
        const int64_t ctas = std::min<int64_t>(n_tiles, sm_count());
        const int64_t per = (n_tiles + ctas - 1) / ctas;
        const size_t smem = state_kernel_smem();
        GDN_CUDA(cudaFuncSetAttribute((const void*)gdn_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
        st = launch_pdl("gdn_state_kernel", gdn_state_kernel, dim3((unsigned)((n_tiles + per - 1) / per)), dim3(256),
                        smem, s, ws.act, ws.gates, ws.proj, D.ldp, S, L->head_norm, tc_out ? nullptr : ws.gated,
                        tc_out ? ws.gated_h : nullptr, conv ? conv_pos : nullptr, D.qkv, D.key, D.hv, D.hk,
                        L->head_map, n_tiles, per, device_error_word());
        if (st) return st;
    }
    if ((st = mark(pe, 3, s))) return st;
    if (ref) {
        st = launch_q8_0_gemv_ref(L->out_qs, L->out_d, d.hidden, D.inner, ws.gated, B, out, d.hidden, s);
    } else if (L->weight_type == GDN_GGML_Q4_K) {
        if (tc_out) {  // the fp16 gated heads on the tensor cores, exact weights, split K
            TcOptions opt;
            opt.splits = kOutSplits;
            opt.workspace = ws.partial;
            opt.workspace_bytes = ws.partial_bytes;
            st = launch_q4_k_gemm_tc(L->out_blocks, d.hidden, D.inner, ws.gated_h, B, out, d.hidden, opt, s);
        } else {
            st = launch_q4_k_gemv(L->out_blocks, d.hidden, D.inner, ws.gated, GDN_DTYPE_F32, B, out, d.hidden, s);
        }
    } else if (tc_out) {  // the fp16 gated heads, one fp16 weight operand (as the q/k/v/z rows), split K
        TcOptions opt;
        opt.splits = kOutSplits;
        opt.workspace = ws.partial;
        opt.workspace_bytes = ws.partial_bytes;
        st = launch_q8_0_gemm_tc(L->out_qs, L->out_d, d.hidden, D.inner, ws.gated_h, false, B, out, d.hidden, opt, s);
    } else {
        st = launch_q8_0_gemv(L->out_qs, L->out_d, d.hidden, D.inner, ws.gated, GDN_DTYPE_F32, B, out, d.hidden, s);
    }
    if (st) return st;
    return mark(pe, 4, s);
}

}  // namespace gdn
