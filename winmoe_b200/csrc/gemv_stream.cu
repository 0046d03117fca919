// Streamed dequant-GEMV for small activation batches (decode of up to 63
// sequences, the GQA projections, the Q4_K sweep), 1, 2, 4 or 8 activation
// rows per CTA.
//
// Memory side.  The row-per-warp GEMVs in quant.cu keep one batch of register
// loads in flight per warp, so at batch 1 their speed is set by HBM latency;
// a warp streaming its own rows as separate 2-4 KB bulk copies is no better
// (about 190 small copies per SM, each with its own fixed cost in the copy
// engine).  Here CTA c owns a contiguous range of about n / 148 weight rows and
// one producer warp streams it in stages of 16 rows -- one bulk copy of the
// int8 rows (Q8_0: plus one of their fp16 scale rows), 18-70 KB each, into a
// ring of 2-8 stages in shared memory with mbarrier completion -- while 16
// consumer warps take one row of a stage each and release it on the stage's
// `empty` barrier.  The stage copies start only once the activation loads are
// requested (a named barrier): issued earlier, they held those loads back by
// microseconds on the SM's return path.  Before griddepcontrol.wait the first
// stages are only prefetched into L2.  Every wait is bounded, and the producer
// leaves no copy in flight.
//
// Arithmetic.  Converting every int8 / 4-bit weight to fp32 and multiplying
// costs about six instructions per weight and lane, which bounds a batch-1
// GEMV by instruction issue, not by HBM.  Instead each CTA splits every 32-block
// of the activations into three int8 levels,
//     x ~= s (a + b / 254 + c / 254^2),   s = max|x| / 127,
// (a = rint(x / s), b and c the rounded residuals, all within +-127; the
// representation error is below 3e-7 max|x| of the block, a few fp32
// roundings), and the dot products become exact integer sums on __dp4a:
//     sum q x = s (A + (B + C / 254) / 254),   A = sum q a, B = sum q b, C = sum q c.
// That keeps the fp32-activation semantics of the reference GPU kernels
//   Q8_0: w = d q                      engine/runtime/gpu_offload.cu:152-199
//   Q4_K: w = (d sc) q - dmin m        engine/runtime/gpu_offload.cu:90-98, 237-250
// to fp32 rounding (results differ from an fp32 FMA chain in the last bits,
// as any other summation order does).  The Q4_K min term uses fp32 sums of x
// over every 16, staged with the levels.
//
// Lanes.  Q8_0: lane l takes the 16 weights at 512 i + 16 l of the row (a
// 512-byte line per warp load), inside one 32-block.  Q4_K: lanes 8 g .. 8 g + 7
// share a superblock (g = 0..3, superblocks g, g + 4, ...): lane j = 2 c + h
// reads quant bytes 32 c + 16 h .. + 15, whose low nibbles are weights
// 64 c + 16 h + e (sub-block 2 c) and high nibbles 64 c + 32 + 16 h + e
// (sub-block 2 c + 1).  The level planes carry 32 bytes of padding after every
// 128 (xq_off), so the 16-byte pieces that a quarter-warp reads fall on 8
// distinct bank groups in both mappings.
#include "gdn_common.cuh"
#include "ptx_sm100.cuh"
#include "quant.cuh"
#include <algorithm>

namespace gdn {
namespace {

using namespace sm100;

constexpr int kWarps = 16;      // consumer warps; one more warp produces
constexpr int kStageRows = 16;  // weight rows per stage: one per consumer warp
constexpr int kMaxSlots = 8;
constexpr int kBarBytes = 1024;  // full[kMaxSlots], empty[kMaxSlots], padded
constexpr size_t kSmemLimit = 227 * 1024;
constexpr float kInv254 = 1.0f / 254.0f;
constexpr int kStageBatch = 8;  // activation blocks a warp loads before it reduces them
constexpr int kEarlyStages = 0;  // stages copied before griddepcontrol.wait (the rest after the activation loads)

__host__ __device__ constexpr int64_t plane_len(int64_t k) { return k + (k >> 2); }
__device__ __forceinline__ int64_t xq_off(int64_t i) { return i + ((i >> 7) << 5); }

// Bytes of the staged activations: MB x 3 level planes, the block scales and,
// for Q4_K, the sums of every 16.
__host__ __device__ constexpr size_t staged_bytes(int fmt, int mb, int64_t k) {
    return (size_t)mb * (3 * plane_len(k) + (k / 32) * 4 + (fmt == 1 ? (k / 16) * 4 : 0));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Q4_K 6-bit scale and min of sub-block j from the 12 packed bytes.
__device__ __forceinline__ void scale_min(int j, const uint8_t* sc, int& s, int& m) {
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

// One warp stages U 32-blocks of one activation row at once (lane l holds
// x[32 b_u + l]; blocks with valid[u] false are computed on and not stored):
// the level bytes, the block scales and (Q4_K) the two 16-sums per block.  The
// U blocks advance step by step together, so their shuffle and rounding
// chains overlap instead of running one after another.
template <int FMT, int U, bool PADDED = true>
__device__ __forceinline__ void stage_blocks(const float (&xv)[U], const bool (&valid)[U], const int (&b)[U],
                                             int lane, int8_t* pa, int64_t pl, float* sx, float* x16) {
    // max |x| per block as an integer max of the magnitude bits: a NaN (bits
    // above those of inf) wins, so that it reaches the outputs through the
    // block scale as it would through fp32 products
    uint32_t ab[U];
#pragma unroll
    for (int u = 0; u < U; u++) ab[u] = __float_as_uint(xv[u]) & 0x7fffffffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < U; u++) ab[u] = max(ab[u], __shfl_xor_sync(0xffffffffu, ab[u], o));
#pragma unroll
    for (int u = 0; u < U; u++) {
        const float mx = __uint_as_float(ab[u]);
        // blocks below 2^-64 are scaled up by 2^64 first so that 1 / s stays finite
        const bool tiny = mx < 5.421010862427522e-20f;
        const float K = tiny ? 18446744073709551616.0f : 1.0f;
        const float s = (mx * K) * (1.0f / 127.0f);
        const float inv = mx > 0.0f ? __frcp_rn(s) : 0.0f;  // u * s = x K up to two roundings
        const float v = (xv[u] * K) * inv;
        const float a = rintf(v);
        const float r1 = v - a;  // exact: a is v rounded to an integer, |v| <= 127
        const float bb = rintf(r1 * 254.0f);
        const float r2 = fmaf(r1, 254.0f, -bb);
        const float c = rintf(r2 * 254.0f);
        if (valid[u]) {
            int8_t* p = pa + (PADDED ? xq_off(32 * b[u] + lane) : (int64_t)(32 * b[u] + lane));
            p[0] = (int8_t)(int)a;
            p[pl] = (int8_t)(int)bb;
            p[2 * pl] = (int8_t)(int)c;
            if (lane == 0) sx[b[u]] = tiny ? s * 5.421010862427522e-20f : s;
        }
    }
    if (FMT == 1) {
        float t[U];
#pragma unroll
        for (int u = 0; u < U; u++) t[u] = xv[u];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1)
#pragma unroll
            for (int u = 0; u < U; u++) t[u] += __shfl_xor_sync(0xffffffffu, t[u], o);
#pragma unroll
        for (int u = 0; u < U; u++)
            if (valid[u] && (lane & 15) == 0) x16[2 * b[u] + (lane >> 4)] = t[u];
    }
}

__device__ __forceinline__ int dot16(const uint4 w, const uint4 p) {
    int s = __dp4a((int)w.x, (int)p.x, 0);
    s = __dp4a((int)w.y, (int)p.y, s);
    s = __dp4a((int)w.z, (int)p.z, s);
    return __dp4a((int)w.w, (int)p.w, s);
}

// s (A + (B + C / 254) / 254) for the integer sums of the three levels.
__device__ __forceinline__ float levels(int A, int B, int C) {
    return fmaf(fmaf((float)C, kInv254, (float)B), kInv254, (float)A);
}

struct Staged {
    const int8_t* q;   // [MB][3][plane_len(k)]
    const float* sx;   // [MB][k / 32]
    const float* x16;  // [MB][k / 16]
    int64_t pl;        // plane_len(k)
};

template <int MB>
__device__ __forceinline__ void q8_row(const uint8_t* row, const uint8_t* scales, int64_t k, const Staged& st, int mb,
                                       int lane, float (&acc)[MB]) {
    const uint16_t* dr = reinterpret_cast<const uint16_t*>(scales);
    const int64_t iters = k >> 9;
#pragma unroll 2
    for (int64_t it = 0; it < iters; it++) {
        const int64_t e = (it << 9) + 16 * lane;
        const uint4 q = *reinterpret_cast<const uint4*>(row + e);
        const float dw = fp16_bits_to_float(dr[e >> 5]);
        const int64_t o = xq_off(e);
#pragma unroll
        for (int j = 0; j < MB; j++) {
            if (j < mb) {
                const int8_t* pj = st.q + (int64_t)j * 3 * st.pl + o;
                const int A = dot16(q, *reinterpret_cast<const uint4*>(pj));
                const int B = dot16(q, *reinterpret_cast<const uint4*>(pj + st.pl));
                const int C = dot16(q, *reinterpret_cast<const uint4*>(pj + 2 * st.pl));
                acc[j] = fmaf(dw * st.sx[j * (k >> 5) + (e >> 5)], levels(A, B, C), acc[j]);
            }
        }
    }
}

template <int MB>
__device__ __forceinline__ void q4k_row(const uint8_t* row, int64_t k, const Staged& st, int mb, int lane,
                                        float (&acc)[MB]) {
    const int64_t nsb = k >> 8;
    const int g = lane >> 3, j = lane & 7, c = j >> 1;
    for (int64_t sb = g; sb < nsb; sb += 4) {
        const uint8_t* blk = row + sb * 144;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 q4 = *reinterpret_cast<const uint4*>(blk + 16 + 16 * j);
        const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hdr);
        const float d = fp16_bits_to_float((uint16_t)(hdr.x & 0xFFFFu));
        const float dmin = fp16_bits_to_float((uint16_t)(hdr.x >> 16));
        int s_lo, m_lo, s_hi, m_hi;
        scale_min(2 * c, hb + 4, s_lo, m_lo);
        scale_min(2 * c + 1, hb + 4, s_hi, m_hi);
        const float sl = d * (float)s_lo, ml = dmin * (float)m_lo;
        const float sh = d * (float)s_hi, mh = dmin * (float)m_hi;
        const uint4 lo = make_uint4(q4.x & 0x0F0F0F0Fu, q4.y & 0x0F0F0F0Fu, q4.z & 0x0F0F0F0Fu, q4.w & 0x0F0F0F0Fu);
        const uint4 hi = make_uint4((q4.x >> 4) & 0x0F0F0F0Fu, (q4.y >> 4) & 0x0F0F0F0Fu, (q4.z >> 4) & 0x0F0F0F0Fu,
                                    (q4.w >> 4) & 0x0F0F0F0Fu);
        const int64_t klo = sb * 256 + 64 * c + 16 * (j & 1), khi = klo + 32;
        const int64_t ol = xq_off(klo), oh = xq_off(khi);
#pragma unroll
        for (int jj = 0; jj < MB; jj++) {
            if (jj < mb) {
                const int8_t* pj = st.q + (int64_t)jj * 3 * st.pl;
                const float vl = levels(dot16(lo, *reinterpret_cast<const uint4*>(pj + ol)),
                                        dot16(lo, *reinterpret_cast<const uint4*>(pj + st.pl + ol)),
                                        dot16(lo, *reinterpret_cast<const uint4*>(pj + 2 * st.pl + ol)));
                const float vh = levels(dot16(hi, *reinterpret_cast<const uint4*>(pj + oh)),
                                        dot16(hi, *reinterpret_cast<const uint4*>(pj + st.pl + oh)),
                                        dot16(hi, *reinterpret_cast<const uint4*>(pj + 2 * st.pl + oh)));
                const float* sx = st.sx + jj * (k >> 5);
                const float* s16 = st.x16 + jj * (k >> 4);
                acc[jj] += (sl * sx[klo >> 5] * vl - ml * s16[klo >> 4]) + (sh * sx[khi >> 5] * vh - mh * s16[khi >> 4]);
            }
        }
    }
}

// FMT 0: Q8_0 planes (wq = int8 [n][k], wd = fp16 [n][k / 32]); FMT 1: Q4_K
// superblocks (wq = [n][k / 256][144], wd unused).  CTA c owns the contiguous
// rows [c n / G, (c + 1) n / G) of G CTAs; warp kWarps (the producer) streams
// them kStageRows at a time through `slots` stages, each one bulk copy of the
// int8 rows (plus one of their scale rows), and the consumer warps take one row
// of a stage each, then release the stage on its `empty` barrier.
template <int FMT, int MB>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1)
    gemv_stream_kernel(const uint8_t* __restrict__ wq, const uint8_t* __restrict__ wd, int64_t n, int64_t k,
                       const void* x, int x_dtype, int64_t m, float* __restrict__ y, int64_t ldy, int slots,
                       uint32_t* __restrict__ err) {
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t qbytes = FMT == 0 ? (uint32_t)k : (uint32_t)(k >> 8) * 144u;  // one row
    const uint32_t dbytes = FMT == 0 ? (uint32_t)(k >> 4) : 0u;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxSlots;
    Staged st;
    st.pl = plane_len(k);
    int8_t* xq = reinterpret_cast<int8_t*>(smem + kBarBytes);
    float* sx = reinterpret_cast<float*>(xq + (size_t)MB * 3 * st.pl);
    float* x16 = sx + MB * (k >> 5);
    st.q = xq;
    st.sx = sx;
    st.x16 = x16;
    uint8_t* ring = smem + kBarBytes + staged_bytes(FMT, MB, k);
    const uint32_t qstage = kStageRows * qbytes;  // a stage: kStageRows int8 rows, then their scale rows
    const uint32_t stage_bytes = qstage + kStageRows * dbytes;

    const int64_t r0 = (int64_t)blockIdx.x * n / gridDim.x, r1 = ((int64_t)blockIdx.x + 1) * n / gridDim.x;
    const int64_t nst = (r1 - r0 + kStageRows - 1) / kStageRows;
    auto issue = [&](int64_t i, int slot) {  // producer lane 0: stage i into `slot` (= i mod slots)
        const int64_t ra = r0 + i * kStageRows;
        const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
        const uint32_t bar = smem_u32(full + slot);
        const uint32_t dst = smem_u32(ring + (size_t)slot * stage_bytes);
        mbar_arrive_expect_tx(bar, rows * (qbytes + dbytes));
        bulk_load(dst, wq + ra * (int64_t)qbytes, rows * qbytes, bar);
        if (FMT == 0) bulk_load(dst + qstage, wd + ra * (int64_t)dbytes, rows * dbytes, bar);
    };
    // Before the wait only L2 prefetches of the first stages go out (the weights
    // never come from an earlier kernel): copies into shared memory issued now
    // would sit ahead of the activation loads on the SM's return path.
    if (warp == kWarps && lane == 0) {
        for (int s = 0; s < slots; s++) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), kWarps);
        }
        fence_barrier_init();
        for (int64_t i = 0; i < min(nst, (int64_t)kEarlyStages); i++) issue(i, (int)i);
        for (int64_t i = kEarlyStages; i < min(nst, (int64_t)kEarlyStages + 2); i++) {
            const int64_t ra = r0 + i * kStageRows;
            const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
            bulk_prefetch_l2(wq + ra * (int64_t)qbytes, rows * qbytes);
            if (FMT == 0) bulk_prefetch_l2(wd + ra * (int64_t)dbytes, rows * dbytes);
        }
    }
    __syncthreads();  // the barriers are initialised

    pdl_wait();
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    if (warp < kWarps) {
        // the warp's blocks kStageBatch at a time: every load of a batch is in
        // flight before the first block's reductions wait on one; once the first
        // batch is requested the producer may start the copies (named barrier 1)
        const int nblk = (int)(k >> 5);
        bool announced = false;
        for (int j = 0; j < mb; j++) {
            for (int b0 = warp; b0 < nblk; b0 += kWarps * kStageBatch) {
                float xv[kStageBatch];
                bool valid[kStageBatch];
                int bs[kStageBatch];
#pragma unroll
                for (int u = 0; u < kStageBatch; u++) {
                    bs[u] = b0 + u * kWarps;
                    valid[u] = bs[u] < nblk;
                    xv[u] = valid[u] ? load_act(x, x_dtype, (size_t)(m0 + j) * k + 32 * bs[u] + lane) : 0.0f;
                }
                if (!announced) {
                    bar_arrive(1, (kWarps + 1) * 32);
                    announced = true;
                }
                stage_blocks<FMT, kStageBatch>(xv, valid, bs, lane, xq + (size_t)j * 3 * st.pl, st.pl, sx + j * nblk,
                                               x16 + j * (k >> 4));
            }
        }
        if (!announced) bar_arrive(1, (kWarps + 1) * 32);
        bar_sync(2, kWarps * 32);  // the consumers: every block staged
    }

    if (warp == kWarps) {  // producer
        bar_sync(1, (kWarps + 1) * 32);  // the activation loads are requested
        if (lane == 0) {
            // slot and phase advance with i (no division in the loop)
            int64_t issued = min(nst, (int64_t)kEarlyStages);
            int slot = (int)issued;
            uint32_t phase = 0;  // parity of the slot's current use: 0 on the first pass over the ring
            if (slot == slots) {
                slot = 0;
                phase = 1;
            }
            for (int64_t i = issued; i < nst; i++) {
                if (i >= slots) {  // the stage that used this slot has been read by every consumer
                    if (!mbar_wait(smem_u32(empty + slot), phase ^ 1u, err)) break;
                    fence_proxy_async_smem();
                }
                issue(i, slot);
                issued = i + 1;
                if (++slot == slots) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
            // leave no copy in flight into this CTA's shared memory: the last
            // min(slots, issued) stages, one per slot, walked backwards
            for (int64_t q = 0; q < min((int64_t)slots, issued); q++) {
                slot = slot == 0 ? slots - 1 : slot - 1;
                if (slot == slots - 1) phase ^= 1u;
                mbar_wait(smem_u32(full + slot), phase, err);
            }
        }
        return;
    }
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t i = 0; i < nst; i++) {
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(full + slot), phase, err))) break;
        const int64_t r = r0 + i * kStageRows + warp;
        if (r < r1) {
            const uint8_t* stage = ring + (size_t)slot * stage_bytes;
            float acc[MB];
#pragma unroll
            for (int j = 0; j < MB; j++) acc[j] = 0.0f;
            if (FMT == 0) {
                q8_row<MB>(stage + (size_t)warp * qbytes, stage + qstage + (size_t)warp * dbytes, k, st, mb, lane,
                           acc);
            } else {
                q4k_row<MB>(stage + (size_t)warp * qbytes, k, st, mb, lane, acc);
            }
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (j < mb) {
                    const float v = warp_sum(acc[j]);
                    if (lane == 0) y[(m0 + j) * ldy + r] = v;
                }
            }
        }
        __syncwarp();  // every lane has read its row of the stage
        if (lane == 0) mbar_arrive(smem_u32(empty + slot));
        if (++slot == slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
}

// ------------------------------------------------------------ Q8_0 on IMMA
//
// For three or more activation rows the per-lane dp4a products above are bound
// by shared memory: every weight row re-reads the activation levels.  Here the
// int8 tensor cores take the products (mma.sync m16n8k32 s8 x s8 -> s32, one
// instruction per 32-block = one Q8_0 block): the A operand is 16 rows of
// activation levels, row 4 jj + l = level l of activation row jj (level 3 a
// copy of level 0 with factor 0), the B operand 8 weight rows of the stage, so
// one A fragment serves 8 weight rows and one B fragment 4 activation rows.
// Each block's int32 sums are scaled in fp32 right away, d_w(row) s_x(jj) lf(l),
// lf = 1, 1/254, 1/254^2, 0, and summed over the levels by two lane exchanges.
// The 16 consumer warps split a stage's k blocks (warp w: blocks w, w + 16,
// ...) and add their partial sums through shared memory (double-buffered, one
// named barrier per stage).  Weight rows land in the stage with 16 bytes of
// padding each (one bulk copy per row, then one for the stage's scale rows),
// and the activation planes with 16 bytes each, so that the fragment loads of
// 8 rows fall on 8 distinct bank groups.

__device__ __forceinline__ void imma_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

__host__ __device__ constexpr int64_t mma_plane_len(int64_t k) { return k + 16; }
__host__ __device__ constexpr int64_t mma_row_len(int64_t k) { return k + 16; }
__host__ __device__ constexpr size_t mma_stage_bytes(int64_t k) {
    return (size_t)kStageRows * mma_row_len(k) + (size_t)kStageRows * (k / 16);
}
// activation planes, block scales, and the two reduction buffers
__host__ __device__ constexpr size_t mma_fixed_bytes(int mt, int64_t k) {
    return (size_t)(4 * mt) * 3 * mma_plane_len(k) + (size_t)(4 * mt) * (k / 32) * 4 +
           (size_t)2 * kWarps * 2 * mt * 32 * 4;
}

template <int MT>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1)
    gemv_mma_kernel(const uint8_t* __restrict__ wq, const uint8_t* __restrict__ wd, int64_t n, int64_t k,
                    const void* x, int x_dtype, int64_t m, float* __restrict__ y, int64_t ldy, int slots,
                    uint32_t* __restrict__ err) {
    constexpr int MB = 4 * MT;
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, qq = lane & 3;
    const int nblk = (int)(k >> 5);
    const int64_t plm = mma_plane_len(k), rl = mma_row_len(k);
    const uint32_t dbytes = (uint32_t)(k >> 4);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxSlots;
    int8_t* xq = reinterpret_cast<int8_t*>(smem + kBarBytes);             // [MB][3][plm]
    float* sx = reinterpret_cast<float*>(xq + (size_t)MB * 3 * plm);     // [MB][nblk]
    float* red = sx + MB * nblk;                                         // [2][kWarps][2][MT][32]
    uint8_t* ring = smem + kBarBytes + mma_fixed_bytes(MT, k);
    const size_t stage_bytes = mma_stage_bytes(k);
    const size_t scale_off = (size_t)kStageRows * rl;

    const int64_t r0 = (int64_t)blockIdx.x * n / gridDim.x, r1 = ((int64_t)blockIdx.x + 1) * n / gridDim.x;
    const int64_t nst = (r1 - r0 + kStageRows - 1) / kStageRows;
    auto issue = [&](int64_t i, int slot) {  // producer lane 0: stage i into `slot`
        const int64_t ra = r0 + i * kStageRows;
        const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
        const uint32_t bar = smem_u32(full + slot);
        const uint32_t dst = smem_u32(ring + (size_t)slot * stage_bytes);
        mbar_arrive_expect_tx(bar, rows * ((uint32_t)k + dbytes));
        for (uint32_t r = 0; r < rows; r++) bulk_load(dst + r * (uint32_t)rl, wq + (ra + r) * k, (uint32_t)k, bar);
        bulk_load(dst + (uint32_t)scale_off, wd + ra * (int64_t)dbytes, rows * dbytes, bar);
    };
    if (warp == kWarps && lane == 0) {
        for (int s = 0; s < slots; s++) {
            mbar_init(smem_u32(full + s), 1);
            mbar_init(smem_u32(empty + s), kWarps);
        }
        fence_barrier_init();
        for (int64_t i = 0; i < min(nst, (int64_t)2); i++) {
            const int64_t ra = r0 + i * kStageRows;
            const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
            bulk_prefetch_l2(wq + ra * k, rows * (uint32_t)k);
            bulk_prefetch_l2(wd + ra * (int64_t)dbytes, rows * dbytes);
        }
    }
    __syncthreads();  // the barriers are initialised

    pdl_wait();
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    if (warp < kWarps) {
        bool announced = false;
        for (int j = 0; j < MB; j++) {  // rows past mb are staged as zeros (their outputs are not stored)
            for (int b0 = warp; b0 < nblk; b0 += kWarps * kStageBatch) {
                float xv[kStageBatch];
                bool valid[kStageBatch];
                int bs[kStageBatch];
#pragma unroll
                for (int u = 0; u < kStageBatch; u++) {
                    bs[u] = b0 + u * kWarps;
                    valid[u] = bs[u] < nblk;
                    xv[u] = valid[u] && j < mb ? load_act(x, x_dtype, (size_t)(m0 + j) * k + 32 * bs[u] + lane)
                                               : 0.0f;
                }
                if (!announced) {
                    bar_arrive(1, (kWarps + 1) * 32);
                    announced = true;
                }
                stage_blocks<0, kStageBatch, false>(xv, valid, bs, lane, xq + (size_t)j * 3 * plm, plm,
                                                    sx + j * nblk, nullptr);
            }
        }
        if (!announced) bar_arrive(1, (kWarps + 1) * 32);
        bar_sync(2, kWarps * 32);  // the consumers: every block staged
    }

    if (warp == kWarps) {  // producer
        bar_sync(1, (kWarps + 1) * 32);
        if (lane == 0) {
            int64_t issued = 0;
            int slot = 0;
            uint32_t phase = 0;
            for (int64_t i = 0; i < nst; i++) {
                if (i >= slots) {
                    if (!mbar_wait(smem_u32(empty + slot), phase ^ 1u, err)) break;
                    fence_proxy_async_smem();
                }
                issue(i, slot);
                issued = i + 1;
                if (++slot == slots) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
            for (int64_t q = 0; q < min((int64_t)slots, issued); q++) {
                slot = slot == 0 ? slots - 1 : slot - 1;
                if (slot == slots - 1) phase ^= 1u;
                mbar_wait(smem_u32(full + slot), phase, err);
            }
        }
        return;
    }

    // A rows of this thread: gq and gq + 8 of each m-tile -> activation row
    // 4 mt + jj, level l (level 3 reads level 0's plane, factor 0)
    const int l = gq & 3, jj0 = gq >> 2;
    const float lf = l == 0 ? 1.0f : l == 1 ? kInv254 : l == 2 ? kInv254 * kInv254 : 0.0f;
    const int lp = l == 3 ? 0 : l;
    const int8_t* arow[MT][2];
    const float* srow[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = 4 * mt + jj0 + 2 * h;
            arow[mt][h] = xq + ((size_t)j * 3 + lp) * plm + 4 * qq;
            srow[mt][h] = sx + j * nblk;
        }
    // The consumers meet at a named barrier every stage, so none may leave the
    // loop alone: a warp whose wait gave up (the error word is set) stops
    // waiting and computing but keeps arriving, so that every warp ends.
    bool bad = false;
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t i = 0; i < nst; i++) {
        if (!bad) bad = !__all_sync(0xffffffffu, mbar_wait(smem_u32(full + slot), phase, err));
        const uint8_t* stage = ring + (size_t)slot * stage_bytes;
        const uint16_t* dsc = reinterpret_cast<const uint16_t*>(stage + scale_off);
        float acc[2][MT][4];
#pragma unroll
        for (int g = 0; g < 2; g++)
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[g][mt][e] = 0.0f;
        for (int kb = bad ? nblk : warp; kb < nblk; kb += kWarps) {
            uint32_t a[MT][4];
            float f[MT][2];
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                a[mt][0] = *reinterpret_cast<const uint32_t*>(arow[mt][0] + 32 * kb);
                a[mt][1] = *reinterpret_cast<const uint32_t*>(arow[mt][1] + 32 * kb);
                a[mt][2] = *reinterpret_cast<const uint32_t*>(arow[mt][0] + 32 * kb + 16);
                a[mt][3] = *reinterpret_cast<const uint32_t*>(arow[mt][1] + 32 * kb + 16);
                f[mt][0] = srow[mt][0][kb] * lf;
                f[mt][1] = srow[mt][1][kb] * lf;
            }
#pragma unroll
            for (int g = 0; g < 2; g++) {
                const uint8_t* brow = stage + (size_t)(8 * g + gq) * rl + 32 * kb + 4 * qq;
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(brow);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(brow + 16);
                const float d0 = fp16_bits_to_float(dsc[(8 * g + 2 * qq) * nblk + kb]);
                const float d1 = fp16_bits_to_float(dsc[(8 * g + 2 * qq + 1) * nblk + kb]);
#pragma unroll
                for (int mt = 0; mt < MT; mt++) {
                    int c[4];
                    imma_16832(c, a[mt], b0, b1);
                    acc[g][mt][0] = fmaf((float)c[0], f[mt][0] * d0, acc[g][mt][0]);
                    acc[g][mt][1] = fmaf((float)c[1], f[mt][0] * d1, acc[g][mt][1]);
                    acc[g][mt][2] = fmaf((float)c[2], f[mt][1] * d0, acc[g][mt][2]);
                    acc[g][mt][3] = fmaf((float)c[3], f[mt][1] * d1, acc[g][mt][3]);
                }
            }
        }
        __syncwarp();  // every lane has read the stage
        if (lane == 0) mbar_arrive(smem_u32(empty + slot));
        // sum over the levels (lanes 4 gq + qq with gq's low two bits = l), then
        // the lanes of level 0 leave the warp's partials for rows jj0 and jj0 + 2
        float* rb = red + (size_t)(i & 1) * kWarps * 2 * MT * 32 + (size_t)warp * 2 * MT * 32;
#pragma unroll
        for (int g = 0; g < 2; g++)
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float v = acc[g][mt][e];
                    v += __shfl_xor_sync(0xffffffffu, v, 4);
                    v += __shfl_xor_sync(0xffffffffu, v, 8);
                    if (l == 0) {
                        const int jj = jj0 + 2 * (e >> 1), col = 2 * qq + (e & 1);
                        rb[(g * MT + mt) * 32 + jj * 8 + col] = v;
                    }
                }
        bar_sync(3, kWarps * 32);  // every warp's partials of this stage
        const float* rs = red + (size_t)(i & 1) * kWarps * 2 * MT * 32;
        for (int t = threadIdx.x; t < kStageRows * MB; t += kWarps * 32) {
            const int row = t & 15, j = t >> 4, g = row >> 3, col = row & 7, mt = j >> 2, jj = j & 3;
            const int64_t r = r0 + i * kStageRows + row;
            if (j < mb && r < r1) {
                float sum = 0.0f;
#pragma unroll 4
                for (int w = 0; w < kWarps; w++) sum += rs[(size_t)w * 2 * MT * 32 + (g * MT + mt) * 32 + jj * 8 + col];
                y[(m0 + j) * ldy + r] = sum;
            }
        }
        if (++slot == slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
}

template <int MT>
int run_mma(const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
            int64_t ldy, int slots, size_t smem, cudaStream_t s) {
    const void* fn = (const void*)gemv_mma_kernel<MT>;
    GDN_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t ctas = std::min<int64_t>(sm_count(), n);
    const dim3 grid((unsigned)ctas, (unsigned)((m + 4 * MT - 1) / (4 * MT)));
    return launch_pdl("gemv_mma_kernel<q8_0>", gemv_mma_kernel<MT>, grid, dim3((kWarps + 1) * 32), smem, s,
                      static_cast<const uint8_t*>(wq), static_cast<const uint8_t*>(wd), n, k, x, dt, m, y, ldy,
                      slots, device_error_word());
}

template <int FMT, int MB>
int run(const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
        int64_t ldy, int slots, size_t smem, cudaStream_t s) {
    const void* fn = (const void*)gemv_stream_kernel<FMT, MB>;
    GDN_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t ctas = std::min<int64_t>(sm_count(), n);
    const dim3 grid((unsigned)ctas, (unsigned)((m + MB - 1) / MB));
    return launch_pdl(FMT == 0 ? "gemv_stream_kernel<q8_0>" : "gemv_stream_kernel<q4_k>",
                      gemv_stream_kernel<FMT, MB>, grid, dim3((kWarps + 1) * 32), smem, s,
                      static_cast<const uint8_t*>(wq), static_cast<const uint8_t*>(wd), n, k, x, dt, m, y, ldy,
                      slots, device_error_word());
}

}  // namespace

// Plans a streamed launch: the activation rows per CTA (1, 2, 4 or 8; more
// rows run as further CTA rows of the grid, each streaming the weights again,
// mostly from L2), the stage slots and the shared memory.  0 when the shape
// does not qualify (k not a multiple of 512 for Q8_0 or 256 for Q4_K, a base
// address not 16-byte aligned, or not even one activation row fitting beside 2
// stages).
static int plan(int fmt, const void* wq, const void* wd, int64_t k, int64_t m, int* mb_out, int* slots_out,
                size_t* smem_out) {
    if (m < 1 || (m + 7) / 8 > 65535 || k < 256 || (k & (fmt == 0 ? 511 : 255)) != 0) return 0;
    if ((reinterpret_cast<uintptr_t>(wq) & 15) != 0) return 0;
    if (fmt == 0 && (reinterpret_cast<uintptr_t>(wd) & 15) != 0) return 0;
    const int64_t stage = (int64_t)kStageRows * (fmt == 0 ? k + k / 16 : (k / 256) * 144);
    for (int mb = m >= 5 ? 8 : m >= 3 ? 4 : (int)m; mb >= 1; mb >>= 1) {
        const size_t base = kBarBytes + staged_bytes(fmt, mb, k);
        if (base >= kSmemLimit) continue;
        const int slots = (int)std::min<int64_t>(kMaxSlots, (int64_t)(kSmemLimit - base) / stage);
        if (slots < 2) continue;
        *mb_out = mb;
        *slots_out = slots;
        *smem_out = base + (size_t)slots * stage;
        return 1;
    }
    return 0;
}

// The IMMA plan (Q8_0, three or more activation rows): 2 m-tiles (8 rows per
// CTA) when 2 stages fit beside them, else 1; 0 if neither fits.
static int plan_mma(const void* wq, const void* wd, int64_t k, int64_t m, int* mt_out, int* slots_out,
                    size_t* smem_out) {
    if (m < 3 || (m + 3) / 4 > 65535 || k < 512 || (k & 511) != 0) return 0;
    if ((reinterpret_cast<uintptr_t>(wq) & 15) != 0 || (reinterpret_cast<uintptr_t>(wd) & 15) != 0) return 0;
    for (int mt = m > 4 ? 2 : 1; mt >= 1; mt--) {
        const size_t base = kBarBytes + mma_fixed_bytes(mt, k);
        if (base >= kSmemLimit) continue;
        const int slots = (int)std::min<size_t>(kMaxSlots, (kSmemLimit - base) / mma_stage_bytes(k));
        if (slots < 2) continue;
        *mt_out = mt;
        *slots_out = slots;
        *smem_out = base + (size_t)slots * mma_stage_bytes(k);
        return 1;
    }
    return 0;
}

int launch_gemv_stream(int fmt, const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt,
                       int64_t m, float* y, int64_t ldy, cudaStream_t s) {
    int mb = 0, slots = 0;
    size_t smem = 0;
    if (fmt == 0 && n > 0 && plan_mma(wq, wd, k, m, &mb, &slots, &smem))
        return mb == 2 ? run_mma<2>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s)
                       : run_mma<1>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
    if (!plan(fmt, wq, wd, k, m, &mb, &slots, &smem)) return GDN_ERR_SHAPE;
    if (n <= 0) return GDN_OK;
    if (fmt == 0) {
        switch (mb) {
            case 1: return run<0, 1>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
            case 2: return run<0, 2>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
            case 4: return run<0, 4>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
            default: return run<0, 8>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
        }
    }
    switch (mb) {
        case 1: return run<1, 1>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
        case 2: return run<1, 2>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
        case 4: return run<1, 4>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
        default: return run<1, 8>(wq, wd, n, k, x, dt, m, y, ldy, slots, smem, s);
    }
}

bool gemv_stream_fits(int fmt, const void* wq, const void* wd, int64_t k, int64_t m) {
    int mb, slots;
    size_t smem;
    return plan(fmt, wq, wd, k, m, &mb, &slots, &smem) != 0;
}

}  // namespace gdn
