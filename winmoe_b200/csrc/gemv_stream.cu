// Streamed dequant-GEMV for small activation batches (decode of up to 63
// sequences, the GQA projections, the Q4_K sweep, the expert FFN's Q4_K / Q5_K
// projections).  Three consumers of one streaming scheme: gemv_stream_kernel
// (dp4a, 1, 2, 4 or 8 activation rows per CTA; every format at 1-2 rows),
// gemv_mma_kernel (Q8_0, 3..63 rows, int8 mma.sync) and gemv_hmma_kernel
// (Q4_K / Q5_K, 3 or more rows, fp16 mma.sync on exact q*sc weights); row
// segment tables (several matrices in one launch) and k-segments (matrices
// side by side along k) serve the expert FFN.
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
// stages are only prefetched into L2.  Every wait is bounded (the GEMV waits
// poll with a suspend-time hint), and the producer leaves no copy in flight.
//
// Arithmetic.  Converting every int8 / 4-bit weight to fp32 and multiplying
// costs about six instructions per weight and lane, which bounds a batch-1
// GEMV by instruction issue, not by HBM.  Instead each CTA splits every 32-block
// of the activations into three int8 levels,
//     x ~= s (a + b / 254 + c / 254^2),   s = max|x| / 127,
// (a = rint(x / s), b and c the rounded residuals, all within +-127; the
// representation error is below 5e-7 max|x| of the block, a few fp32
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
constexpr int kStageBatch = 4;  // 128-element pieces a warp loads from global memory before it reduces them
constexpr int kSmemBatch = 2;   // ... from shared memory (the activations brought in by a bulk copy)

__host__ __device__ constexpr int64_t plane_len(int64_t k) { return k + (k >> 2); }

// Weight formats: 0 = Q8_0 planes (int8 row + fp16 scale row), 1 = Q4_K and
// 2 = Q5_K superblocks (144 / 176 bytes per 256 weights).  Bytes of one
// weight row in global memory (the int8 plane's row for Q8_0).
__host__ __device__ constexpr int64_t row_qbytes(int fmt, int64_t k) {
    return fmt == 0 ? k : (k / 256) * (fmt == 1 ? 144 : 176);
}
__device__ __forceinline__ int64_t xq_off(int64_t i) { return i + ((i >> 7) << 5); }


// Bytes of the staged activations: MB x 3 level planes, the block scales and,
// for Q4_K, the sums of every 16.
__host__ __device__ constexpr size_t staged_bytes(int fmt, int mb, int64_t k) {
    return (size_t)mb * (3 * plane_len(k) + (k / 32) * 4 + (fmt != 0 ? (k / 16) * 4 : 0));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Q4_K / Q5_K 6-bit scales and mins (q4k_dequant.h:43-60): sub-block j < 4 takes
// scale = sc[j] & 63, min = sc[j + 4] & 63; j >= 4 takes scale = (sc[j + 4] & 15)
// | (sc[j - 4] >> 6) << 4, min = (sc[j + 4] >> 4) | (sc[j] >> 6) << 4.  With the
// 12 bytes as words W0 W1 W2, one byte per sub-block:
//   scales 0-3 = W0 & 0x3F3F3F3F,  4-7 = (W2 & 0x0F0F0F0F) | ((W0 >> 2) & 0x30303030)
//   mins   0-3 = W1 & 0x3F3F3F3F,  4-7 = ((W2 >> 4) & 0x0F0F0F0F) | ((W1 >> 2) & 0x30303030)

// Rounds v (|v| < 2^22) to the nearest integer, ties to even, by adding
// 1.5 * 2^23: returns the integer, and the rounded value as a float in *f.
__device__ __forceinline__ int round_magic(float v, float* f) {
    const float t = v + 12582912.0f;
    *f = t - 12582912.0f;
    return __float_as_int(t) - 0x4B400000;
}

__device__ __forceinline__ float rcp_approx(float s) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
    return r;
}

// One warp stages 128 activations of one row (four 32-blocks): lane l holds
// x[4 l .. 4 l + 3] (its block is l / 8), writes the four level bytes of each
// plane as one 32-bit word at p (plane a; b and c at +pl, +2 pl), lanes 8 q
// the block scales at sxp[q], and (Q4_K) lanes 4 h the 16-sums at x16p[h].
// The block max needs three lane exchanges.  Every CTA stages the
// activations itself, so this is kept to about twenty instructions per block.
template <int FMT>
__device__ __forceinline__ void stage_128(float4 xv, bool valid, int8_t* p, float* sxp, float* x16p, int pl,
                                          int lane) {
    // max |x| of the block as an integer max of the magnitude bits: a NaN (bits
    // above those of inf) wins and makes the block scale NaN, so that it
    // reaches the outputs as it would through fp32 products
    uint32_t ab = max(max(__float_as_uint(xv.x) & 0x7fffffffu, __float_as_uint(xv.y) & 0x7fffffffu),
                      max(__float_as_uint(xv.z) & 0x7fffffffu, __float_as_uint(xv.w) & 0x7fffffffu));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, o));
    const float mx = __uint_as_float(ab);
    // blocks below 2^-64 are scaled up by 2^64 first so that 1 / s stays finite
    const bool tiny = mx < 5.421010862427522e-20f;
    const float K = tiny ? 18446744073709551616.0f : 1.0f;
    const float s = (mx * K) * (1.0f / 127.0f);
    // 1 / s within an ulp: v s = x K up to a few roundings, |v| <= 127 + tiny
    const float inv = mx > 0.0f ? rcp_approx(s) : 0.0f;
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t wa = 0, wb = 0, wc = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float v = (xs[e] * K) * inv;  // x K exact (a power of two), below 1 when tiny
        float af, bf, cf;
        const int a = round_magic(v, &af);
        const float r1 = v - af;  // exact: af is v rounded to an integer
        const int bb = round_magic(r1 * 254.0f, &bf);
        const float r2 = fmaf(r1, 254.0f, -bf);
        const int c = round_magic(r2 * 254.0f, &cf);
        wa |= (uint32_t)(a & 0xff) << (8 * e);
        wb |= (uint32_t)(bb & 0xff) << (8 * e);
        wc |= (uint32_t)(c & 0xff) << (8 * e);
    }
    if (valid) {
        *reinterpret_cast<uint32_t*>(p) = wa;
        *reinterpret_cast<uint32_t*>(p + pl) = wb;
        *reinterpret_cast<uint32_t*>(p + 2 * pl) = wc;
        if ((lane & 7) == 0) sxp[lane >> 3] = tiny ? s * 5.421010862427522e-20f : s;
    }
    if (FMT != 0) {
        float t = (xv.x + xv.y) + (xv.z + xv.w);
        t += __shfl_xor_sync(0xffffffffu, t, 1);
        t += __shfl_xor_sync(0xffffffffu, t, 2);
        if (valid && (lane & 3) == 0) x16p[lane >> 2] = t;
    }
}

// Plane a of activation row j at xq + 3 j pl; element e at xq_off(e)
// (PADDED) or e.
template <bool PADDED>
__device__ __forceinline__ int8_t* level_ptr(int8_t* xq, int pl, int j, int e) {
    return xq + 3 * j * pl + (PADDED ? (int)xq_off(e) : e);
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

// Q4_K (Q5 = false) or Q5_K (Q5 = true, 176-byte superblocks: d, dmin, the
// 12 scale bytes, qh[32], qs[128]; weight 64 c + 16 h + e takes bit 2 c of
// qh[16 h + e] as its fifth bit, weight 64 c + 32 + 16 h + e bit 2 c + 1,
// gpu_offload.cu:302-309).
template <int MB, bool Q5 = false>
__device__ __forceinline__ void q4k_row(const uint8_t* row, int64_t k, const Staged& st, int mb, int lane,
                                        float (&acc)[MB]) {
    const int64_t nsb = k >> 8;
    const int g = lane >> 3, j = lane & 7, c = j >> 1;
    for (int64_t sb = g; sb < nsb; sb += 4) {
        const uint8_t* blk = row + sb * (Q5 ? 176 : 144);
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 q4 = *reinterpret_cast<const uint4*>(blk + (Q5 ? 48 : 16) + 16 * j);
        const float d = fp16_bits_to_float((uint16_t)(hdr.x & 0xFFFFu));
        const float dmin = fp16_bits_to_float((uint16_t)(hdr.x >> 16));
        // the 6-bit scales / mins of sub-blocks 2 c and 2 c + 1 from the packed
        // words (all eight at once, one byte each)
        const uint32_t scw = c < 2 ? (hdr.y & 0x3F3F3F3Fu) : ((hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u));
        const uint32_t mnw = c < 2 ? (hdr.z & 0x3F3F3F3Fu)
                                   : (((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u));
        const int bs = 16 * (c & 1);  // byte 2 c & 3 of the word, and the next
        const int s_lo = (int)((scw >> bs) & 0xFFu), s_hi = (int)((scw >> (bs + 8)) & 0xFFu);
        const int m_lo = (int)((mnw >> bs) & 0xFFu), m_hi = (int)((mnw >> (bs + 8)) & 0xFFu);
        const float sl = d * (float)s_lo, ml = dmin * (float)m_lo;
        const float sh = d * (float)s_hi, mh = dmin * (float)m_hi;
        uint4 lo = make_uint4(q4.x & 0x0F0F0F0Fu, q4.y & 0x0F0F0F0Fu, q4.z & 0x0F0F0F0Fu, q4.w & 0x0F0F0F0Fu);
        uint4 hi = make_uint4((q4.x >> 4) & 0x0F0F0F0Fu, (q4.y >> 4) & 0x0F0F0F0Fu, (q4.z >> 4) & 0x0F0F0F0Fu,
                              (q4.w >> 4) & 0x0F0F0F0Fu);
        if (Q5) {
            const uint4 qh = *reinterpret_cast<const uint4*>(blk + 16 + 16 * (j & 1));
            const int bl = 2 * c, bh = 2 * c + 1;
            lo.x |= ((qh.x >> bl) & 0x01010101u) << 4;
            lo.y |= ((qh.y >> bl) & 0x01010101u) << 4;
            lo.z |= ((qh.z >> bl) & 0x01010101u) << 4;
            lo.w |= ((qh.w >> bl) & 0x01010101u) << 4;
            hi.x |= ((qh.x >> bh) & 0x01010101u) << 4;
            hi.y |= ((qh.y >> bh) & 0x01010101u) << 4;
            hi.z |= ((qh.z >> bh) & 0x01010101u) << 4;
            hi.w |= ((qh.w >> bh) & 0x01010101u) << 4;
        }
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

// Stages rows 0 .. rows-1 of the activations (x read for rows < mb, zeros
// beyond) into level planes, from global memory (x: all rows, this CTA's from
// row m0) or from shared memory (SMEM: xs holds this CTA's rows).  The
// 128-element pieces of all rows form one list; warp w takes pieces w,
// w + kWarps, ..., U at a time, every read of a batch issued before its
// reductions.  From global memory the warp arrives on named barrier 1 (the
// producer's go) once its first batch is requested.
// The SwiGLU input for elements e .. e + 3 of an fp32 activation row xr that
// holds [g | u] (k values each), or [s][g | u] per k-segment s of k / kseg
// values (o.kseg > 0; the four elements lie in one segment), times the
// segment's scale: (g * sigmoid(g)) * u, as the reference's swiglu_kernel.
__device__ __forceinline__ float4 swiglu4(const char* xr, int64_t e, int64_t k, const GemvOpts& o) {
    int64_t go = e, uo = k + e;
    float sc = 1.0f;
    if (o.kseg) {
        const int64_t ks = k / o.kseg;
        const int sgm = (int)(e / ks);
        go = e + (int64_t)sgm * ks;
        uo = go + ks;
#pragma unroll
        for (int i = 0; i < kGemvMaxSeg; i++)  // static indices: no copy of the parameter block
            if (i == sgm) sc = o.kscale[i];
    }
    const float4 gv = *reinterpret_cast<const float4*>(xr + (size_t)go * 4);
    const float4 uv = *reinterpret_cast<const float4*>(xr + (size_t)uo * 4);
    float4 r = make_float4((gv.x * (1.0f / (1.0f + expf(-gv.x)))) * uv.x, (gv.y * (1.0f / (1.0f + expf(-gv.y)))) * uv.y,
                           (gv.z * (1.0f / (1.0f + expf(-gv.z)))) * uv.z, (gv.w * (1.0f / (1.0f + expf(-gv.w)))) * uv.w);
    if (o.kseg) r = make_float4(r.x * sc, r.y * sc, r.z * sc, r.w * sc);
    return r;
}

template <int FMT, bool PADDED, bool SMEM, int U>
__device__ __forceinline__ void stage_rows(const void* x, int x_dtype, int64_t ldx, int64_t m0, int mb, int rows,
                                           int64_t k, int warp, int lane, int8_t* xq, int pl, float* sx, float* x16,
                                           const GemvOpts& o) {
    const int npc = (int)(k >> 7), nblk = (int)(k >> 5);
    const size_t es = x_dtype == GDN_DTYPE_F32 ? 4 : 2;
    const int64_t xk = ldx;  // elements between activation rows
    const char* x0 = static_cast<const char*>(x) + (SMEM ? 0 : (size_t)m0 * xk * es);
    const bool vec = x_dtype == GDN_DTYPE_F32 && (reinterpret_cast<uintptr_t>(x0) & 15) == 0;
    bool announced = SMEM;
    // (j, c): row and piece of this warp's next item; advanced by kWarps pieces
    int j = 0, c = warp;
    while (c >= npc && j < rows) {
        c -= npc;
        j++;
    }
    while (j < rows) {
        float4 xv[U];
        int ju[U], cu[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            ju[u] = j;
            cu[u] = c;
            const int e = 128 * c + 4 * lane;
            xv[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (j < rows && j < mb) {
                const char* xr = x0 + (size_t)j * xk * es;
                if (o.swiglu) {
                    xv[u] = swiglu4(xr, e, k, o);
                } else if (vec) {
                    xv[u] = *reinterpret_cast<const float4*>(xr + (size_t)e * 4);
                } else {
                    xv[u] = make_float4(load_act(xr, x_dtype, e), load_act(xr, x_dtype, e + 1),
                                        load_act(xr, x_dtype, e + 2), load_act(xr, x_dtype, e + 3));
                }
            }
            c += kWarps;
            while (c >= npc && j < rows) {
                c -= npc;
                j++;
            }
        }
        if (!announced) {
            bar_arrive(1, (kWarps + 1) * 32);
            announced = true;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const bool valid = ju[u] < rows;
            const int jj = valid ? ju[u] : 0, cc = valid ? cu[u] : 0;
            stage_128<FMT>(xv[u], valid, level_ptr<PADDED>(xq, pl, jj, 128 * cc + 4 * lane), sx + jj * nblk + 4 * cc,
                           FMT != 0 ? x16 + jj * 2 * nblk + 8 * cc : nullptr, pl, lane);
        }
    }
    if (!announced) bar_arrive(1, (kWarps + 1) * 32);
}

// The ring shared by both kernels.  Before griddepcontrol.wait the producer
// lane only initialises the barriers and prefetches the first stages into L2.
// After it, when the activations come by bulk copy (nx > 0 slots at the end of
// the ring hold them until every consumer warp has staged its blocks: `xdone`),
// that copy is issued first, so that no weight stage sits ahead of it; else the
// consumers load them from global memory and the producer waits (named barrier
// 1) until those loads are requested.  Every wait is bounded; the producer
// leaves no copy in flight into the CTA's shared memory.
struct Ring {
    uint64_t* full;   // [kMaxSlots] a stage landed
    uint64_t* empty;  // [kMaxSlots] every consumer warp has read it
    uint64_t* xbar;   // the activations landed
    uint64_t* xdone;  // every consumer warp has staged its activation blocks
    int slots, nx;
};

__device__ __forceinline__ Ring ring_of(uint8_t* smem, int slots, int nx) {
    uint64_t* b = reinterpret_cast<uint64_t*>(smem);
    return Ring{b, b + kMaxSlots, b + 2 * kMaxSlots, b + 2 * kMaxSlots + 1, slots, nx};
}

__device__ __forceinline__ void ring_init(const Ring& R) {
    for (int s = 0; s < R.slots; s++) {
        mbar_init(smem_u32(R.full + s), 1);
        mbar_init(smem_u32(R.empty + s), kWarps);
    }
    mbar_init(smem_u32(R.xbar), 1);
    mbar_init(smem_u32(R.xdone), kWarps);
    fence_barrier_init();
}

template <class Issue>
__device__ __forceinline__ void produce(const Ring& R, int64_t nst, Issue issue, const void* xsrc, int xrows,
                                        uint32_t xrow_bytes, size_t xsrc_stride, const uint8_t* xdst, uint32_t* err) {
    if (R.nx > 0) {  // the activation rows, packed at xdst (one copy, or one per row when strided)
        mbar_arrive_expect_tx(smem_u32(R.xbar), (uint32_t)xrows * xrow_bytes);
        if (xsrc_stride == xrow_bytes) {
            bulk_load(smem_u32(xdst), xsrc, (uint32_t)xrows * xrow_bytes, smem_u32(R.xbar));
        } else {
            for (int j = 0; j < xrows; j++)
                bulk_load(smem_u32(xdst) + (uint32_t)j * xrow_bytes, static_cast<const char*>(xsrc) + j * xsrc_stride,
                          xrow_bytes, smem_u32(R.xbar));
        }
    }
    int64_t issued = 0;
    int slot = 0;
    uint32_t phase = 0;  // parity of the slot's current use: 0 on the first pass over the ring
    bool xfree = R.nx == 0;
    for (int64_t i = 0; i < nst; i++) {
        if (i >= R.slots) {  // the stage that used this slot has been read by every consumer
            if (!mbar_wait_sleep(smem_u32(R.empty + slot), phase ^ 1u, err)) break;
            fence_proxy_async_smem();
        } else if (!xfree && slot >= R.slots - R.nx) {  // the slot still holds the activations
            if (!mbar_wait_sleep(smem_u32(R.xdone), 0, err)) break;
            xfree = true;
            fence_proxy_async_smem();
        }
        issue(i, slot);
        issued = i + 1;
        if (++slot == R.slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
    // the last min(slots, issued) stages, one per slot, walked backwards
    for (int64_t q = 0; q < min((int64_t)R.slots, issued); q++) {
        slot = slot == 0 ? R.slots - 1 : slot - 1;
        if (slot == R.slots - 1) phase ^= 1u;
        mbar_wait_sleep(smem_u32(R.full + slot), phase, err);
    }
    if (R.nx > 0) mbar_wait_sleep(smem_u32(R.xbar), 0, err);
}

// Consumers: the activations into level planes, then named barrier 2 (every
// block staged).  Returns false if the activation copy never landed (the
// error word is set; the planes are then not staged, and every wait of the
// caller still ends).
template <int FMT, bool PADDED>
__device__ __forceinline__ bool consume_activations(const Ring& R, const void* x, int x_dtype, int64_t ldx,
                                                    const uint8_t* xs, int64_t m0, int mb, int rows, int64_t k,
                                                    int warp, int lane, int8_t* xq, int pl, float* sx, float* x16,
                                                    const GemvOpts& o, uint32_t* err) {
    bool ok = true;
    if (R.nx > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_sleep(smem_u32(R.xbar), 0, err));
        if (ok)
            stage_rows<FMT, PADDED, true, kSmemBatch>(xs, x_dtype, o.swiglu ? 2 * k : k, 0, mb, rows, k, warp, lane,
                                                      xq, pl, sx, x16, o);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(R.xdone));
    } else {
        stage_rows<FMT, PADDED, false, kStageBatch>(x, x_dtype, ldx, m0, mb, rows, k, warp, lane, xq, pl, sx, x16, o);
    }
    bar_sync(2, kWarps * 32);
    return ok;
}

// This CTA's weight rows [r0, r1): with one matrix CTA c of G owns rows
// [c n / G, (c + 1) n / G); with a segment table (o.nseg matrices of seg_rows
// rows), G / nseg CTAs split each matrix (the rest own nothing), so that no
// CTA's rows -- and no stage's bulk copy -- straddle two matrices.  Row r is
// then row r - rb of the matrix wb, and sg the CTA's matrix (0 without a table).
__device__ __forceinline__ void row_range(int64_t n, const GemvOpts& o, int64_t& r0, int64_t& r1,
                                          const uint8_t*& wb, int64_t& rb, int& sg, const uint8_t* wq) {
    const int64_t c = blockIdx.x, G = gridDim.x;
    if (o.nseg == 0) {
        r0 = c * n / G;
        r1 = (c + 1) * n / G;
        wb = wq;
        rb = 0;
        sg = 0;
        return;
    }
    const int64_t Gs = G / o.nseg;
    sg = (int)min(c / Gs, (int64_t)o.nseg - 1);
    const int64_t cs = c - (int64_t)sg * Gs;
    rb = (int64_t)sg * o.seg_rows;
    wb = o.seg[sg];
    if (cs >= Gs) {  // beyond the last matrix's share: nothing
        r0 = r1 = rb;
        return;
    }
    r0 = rb + cs * o.seg_rows / Gs;
    r1 = rb + (cs + 1) * o.seg_rows / Gs;
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
                       const void* x, int x_dtype, int64_t m, float* __restrict__ y, int64_t ldy, int slots, int nx,
                       GemvOpts o, uint32_t* __restrict__ err) {
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t qbytes = (uint32_t)row_qbytes(FMT, k);  // one row
    const uint32_t dbytes = FMT == 0 ? (uint32_t)(k >> 4) : 0u;
    const Ring R = ring_of(smem, slots, nx);
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

    int64_t r0, r1, rb;  // this CTA's rows [r0, r1); row r is row r - rb of matrix wb
    const uint8_t* wb;
    int sg;
    row_range(n, o, r0, r1, wb, rb, sg, wq);
    const int64_t nst = (r1 - r0 + kStageRows - 1) / kStageRows;
    auto issue = [&](int64_t i, int slot) {  // producer lane 0: stage i into `slot` (= i mod slots)
        const int64_t ra = r0 + i * kStageRows;
        const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
        const uint32_t bar = smem_u32(R.full + slot);
        const uint32_t dst = smem_u32(ring + (size_t)slot * stage_bytes);
        mbar_arrive_expect_tx(bar, rows * (qbytes + dbytes));
        if (FMT != 0 && o.kseg) {  // k-segments: row r = the matrices' rows r side by side
            const uint32_t qs = qbytes / (uint32_t)o.kseg;
            for (uint32_t r = 0; r < rows; r++)
                for (int sgm = 0; sgm < o.kseg; sgm++)
                    bulk_load(dst + r * qbytes + (uint32_t)sgm * qs, o.seg[sgm] + (ra + r) * (int64_t)qs, qs, bar);
        } else {
            bulk_load(dst, wb + (ra - rb) * (int64_t)qbytes, rows * qbytes, bar);
        }
        if (FMT == 0) bulk_load(dst + qstage, wd + ra * (int64_t)dbytes, rows * dbytes, bar);
    };
    if (warp == kWarps && lane == 0) {
        ring_init(R);
        for (int64_t i = 0; i < min(nst, (int64_t)2); i++) {  // the weights never come from an earlier kernel
            const int64_t ra = r0 + i * kStageRows;
            const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
            if (FMT != 0 && o.kseg) {
                const uint32_t qs = qbytes / (uint32_t)o.kseg;
                for (int sgm = 0; sgm < o.kseg; sgm++) bulk_prefetch_l2(o.seg[sgm] + ra * (int64_t)qs, rows * qs);
            } else {
                bulk_prefetch_l2(wb + (ra - rb) * (int64_t)qbytes, rows * qbytes);
            }
            if (FMT == 0) bulk_prefetch_l2(wd + ra * (int64_t)dbytes, rows * dbytes);
        }
    }
    __syncthreads();  // the barriers are initialised

    pdl_wait();
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    const size_t esize = x_dtype == GDN_DTYPE_F32 ? 4 : 2;
    const int64_t xrow = o.swiglu ? 2 * k : k;  // activation elements per row read
    const int64_t ldx = o.ldx ? o.ldx : xrow;   // ... and between rows in memory
    const void* xe = static_cast<const char*>(x) + (size_t)sg * o.x_seg * esize;  // this CTA's matrix's input
    const uint8_t* xs = ring + (size_t)(slots - nx) * stage_bytes;  // the activations, when nx > 0
    if (warp < kWarps)
        consume_activations<FMT, true>(R, xe, x_dtype, ldx, xs, m0, mb, mb, k, warp, lane, xq, (int)st.pl, sx, x16,
                                       o, err);

    if (warp == kWarps) {  // producer
        if (nx == 0) bar_sync(1, (kWarps + 1) * 32);  // the activation loads are requested
        if (lane == 0)
            produce(R, nst, issue, static_cast<const uint8_t*>(xe) + (size_t)m0 * ldx * esize, mb,
                    (uint32_t)((size_t)xrow * esize), (size_t)ldx * esize, xs, err);
        return;
    }
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t i = 0; i < nst; i++) {
        if (!__all_sync(0xffffffffu, mbar_wait_sleep(smem_u32(R.full + slot), phase, err))) break;
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
                q4k_row<MB, FMT == 2>(stage + (size_t)warp * qbytes, k, st, mb, lane, acc);
            }
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (j < mb) {
                    const float v = warp_sum(acc[j]);
                    if (lane == 0) {
                        float* yp = y + (m0 + j) * ldy + r;
                        *yp = o.accumulate ? fmaf(o.alpha, v, *yp) : o.alpha * v;
                    }
                }
            }
        }
        __syncwarp();  // every lane has read its row of the stage
        if (lane == 0) mbar_arrive(smem_u32(R.empty + slot));
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
// Bytes of a weight row in the stage: Q8_0 k int8 + 16; Q4_K / Q5_K its
// superblocks (144 / 176 B each) padded so that the row stride is 4 (mod 32)
// words.
__host__ __device__ constexpr int64_t mma_row_len(int fmt, int64_t k) {
    return fmt == 0 ? k + 16 : row_qbytes(fmt, k) + 4 * ((4 - row_qbytes(fmt, k) / 4) & 31);
}
__host__ __device__ constexpr size_t mma_stage_bytes(int fmt, int64_t k) {
    return (size_t)kStageRows * mma_row_len(fmt, k) + (fmt == 0 ? (size_t)kStageRows * (k / 16) : 0);
}
// activation planes, block scales and the two reduction buffers (Q8_0)
__host__ __device__ constexpr size_t mma_fixed_bytes(int mt, int64_t k) {
    return (size_t)(4 * mt) * 3 * mma_plane_len(k) + (size_t)(4 * mt) * (k / 32) * 4 +
           (size_t)2 * kWarps * 2 * mt * 32 * 4;
}

template <int FMT, int MT>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1)
    gemv_mma_kernel(const uint8_t* __restrict__ wq, const uint8_t* __restrict__ wd, int64_t n, int64_t k,
                    const void* x, int x_dtype, int64_t m, float* __restrict__ y, int64_t ldy, int slots, int nx,
                    GemvOpts o, uint32_t* __restrict__ err) {
    static_assert(FMT == 0, "Q8_0 only: the K-quants take gemv_hmma_kernel");
    constexpr int MB = 4 * MT;
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, qq = lane & 3;
    const int nblk = (int)(k >> 5);
    const int64_t plm = mma_plane_len(k), rl = mma_row_len(FMT, k);
    const uint32_t qbytes = (uint32_t)row_qbytes(FMT, k);  // one row in global memory
    const uint32_t dbytes = FMT == 0 ? (uint32_t)(k >> 4) : 0u;
    const Ring R = ring_of(smem, slots, nx);
    int8_t* xq = reinterpret_cast<int8_t*>(smem + kBarBytes);             // [MB][3][plm]
    float* sx = reinterpret_cast<float*>(xq + (size_t)MB * 3 * plm);     // [MB][nblk]
    float* red = sx + MB * nblk;                                         // [2][kWarps][2][MT][32]
    uint8_t* ring = smem + kBarBytes + mma_fixed_bytes(MT, k);
    const size_t stage_bytes = mma_stage_bytes(FMT, k);
    const size_t scale_off = (size_t)kStageRows * rl;

    int64_t r0, r1, rb;  // this CTA's rows [r0, r1); row r is row r - rb of matrix wb
    const uint8_t* wb;
    int sg;
    row_range(n, o, r0, r1, wb, rb, sg, wq);
    const int64_t nst = (r1 - r0 + kStageRows - 1) / kStageRows;
    auto issue = [&](int64_t i, int slot) {  // producer lane 0: stage i into `slot`
        const int64_t ra = r0 + i * kStageRows;
        const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
        const uint32_t bar = smem_u32(R.full + slot);
        const uint32_t dst = smem_u32(ring + (size_t)slot * stage_bytes);
        mbar_arrive_expect_tx(bar, rows * (qbytes + dbytes));
        for (uint32_t r = 0; r < rows; r++)
            bulk_load(dst + r * (uint32_t)rl, wb + (ra - rb + r) * (int64_t)qbytes, qbytes, bar);
        if (FMT == 0) bulk_load(dst + (uint32_t)scale_off, wd + ra * (int64_t)dbytes, rows * dbytes, bar);
    };
    if (warp == kWarps && lane == 0) {
        ring_init(R);
        for (int64_t i = 0; i < min(nst, (int64_t)2); i++) {  // the weights never come from an earlier kernel
            const int64_t ra = r0 + i * kStageRows;
            const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
            bulk_prefetch_l2(wb + (ra - rb) * (int64_t)qbytes, rows * qbytes);
            if (FMT == 0) bulk_prefetch_l2(wd + ra * (int64_t)dbytes, rows * dbytes);
        }
    }
    __syncthreads();  // the barriers are initialised

    pdl_wait();
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    const size_t esize = x_dtype == GDN_DTYPE_F32 ? 4 : 2;
    const int64_t xrow = o.swiglu ? 2 * k : k;  // activation elements per row read
    const int64_t ldx = o.ldx ? o.ldx : xrow;   // ... and between rows in memory
    const void* xe = static_cast<const char*>(x) + (size_t)sg * o.x_seg * esize;  // this CTA's matrix's input
    const uint8_t* xs = ring + (size_t)(slots - nx) * stage_bytes;  // the activations, when nx > 0
    if (warp < kWarps)  // rows past mb are staged as zeros (their outputs are not stored)
        consume_activations<FMT, false>(R, xe, x_dtype, ldx, xs, m0, mb, MB, k, warp, lane, xq, (int)plm, sx,
                                        nullptr, o, err);

    if (warp == kWarps) {  // producer
        if (nx == 0) bar_sync(1, (kWarps + 1) * 32);
        if (lane == 0)
            produce(R, nst, issue, static_cast<const uint8_t*>(xe) + (size_t)m0 * ldx * esize, mb,
                    (uint32_t)((size_t)xrow * esize), (size_t)ldx * esize, xs, err);
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
        if (!bad) bad = !__all_sync(0xffffffffu, mbar_wait_sleep(smem_u32(R.full + slot), phase, err));
        const uint8_t* stage = ring + (size_t)slot * stage_bytes;
        const uint16_t* dsc = reinterpret_cast<const uint16_t*>(stage + scale_off);
        float acc[2][MT][4];
#pragma unroll
        for (int g = 0; g < 2; g++)
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
                for (int e = 0; e < 4; e++) acc[g][mt][e] = 0.0f;
#pragma unroll 2
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
        if (lane == 0) mbar_arrive(smem_u32(R.empty + slot));
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
                float* yp = y + (m0 + j) * ldy + r;
                *yp = o.accumulate ? fmaf(o.alpha, sum, *yp) : o.alpha * sum;
            }
        }
        if (++slot == slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
}

template <int FMT, int MT>
int run_mma(const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
            int64_t ldy, int slots, int nx, const GemvOpts& o, size_t smem, cudaStream_t s) {
    const void* fn = (const void*)gemv_mma_kernel<FMT, MT>;
    GDN_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t ctas = std::min<int64_t>(sm_count(), n);
    const dim3 grid((unsigned)ctas, (unsigned)((m + 4 * MT - 1) / (4 * MT)));
    return launch_pdl(FMT == 0 ? "gemv_mma_kernel<q8_0>" : FMT == 1 ? "gemv_mma_kernel<q4_k>" : "gemv_mma_kernel<q5_k>",
                      gemv_mma_kernel<FMT, MT>, grid,
                      dim3((kWarps + 1) * 32), smem, s,
                      static_cast<const uint8_t*>(wq), static_cast<const uint8_t*>(wd), n, k, x, dt, m, y, ldy,
                      slots, nx, o, device_error_word());
}

// ------------------------------------------------- Q4_K / Q5_K on fp16 MMA
//
// A K-quant weight is d sc q - dmin m with integers q < 32 and sc, m < 64, so
// q sc (< 2048) is exact in fp16.  Each activation row's 256-element piece (one
// superblock's columns) is scaled by a power of two 2^E that brings its max |x|
// into [2^14, 2^15) and split into two fp16 parts, x 2^E = hi + lo (22
// significant bits; the sum of the parts is x 2^E to within about 1e-7 of the
// piece's scaled max).  mma.sync m16n8k16 takes A = q sc of the stage's 16
// weight rows and B = 8 activation rows, the hi parts and then the lo parts
// into the same fp32 accumulators, which sum a whole superblock, so that the
// only per-superblock work left is C d 2^-E per output.  The min term
// dmin sum_s m_s X_s (X_s the fp32 sum of sub-block s's activations) is one
// more mma pair per superblock: A = the rows' eight m_s, B = the eight
// X_s 2^(E-5) as hi + lo.  The k order inside an mma is free: k slots 2 t,
// 2 t + 1, 2 t + 8, 2 t + 9 of lane group t hold elements 4 t .. 4 t + 3 of the
// 16-element run, so that both operands are plain 4-element loads.  The 16
// consumer warps split a stage into (superblock, sub-block range) units of all
// 16 rows and add their partial sums through shared memory once per stage.

__host__ __device__ constexpr int64_t h_plane(int64_t k) { return 2 * k + 32; }      // fp16 row, 32 (mod 128) B
__host__ __device__ constexpr int64_t h_sums(int64_t k) { return 16 * (k >> 8) + 16; }  // 8 fp16 per superblock
// floats per warp, [mt][16][8] + 8: the warps a reducing thread reads are 8 banks apart
__host__ __device__ constexpr int h_red_stride(int mt) { return 128 * mt + 8; }
// hi and lo planes, hi and lo sub-block sums, the 2^-E factors, the two reduction buffers
__host__ __device__ constexpr size_t hmma_fixed_bytes(int mt, int64_t k) {
    return (size_t)(8 * mt) * (2 * h_plane(k) + 2 * h_sums(k) + 4 * (k >> 8)) +
           (size_t)2 * kWarps * h_red_stride(mt) * 4;
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {  // lo -> bits 0-15
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ void unpack_h2(uint32_t h, float& lo, float& hi) {
    asm("{.reg .f16 a, b;\n mov.b32 {a, b}, %2;\n cvt.f32.f16 %0, a;\n cvt.f32.f16 %1, b;}"
        : "=f"(lo), "=f"(hi)
        : "r"(h));
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void hmma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}

constexpr uint32_t kH2Magic = 0x64006400u;  // fp16 1024 in both halves: 0x6400 | i = 1024 + i for i < 1024

// Integer bytes b (< 1024) of w at the byte positions of selector sel (two
// bytes) as an exact fp16 pair.
__device__ __forceinline__ uint32_t bytes_h2(uint32_t w, uint32_t sel) {
    return hsub2(__byte_perm(w, 0, sel) | kH2Magic, kH2Magic);
}

// The staged activations of one CTA row of the grid.
struct HPlanes {
    uint8_t* hi;   // [MB][h_plane] fp16 hi parts
    uint8_t* lo;   // [MB][h_plane] fp16 lo parts
    uint8_t* shi;  // [MB][h_sums] sub-block sums 2^(E-5), hi parts
    uint8_t* slo;  // [MB][h_sums] lo parts
    float* sc;     // [MB][k / 256] 2^-E (NaN when the piece holds an inf or NaN)
    int64_t P, SS;
    int nsb;
};

// One warp stages piece c (256 elements, one superblock's columns) of
// activation row j: lane l holds elements 8 l .. 8 l + 7 (sub-block l / 4).
__device__ __forceinline__ void stage_256(const float (&v)[8], bool valid, const HPlanes& h, int j, int c,
                                          int lane) {
    // max |x| of the piece as an integer max of the magnitude bits (a NaN wins)
    uint32_t ab = max(max(max(__float_as_uint(v[0]) & 0x7fffffffu, __float_as_uint(v[1]) & 0x7fffffffu),
                          max(__float_as_uint(v[2]) & 0x7fffffffu, __float_as_uint(v[3]) & 0x7fffffffu)),
                      max(max(__float_as_uint(v[4]) & 0x7fffffffu, __float_as_uint(v[5]) & 0x7fffffffu),
                          max(__float_as_uint(v[6]) & 0x7fffffffu, __float_as_uint(v[7]) & 0x7fffffffu)));
    ab = __reduce_max_sync(0xffffffffu, ab);
    // 2^E = p1 p2 (each a normal power of two; p2 = 1 unless E > 127) and
    // s = 2^-E (subnormal for E > 126); all warp-uniform
    float p1 = 1.0f, p2 = 1.0f, s = 0.0f;
    if (ab >= 0x7f800000u) {
        s = __uint_as_float(0x7fc00000u);  // an inf or NaN: every output of the row becomes NaN
    } else if (ab != 0) {
        const int E = 141 - (int)(ab >> 23);  // max 2^E in [2^14, 2^15); E in [-113, 141]
        const int e1 = min(E, 127), e2 = E - e1;
        p1 = __int_as_float((e1 + 127) << 23);
        p2 = __int_as_float((e2 + 127) << 23);
        s = E <= 126 ? __int_as_float((127 - E) << 23) : __int_as_float(1 << (149 - E));
    }
    float xs[8];
    if (p2 == 1.0f) {
#pragma unroll
        for (int e = 0; e < 8; e++) xs[e] = v[e] * p1;  // exact: a power of two, no overflow
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) xs[e] = (v[e] * p1) * p2;
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        const uint32_t hh = pack_h2(xs[e], xs[e + 1]);
        float ha, hb;
        unpack_h2(hh, ha, hb);
        hw[e >> 1] = hh;
        lw[e >> 1] = pack_h2(xs[e] - ha, xs[e + 1] - hb);  // the differences are exact in fp32
    }
    float t = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    t += __shfl_xor_sync(0xffffffffu, t, 1);  // the sub-block's 32 activations
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    const float ts = (t * p1) * (p2 * 0.03125f);  // X 2^(E-5), |.| < 2^15
    const uint32_t th = pack_h2(ts, 0.0f);
    float thf, unused;
    unpack_h2(th, thf, unused);
    const uint32_t tl = pack_h2(ts - thf, 0.0f);
    if (valid) {
        const size_t off = (size_t)j * h.P + 512 * c + 16 * lane;
        *reinterpret_cast<uint4*>(h.hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(h.lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        if ((lane & 3) == 0) {
            const size_t so = (size_t)j * h.SS + 16 * c + 2 * (lane >> 2);
            *reinterpret_cast<uint16_t*>(h.shi + so) = (uint16_t)(th & 0xFFFFu);
            *reinterpret_cast<uint16_t*>(h.slo + so) = (uint16_t)(tl & 0xFFFFu);
        }
        if (lane == 0) h.sc[j * h.nsb + c] = s;
    }
}

// stage_rows for the fp16 planes: the 256-element pieces of all rows form one
// list, warp w takes pieces w, w + kWarps, ..., U at a time.
template <bool SMEM, int U>
__device__ __forceinline__ void stage_f16_rows(const void* x, int x_dtype, int64_t ldx, int64_t m0, int mb, int rows,
                                               int64_t k, int warp, int lane, const HPlanes& h, const GemvOpts& o) {
    const int npc = h.nsb;
    const size_t es = x_dtype == GDN_DTYPE_F32 ? 4 : 2;
    const char* x0 = static_cast<const char*>(x) + (SMEM ? 0 : (size_t)m0 * ldx * es);
    const bool vec = x_dtype == GDN_DTYPE_F32 && (reinterpret_cast<uintptr_t>(x0) & 15) == 0 &&
                     ((size_t)ldx * 4) % 16 == 0;
    bool announced = SMEM;
    int j = 0, c = warp;
    while (c >= npc && j < rows) {
        c -= npc;
        j++;
    }
    while (j < rows) {
        float v[U][8];
        int ju[U], cu[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            ju[u] = j;
            cu[u] = c;
            const int64_t e = 256 * (int64_t)c + 8 * lane;
#pragma unroll
            for (int i = 0; i < 8; i++) v[u][i] = 0.0f;
            if (j < rows && j < mb) {
                const char* xr = x0 + (size_t)j * ldx * es;
                if (o.swiglu) {
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const float4 a = swiglu4(xr, e + 4 * q, k, o);
                        v[u][4 * q + 0] = a.x, v[u][4 * q + 1] = a.y, v[u][4 * q + 2] = a.z, v[u][4 * q + 3] = a.w;
                    }
                } else if (vec) {
                    const float4 a = *reinterpret_cast<const float4*>(xr + (size_t)e * 4);
                    const float4 b = *reinterpret_cast<const float4*>(xr + (size_t)(e + 4) * 4);
                    v[u][0] = a.x, v[u][1] = a.y, v[u][2] = a.z, v[u][3] = a.w;
                    v[u][4] = b.x, v[u][5] = b.y, v[u][6] = b.z, v[u][7] = b.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) v[u][i] = load_act(xr, x_dtype, (size_t)e + i);
                }
            }
            c += kWarps;
            while (c >= npc && j < rows) {
                c -= npc;
                j++;
            }
        }
        if (!announced) {
            bar_arrive(1, (kWarps + 1) * 32);
            announced = true;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const bool valid = ju[u] < rows;
            stage_256(v[u], valid, h, valid ? ju[u] : 0, valid ? cu[u] : 0, lane);
        }
    }
    if (!announced) bar_arrive(1, (kWarps + 1) * 32);
}

// consume_activations for the fp16 planes.
__device__ __forceinline__ bool consume_activations_f16(const Ring& R, const void* x, int x_dtype, int64_t ldx,
                                                        const uint8_t* xs, int64_t m0, int mb, int rows, int64_t k,
                                                        int warp, int lane, const HPlanes& h, const GemvOpts& o,
                                                        uint32_t* err) {
    bool ok = true;
    if (R.nx > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_sleep(smem_u32(R.xbar), 0, err));
        if (ok)
            stage_f16_rows<true, kSmemBatch>(xs, x_dtype, o.swiglu ? 2 * k : k, 0, mb, rows, k, warp, lane, h, o);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(R.xdone));
    } else {
        stage_f16_rows<false, kStageBatch>(x, x_dtype, ldx, m0, mb, rows, k, warp, lane, h, o);
    }
    bar_sync(2, kWarps * 32);
    return ok;
}

// q sc of sub-blocks 2 cg (low nibbles: rows' A registers 0-3 of `lo`) and 2 cg
// + 1 (high nibbles: `hi`) for the 4 elements of each of this lane's two weight
// rows (gq: word w0, gq + 8: w1) in one 16-element chunk, as the A fragment
// (row gq, k slots 2 qq ..), (gq + 8, 2 qq ..), (gq, 2 qq + 8 ..), (gq + 8, 2 qq + 8 ..).
template <int FMT>
__device__ __forceinline__ void k_quant_a(uint32_t w0, uint32_t w1, uint32_t hw0, uint32_t hw1, int cg,
                                          const uint32_t (&SA)[2], const uint32_t (&NA)[2], const uint32_t (&SB)[2],
                                          const uint32_t (&NB)[2], uint32_t (&lo)[4], uint32_t (&hi)[4]) {
    const uint32_t w[2] = {w0, w1}, hw[2] = {hw0, hw1};
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint32_t t01 = __byte_perm(w[r], 0, 0x4140), t23 = __byte_perm(w[r], 0, 0x4342);
        uint32_t vl0 = (t01 & 0x000F000Fu) | kH2Magic, vl1 = (t23 & 0x000F000Fu) | kH2Magic;
        uint32_t vh0 = (t01 & 0x00F000F0u) | kH2Magic, vh1 = (t23 & 0x00F000F0u) | kH2Magic;
        if (FMT == 2) {  // fifth bits: bit 2 cg (low) and 2 cg + 1 (high) of each qh byte
            const uint32_t h01 = __byte_perm(hw[r], 0, 0x4140), h23 = __byte_perm(hw[r], 0, 0x4342);
            vl0 |= ((h01 >> (2 * cg)) & 0x00010001u) << 4;
            vl1 |= ((h23 >> (2 * cg)) & 0x00010001u) << 4;
            vh0 |= ((h01 >> (2 * cg + 1)) & 0x00010001u) << 8;
            vh1 |= ((h23 >> (2 * cg + 1)) & 0x00010001u) << 8;
        }
        // (1024 + q) sc - 1024 sc and (1024 + 16 q) sc / 16 - 64 sc: q sc, exact
        lo[r] = hfma2(vl0, SA[r], NA[r]);
        lo[2 + r] = hfma2(vl1, SA[r], NA[r]);
        hi[r] = hfma2(vh0, SB[r], NB[r]);
        hi[2 + r] = hfma2(vh1, SB[r], NB[r]);
    }
}

// Sub-block pair cg of a unit: the two 16-element chunks of sub-blocks 2 cg and
// 2 cg + 1 of the stage's 16 weight rows (A) against every m-tile of
// activations (B: hi parts, then lo parts, into the same accumulators).  blk0
// / blk1 are this lane's rows' superblock in the stage, sc_lo / sc_hi their
// eight 6-bit scales, one per byte.
template <int FMT, int MT>
__device__ __forceinline__ void hmma_pair(int cg, uint32_t blk0, uint32_t blk1, const uint32_t (&sc_lo)[2],
                                          const uint32_t (&sc_hi)[2], int qq, uint32_t sbo, const uint32_t (&hrow)[MT],
                                          const uint32_t (&lrow)[MT], float (&C)[MT][4]) {
    constexpr int kQs = FMT == 2 ? 48 : 16;
    const uint32_t bl = (uint32_t)(2 * cg) & 3u;  // byte of sub-block 2 cg; 2 cg + 1 is the next
    uint32_t SA[2], NA[2], SB[2], NB[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint32_t scw = cg < 2 ? sc_lo[r] : sc_hi[r];
        SA[r] = bytes_h2(scw, 0x4040u | bl | (bl << 8));
        const uint32_t sb1 = bytes_h2(scw, 0x4040u | (bl + 1) | ((bl + 1) << 8));
        NA[r] = hmul2(SA[r], 0xE400E400u);   // -1024 sc
        SB[r] = hmul2(sb1, 0x2C002C00u);     // sc / 16
        NB[r] = hmul2(sb1, 0xD400D400u);     // -64 sc
    }
#pragma unroll
    for (int ch = 0; ch < 2; ch++) {
        // quant bytes 32 cg + 16 ch + 4 qq ..: low nibbles = elements of sub-block
        // 2 cg, high nibbles = the same elements of 2 cg + 1
        const uint32_t qo = kQs + 32 * cg + 16 * ch;  // blk0 / blk1 include 4 qq
        const uint32_t w0 = lds32(blk0 + qo), w1 = lds32(blk1 + qo);
        uint32_t hw0 = 0, hw1 = 0;
        if (FMT == 2) {
            hw0 = lds32(blk0 + 16 + 16 * ch);
            hw1 = lds32(blk1 + 16 + 16 * ch);
        }
        uint32_t alo[4], ahi[4];
        k_quant_a<FMT>(w0, w1, hw0, hw1, cg, SA, NA, SB, NB, alo, ahi);
        const uint32_t eo = sbo + 2 * (64 * cg + 16 * ch);  // byte offset of the chunk of sub-block 2 cg
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            const uint2 h0 = lds64(hrow[mt] + eo), l0 = lds64(lrow[mt] + eo);
            const uint2 h1 = lds64(hrow[mt] + eo + 64), l1 = lds64(lrow[mt] + eo + 64);
            hmma_16816(C[mt], alo, h0.x, h0.y);
            hmma_16816(C[mt], alo, l0.x, l0.y);
            hmma_16816(C[mt], ahi, h1.x, h1.y);
            hmma_16816(C[mt], ahi, l1.x, l1.y);
        }
    }
}

// FMT 1: Q4_K, 2: Q5_K; 8 MT activation rows per CTA row of the grid.
template <int FMT, int MT>
__global__ void __launch_bounds__((kWarps + 1) * 32, 1)
    gemv_hmma_kernel(const uint8_t* __restrict__ wq, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                     float* __restrict__ y, int64_t ldy, int slots, int nx, GemvOpts o, uint32_t* __restrict__ err) {
    static_assert(FMT == 1 || FMT == 2, "K-quants only");
    static_assert(MT == 1 || MT == 2, "one or two m-tiles");
    constexpr int MB = 8 * MT;
    constexpr int kSb = FMT == 2 ? 176 : 144;
    constexpr int RW = h_red_stride(MT);
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, qq = lane & 3;
    const int nsb = (int)(k >> 8);
    const int64_t rl = mma_row_len(FMT, k);
    const uint32_t qbytes = (uint32_t)row_qbytes(FMT, k);
    const Ring R = ring_of(smem, slots, nx);
    HPlanes hp;
    hp.P = h_plane(k);
    hp.SS = h_sums(k);
    hp.nsb = nsb;
    hp.hi = smem + kBarBytes;
    hp.lo = hp.hi + MB * hp.P;
    hp.shi = hp.lo + MB * hp.P;
    hp.slo = hp.shi + MB * hp.SS;
    hp.sc = reinterpret_cast<float*>(hp.slo + MB * hp.SS);
    float* red = hp.sc + MB * nsb;  // [2][kWarps][RW]
    uint8_t* ring = smem + kBarBytes + hmma_fixed_bytes(MT, k);
    const size_t stage_bytes = mma_stage_bytes(FMT, k);

    int64_t r0, r1, rb;  // this CTA's rows [r0, r1); row r is row r - rb of matrix wb
    const uint8_t* wb;
    int sg;
    row_range(n, o, r0, r1, wb, rb, sg, wq);
    const int64_t nst = (r1 - r0 + kStageRows - 1) / kStageRows;
    auto issue = [&](int64_t i, int slot) {  // producer lane 0: stage i into `slot`
        const int64_t ra = r0 + i * kStageRows;
        const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
        const uint32_t bar = smem_u32(R.full + slot);
        const uint32_t dst = smem_u32(ring + (size_t)slot * stage_bytes);
        mbar_arrive_expect_tx(bar, rows * qbytes);
        if (o.kseg) {  // k-segments: row r = the matrices' rows r side by side
            const uint32_t qs = qbytes / (uint32_t)o.kseg;
            for (uint32_t r = 0; r < rows; r++)
                for (int sgm = 0; sgm < o.kseg; sgm++)
                    bulk_load(dst + r * (uint32_t)rl + (uint32_t)sgm * qs, o.seg[sgm] + (ra + r) * (int64_t)qs, qs,
                              bar);
        } else {
            for (uint32_t r = 0; r < rows; r++)
                bulk_load(dst + r * (uint32_t)rl, wb + (ra - rb + r) * (int64_t)qbytes, qbytes, bar);
        }
    };
    if (warp == kWarps && lane == 0) {
        ring_init(R);
        for (int64_t i = 0; i < min(nst, (int64_t)2); i++) {  // the weights never come from an earlier kernel
            const int64_t ra = r0 + i * kStageRows;
            const uint32_t rows = (uint32_t)min((int64_t)kStageRows, r1 - ra);
            if (o.kseg) {
                const uint32_t qs = qbytes / (uint32_t)o.kseg;
                for (int sgm = 0; sgm < o.kseg; sgm++) bulk_prefetch_l2(o.seg[sgm] + ra * (int64_t)qs, rows * qs);
            } else {
                bulk_prefetch_l2(wb + (ra - rb) * (int64_t)qbytes, rows * qbytes);
            }
        }
    }
    __syncthreads();  // the barriers are initialised

    pdl_wait();
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    const size_t esize = x_dtype == GDN_DTYPE_F32 ? 4 : 2;
    const int64_t xrow = o.swiglu ? 2 * k : k;  // activation elements per row read
    const int64_t ldx = o.ldx ? o.ldx : xrow;   // ... and between rows in memory
    const void* xe = static_cast<const char*>(x) + (size_t)sg * o.x_seg * esize;  // this CTA's matrix's input
    const uint8_t* xs = ring + (size_t)(slots - nx) * stage_bytes;  // the activations, when nx > 0
    if (warp < kWarps)  // rows past mb are not staged: their A rows only reach outputs that are not stored
        consume_activations_f16(R, xe, x_dtype, ldx, xs, m0, mb, mb, k, warp, lane, hp, o, err);

    if (warp == kWarps) {  // producer
        if (nx == 0) bar_sync(1, (kWarps + 1) * 32);
        if (lane == 0)
            produce(R, nst, issue, static_cast<const uint8_t*>(xe) + (size_t)m0 * ldx * esize, mb,
                    (uint32_t)((size_t)xrow * esize), (size_t)ldx * esize, xs, err);
        return;
    }

    // Units of a stage: (superblock sb, part p of np = 2^lnp: sub-block pairs
    // [4 p / np, 4 (p + 1) / np)) of all 16 weight rows; np grows for short
    // rows so that the 16 warps have work.  Warp w takes units w, w + 16, ...
    const int lnp = nsb >= 16 ? 0 : nsb >= 8 ? 1 : 2;
    const int nu = nsb << lnp;
    // shared-memory addresses: this lane's activation fragments, sums, factors
    uint32_t hrow[MT], lrow[MT];
#pragma unroll
    for (int mt = 0; mt < MT; mt++) {
        hrow[mt] = smem_u32(hp.hi) + (uint32_t)((8 * mt + gq) * hp.P + 8 * qq);
        lrow[mt] = smem_u32(hp.lo) + (uint32_t)((8 * mt + gq) * hp.P + 8 * qq);
    }
    const uint32_t shi_s = smem_u32(hp.shi), slo_s = smem_u32(hp.slo), sc_s = smem_u32(hp.sc);
    // The consumers meet at a named barrier every stage, so none may leave the
    // loop alone: a warp whose wait gave up (the error word is set) stops
    // waiting and computing but keeps arriving, so that every warp ends.
    bool bad = false;
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t i = 0; i < nst; i++) {
        if (!bad) bad = !__all_sync(0xffffffffu, mbar_wait_sleep(smem_u32(R.full + slot), phase, err));
        const uint32_t stage = smem_u32(ring) + (uint32_t)(slot * stage_bytes);
        // this lane's outputs: weight rows gq, gq + 8 (e = 0, 1 / 2, 3) x activation
        // rows 8 mt + 2 qq, + 1 (e = 0, 2 / 1, 3)
        float acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;
        for (int u = bad ? nu : warp; u < nu; u += kWarps) {
            const int sb = u >> lnp, p = u & ((1 << lnp) - 1);
            const uint32_t blk0 = stage + (uint32_t)(gq * rl + sb * kSb);  // this lane's A rows gq, gq + 8
            const uint32_t blk1 = blk0 + (uint32_t)(8 * rl);
            uint32_t hdr[2], W1[2], W2[2], sc_lo[2], sc_hi[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const uint32_t b = r ? blk1 : blk0;
                hdr[r] = lds32(b);
                const uint32_t W0 = lds32(b + 4);
                W1[r] = lds32(b + 8);
                W2[r] = lds32(b + 12);
                sc_lo[r] = W0 & 0x3F3F3F3Fu;  // the 6-bit scales of sub-blocks 0-3 and 4-7, one per byte
                sc_hi[r] = (W2[r] & 0x0F0F0F0Fu) | ((W0 >> 2) & 0x30303030u);
            }
            float C[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; mt++) C[mt][0] = C[mt][1] = C[mt][2] = C[mt][3] = 0.0f;
            const uint32_t sbo = 512u * (uint32_t)sb;  // byte offset of the superblock's activations
            const uint32_t q0 = blk0 + 4 * qq, q1 = blk1 + 4 * qq;
            if (lnp == 0) {  // the whole superblock: selectors and branches fold
#pragma unroll
                for (int cg = 0; cg < 4; cg++) hmma_pair<FMT, MT>(cg, q0, q1, sc_lo, sc_hi, qq, sbo, hrow, lrow, C);
            } else {
                const int cg0 = p << (2 - lnp);
                for (int cg = cg0; cg < cg0 + (4 >> lnp); cg++)
                    hmma_pair<FMT, MT>(cg, q0, q1, sc_lo, sc_hi, qq, sbo, hrow, lrow, C);
            }
            // the min term (unit part 0): A = m of sub-blocks 4 qq .. 4 qq + 3 for
            // lane groups 0 and 1, zero for 2 and 3 (k slots 4-7 and 12-15 unused);
            // B = the activations' sub-block sums, hi then lo
            float Cm[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; mt++) Cm[mt][0] = Cm[mt][1] = Cm[mt][2] = Cm[mt][3] = 0.0f;
            if (p == 0) {
                uint32_t am[4] = {0u, 0u, 0u, 0u};
                if (qq < 2) {
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        const uint32_t mw = qq == 0 ? (W1[r] & 0x3F3F3F3Fu)
                                                    : (((W2[r] >> 4) & 0x0F0F0F0Fu) | ((W1[r] >> 2) & 0x30303030u));
                        am[r] = bytes_h2(mw, 0x4140);
                        am[2 + r] = bytes_h2(mw, 0x4342);
                    }
                }
#pragma unroll
                for (int mt = 0; mt < MT; mt++) {
                    uint2 sh = make_uint2(0u, 0u), sl = make_uint2(0u, 0u);
                    if (qq < 2) {
                        const uint32_t so = (uint32_t)((8 * mt + gq) * hp.SS + 16 * sb + 8 * qq);
                        sh = lds64(shi_s + so);
                        sl = lds64(slo_s + so);
                    }
                    hmma_16816(Cm[mt], am, sh.x, sh.y);
                    hmma_16816(Cm[mt], am, sl.x, sl.y);
                }
            }
            // (C d - 32 dmin Cm) 2^-E per output
            float d[2], nm[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                d[r] = fp16_bits_to_float((uint16_t)(hdr[r] & 0xFFFFu));
                nm[r] = -32.0f * fp16_bits_to_float((uint16_t)(hdr[r] >> 16));
            }
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                const float s0 = lds_f32(sc_s + 4u * (uint32_t)((8 * mt + 2 * qq) * nsb + sb));
                const float s1 = lds_f32(sc_s + 4u * (uint32_t)((8 * mt + 2 * qq + 1) * nsb + sb));
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int r = e >> 1;
                    const float v = fmaf(nm[r], Cm[mt][e], C[mt][e] * d[r]);
                    acc[mt][e] = fmaf(v, (e & 1) ? s1 : s0, acc[mt][e]);
                }
            }
        }
        __syncwarp();  // every lane has read the stage
        if (lane == 0) mbar_arrive(smem_u32(R.empty + slot));
        // partials as [mt][weight row][activation row]
        float* rw = red + ((size_t)(i & 1) * kWarps + warp) * RW;
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
            *reinterpret_cast<float2*>(rw + mt * 128 + gq * 8 + 2 * qq) = make_float2(acc[mt][0], acc[mt][1]);
            *reinterpret_cast<float2*>(rw + mt * 128 + (gq + 8) * 8 + 2 * qq) = make_float2(acc[mt][2], acc[mt][3]);
        }
        bar_sync(3, kWarps * 32);  // every warp's partials of this stage
        {   // output t of the 128 MT: TPO = 4 / MT consecutive threads add warps q, q + TPO, ...
            constexpr int TPO = 4 / MT;
            const float* rs = red + (size_t)(i & 1) * kWarps * RW;
            const int t = threadIdx.x / TPO, q = threadIdx.x % TPO;
            float sum = 0.0f;
#pragma unroll
            for (int w = q; w < kWarps; w += TPO) sum += rs[(size_t)w * RW + t];
#pragma unroll
            for (int o2 = 1; o2 < TPO; o2 <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o2);
            const int row = (t >> 3) & 15, j = 8 * (t >> 7) + (t & 7);
            const int64_t r = r0 + i * kStageRows + row;
            if (q == 0 && j < mb && r < r1) {
                float* yp = y + (m0 + j) * ldy + r;
                *yp = o.accumulate ? fmaf(o.alpha, sum, *yp) : o.alpha * sum;
            }
        }
        if (++slot == slots) {
            slot = 0;
            phase ^= 1u;
        }
    }
}

template <int FMT, int MT>
int run_hmma(const void* wq, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y, int64_t ldy, int slots,
             int nx, const GemvOpts& o, size_t smem, cudaStream_t s) {
    const void* fn = (const void*)gemv_hmma_kernel<FMT, MT>;
    GDN_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t ctas = std::min<int64_t>(sm_count(), n);
    const dim3 grid((unsigned)ctas, (unsigned)((m + 8 * MT - 1) / (8 * MT)));
    return launch_pdl(FMT == 1 ? "gemv_hmma_kernel<q4_k>" : "gemv_hmma_kernel<q5_k>", gemv_hmma_kernel<FMT, MT>, grid,
                      dim3((kWarps + 1) * 32), smem, s, static_cast<const uint8_t*>(wq), n, k, x, dt, m, y, ldy,
                      slots, nx, o, device_error_word());
}

template <int FMT, int MB>
int run(const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
        int64_t ldy, int slots, int nx, const GemvOpts& o, size_t smem, cudaStream_t s) {
    const void* fn = (const void*)gemv_stream_kernel<FMT, MB>;
    GDN_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t ctas = std::min<int64_t>(sm_count(), n);
    const dim3 grid((unsigned)ctas, (unsigned)((m + MB - 1) / MB));
    return launch_pdl(FMT == 0 ? "gemv_stream_kernel<q8_0>" : FMT == 1 ? "gemv_stream_kernel<q4_k>"
                                                                    : "gemv_stream_kernel<q5_k>",
                      gemv_stream_kernel<FMT, MB>, grid, dim3((kWarps + 1) * 32), smem, s,
                      static_cast<const uint8_t*>(wq), static_cast<const uint8_t*>(wd), n, k, x, dt, m, y, ldy,
                      slots, nx, o, device_error_word());
}

// Ring slots that first hold the activations (one bulk copy of the CTA's
// rows): 0 -- load them from global memory instead -- unless x is 16-byte
// aligned and they leave at least one slot for the weights.
static int activation_slots(const void* x, int dt, int64_t xrow, int mb, size_t stage_bytes, int slots) {
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return 0;
    const size_t bytes = (size_t)mb * xrow * (dt == GDN_DTYPE_F32 ? 4 : 2);
    const int nx = (int)((bytes + stage_bytes - 1) / stage_bytes);
    return nx < slots ? nx : 0;
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
    const int64_t stage = (int64_t)kStageRows * (fmt == 0 ? k + k / 16 : row_qbytes(fmt, k));
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
static int plan_mma(int fmt, const void* wq, const void* wd, int64_t k, int64_t m, int* mt_out, int* slots_out,
                    size_t* smem_out) {
    if (fmt != 0 || m < 3 || (m + 3) / 4 > 65535 || k < 512 || (k & 511) != 0) return 0;
    if ((reinterpret_cast<uintptr_t>(wq) & 15) != 0) return 0;
    if (fmt == 0 && (reinterpret_cast<uintptr_t>(wd) & 15) != 0) return 0;
    for (int mt = m > 4 ? 2 : 1; mt >= 1; mt--) {
        const size_t base = kBarBytes + mma_fixed_bytes(mt, k);
        if (base >= kSmemLimit) continue;
        const int slots = (int)std::min<size_t>(kMaxSlots, (kSmemLimit - base) / mma_stage_bytes(fmt, k));
        if (slots < 2) continue;
        *mt_out = mt;
        *slots_out = slots;
        *smem_out = base + (size_t)slots * mma_stage_bytes(fmt, k);
        return 1;
    }
    return 0;
}

// The fp16-MMA plan (Q4_K / Q5_K, three or more activation rows): 2 m-tiles
// (16 rows per CTA) for more than 8 rows when 2 stages fit beside them, else 1.
static int plan_hmma(int fmt, const void* wq, int64_t k, int64_t m, int* mt_out, int* slots_out, size_t* smem_out) {
    if (fmt == 0 || m < 3 || (m + 7) / 8 > 65535 || k < 256 || (k & 255) != 0) return 0;
    if ((reinterpret_cast<uintptr_t>(wq) & 15) != 0) return 0;
    for (int mt = m > 8 ? 2 : 1; mt >= 1; mt--) {
        const size_t base = kBarBytes + hmma_fixed_bytes(mt, k);
        if (base >= kSmemLimit) continue;
        const int slots = (int)std::min<size_t>(kMaxSlots, (kSmemLimit - base) / mma_stage_bytes(fmt, k));
        if (slots < 2) continue;
        *mt_out = mt;
        *slots_out = slots;
        *smem_out = base + (size_t)slots * mma_stage_bytes(fmt, k);
        return 1;
    }
    return 0;
}

// mma: 1 = IMMA (Q8_0), 2 = fp16 MMA (K-quants), 0 = the streamed dp4a kernel.
template <int FMT>
static int run_fmt(int mb, int mma, const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt,
                   int64_t m, float* y, int64_t ldy, int slots, int nx, const GemvOpts& o, size_t smem,
                   cudaStream_t s) {
    if (FMT == 0 && mma == 1)
        return mb == 2 ? run_mma<0, 2>(wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s)
                       : run_mma<0, 1>(wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
    if (FMT != 0 && mma == 2)
        return mb == 2 ? run_hmma<FMT != 0 ? FMT : 1, 2>(wq, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s)
                       : run_hmma<FMT != 0 ? FMT : 1, 1>(wq, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
    switch (mb) {
        case 1: return run<FMT, 1>(wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
        case 2: return run<FMT, 2>(wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
        case 4: return run<FMT, 4>(wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
        default: return run<FMT, 8>(wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
    }
}

int launch_gemv_stream(int fmt, const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int dt,
                       int64_t m, float* y, int64_t ldy, cudaStream_t s, const GemvOpts& o) {
    if (fmt < 0 || fmt > 2) return GDN_ERR_TYPE;
    if (o.nseg) {
        if (fmt == 0 || o.nseg > kGemvMaxSeg || o.seg_rows <= 0 || n != o.nseg * o.seg_rows) return GDN_ERR_ARG;
        for (int i = 0; i < o.nseg; i++)
            if (!o.seg[i] || (reinterpret_cast<uintptr_t>(o.seg[i]) & 15) != 0) return GDN_ERR_ARG;
        if (std::min<int64_t>(sm_count(), n) < o.nseg) return GDN_ERR_SHAPE;
    }
    if (o.kseg) {  // K-quant matrices side by side along k, SwiGLU inputs, no row segments
        if (fmt == 0 || !o.swiglu || o.nseg || o.kseg > kGemvMaxSeg || k % o.kseg != 0 || (k / o.kseg) % 256 != 0)
            return GDN_ERR_ARG;
        for (int i = 0; i < o.kseg; i++)
            if (!o.seg[i] || (reinterpret_cast<uintptr_t>(o.seg[i]) & 15) != 0) return GDN_ERR_ARG;
    }
    if (o.swiglu && (dt != GDN_DTYPE_F32 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)) return GDN_ERR_ARG;
    const int64_t xrow = o.swiglu ? 2 * k : k;
    // strided or offset activations: every row start 16-byte aligned for the bulk copies
    const size_t es = dt == GDN_DTYPE_F32 ? 4 : 2;
    if ((o.ldx && (o.ldx < xrow || (o.ldx * es) % 16)) || (o.x_seg * es) % 16) return GDN_ERR_ARG;
    int mb = 0, slots = 0, nx = 0, mma = 0;
    size_t smem = 0;
    if (n > 0 && plan_mma(fmt, wq, wd, k, m, &mb, &slots, &smem)) {
        mma = 1;
        nx = activation_slots(x, dt, xrow, 4 * mb, mma_stage_bytes(fmt, k), slots);
    } else if (n > 0 && plan_hmma(fmt, wq, k, m, &mb, &slots, &smem)) {
        mma = 2;
        nx = activation_slots(x, dt, xrow, 8 * mb, mma_stage_bytes(fmt, k), slots);
    } else {
        if (!plan(fmt, wq, wd, k, m, &mb, &slots, &smem)) return GDN_ERR_SHAPE;
        if (n <= 0) return GDN_OK;
        const size_t stage = (size_t)kStageRows * (fmt == 0 ? k + k / 16 : row_qbytes(fmt, k));
        nx = activation_slots(x, dt, xrow, mb, stage, slots);
    }
    if (fmt == 0) return run_fmt<0>(mb, mma, wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
    if (fmt == 1) return run_fmt<1>(mb, mma, wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
    return run_fmt<2>(mb, mma, wq, wd, n, k, x, dt, m, y, ldy, slots, nx, o, smem, s);
}

bool gemv_stream_fits(int fmt, const void* wq, const void* wd, int64_t k, int64_t m) {
    int mb, slots;
    size_t smem;
    return plan(fmt, wq, wd, k, m, &mb, &slots, &smem) != 0;
}

}  // namespace gdn
