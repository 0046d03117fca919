// Q8_0 dequant-GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   y[m][n] = sum_k a[m][k] * W[n][k]      (y row stride ldy)
//   a: fp16 or bf16 [m][k] activations (tokens / sequences), row-major
//   W: Q8_0 planes qs [n][k] int8 and d [n][k/32] fp16 (see gdn_q8_0_repack)
//
// This is the batched form of quant_matvec type 8 (engine/runtime/transformer.h
// :157-194; the reference GPU kernel is engine/runtime/gpu_offload.cu:152-199).
// The weights are never materialised in HBM: each int8 tile arrives in shared
// memory by TMA and is dequantised there straight into the MMA operand layout.
//
// Weight precision.  w = d*q is exact in fp32 (11 x 7 significant bits).
//   single:  one operand w_hi = round(w) in the activation type (fp16: 11 bits,
//            bf16: 8 bits), one MMA per K step.
//   split:   (fp16 only) w = w_hi + w_lo * 2^-11 with w_hi = RN(q*d) and
//            w_lo = RN(q*(2^11 d) - 2^11 w_hi) -- both exact, so w_hi + w_lo*2^-11
//            is w.  Two MMAs into two TMEM accumulators, y = acc_hi +
//            acc_lo * 2^-11: the product differs from an fp32 GEMV only by
//            summation order (the decode path's 1e-3 parity bound).
//
// One CTA computes MT x 128 rows (tokens) by BN columns (weight rows) over its
// K range in BK = 64 steps:
//   warp 0      TMA producer of the activation tiles (128B swizzle)
//   warp 1      TMEM allocator; lane 0 issues tcgen05.mma (M=128, N=BN, K=16)
//   warp 2      TMA producer of the int8 weight tiles
//   warps 3-10  dequant int8 -> operand type into the swizzled B tile(s), shared
//               by the MT activation tiles (one mbarrier arrival per warp); then
//               the epilogue (tcgen05.ld TMEM -> registers -> staged in shared
//               memory -> coalesced global fp32), two warps per TMEM lane quadrant
// The three rings (activation, dequantised weight, raw weight) have separate
// full/empty mbarriers, so the raw weight slot is refilled as soon as the
// dequant warps have read it rather than after the MMA -- the weight stream
// from HBM runs several k-tiles ahead of the tensor cores.
// Split-K (grid.z > 1) writes fp32 partials that a second kernel sums in a
// fixed order, so results do not depend on scheduling.
//
// Q4_K weights (Q4K = true) use the same pipeline: the raw ring holds whole
// 144-byte superblock rows (256 weights, four k-tiles), the dequant warps read
// a superblock row once, release the slot and expand each 64-weight quarter
// with the reference's formula w = (d sc) q - (dmin m) (gpu_offload.cu:237-250,
// each operation rounded once) into the operand tiles.
#include <cuda.h>
#include <algorithm>
#include <string.h>
#include <type_traits>
#include "gdn_common.cuh"
#include "ptx_sm100.cuh"
#include "quant.cuh"

namespace gdn {

using namespace sm100;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kDeqThreads = 256;
constexpr int kDeqWarp0 = 3;  // warps 0: A producer, 1: MMA issuer + TMEM owner, 2: weight producer
constexpr int kDeqWarps = kDeqThreads / 32;
constexpr int kThreads = 32 * kDeqWarp0 + kDeqThreads;
constexpr int kWin = 8;  // k-tiles per scale window (16 fp16 scales = 32 bytes per row)

// Shared memory: three rings, each with its own depth --
//   A   [SA]  MT activation tiles (128 x 64, 128B-swizzled), freed by the MMA
//   B16 [S16] the dequantised weight tile(s) (hi, and lo when split), freed by the MMA
//   B8  [S8]  the raw int8 weight tile, freed as soon as the dequant warps have read it
constexpr int kQ4kBytes = 144;   // Q4_K superblock: fp16 d, fp16 dmin, 12 scale bytes, 128 quant bytes
constexpr int kQ4kTiles = 4;     // k-tiles per superblock (256 / BK)

template <int BN, int MT, int SA, int S16, int S8, bool SPLIT, bool Q4K = false>
struct TcLayout {
    static constexpr uint32_t A_BYTES = BM * BK * 2;  // one 128-row activation tile
    static constexpr uint32_t B16_BYTES = BN * BK * 2;
    static constexpr uint32_t B8_BYTES = Q4K ? BN * kQ4kBytes : BN * BK;  // raw slot: a k-tile / a superblock
    static constexpr int NB = SPLIT ? 2 : 1;
    static constexpr uint32_t A_OFF = 0;
    static constexpr uint32_t B16_OFF = A_OFF + SA * MT * A_BYTES;
    static constexpr uint32_t B8_OFF = B16_OFF + S16 * NB * B16_BYTES;
    static constexpr uint32_t BAR_OFF = B8_OFF + S8 * B8_BYTES;
    // a_full[SA] a_empty[SA] b16_full[S16] b16_empty[S16] b8_full[S8] b8_empty[S8] accf
    static constexpr uint32_t NBARS = 2 * SA + 2 * S16 + 2 * S8 + 1;
    static constexpr uint32_t TMEM_SLOT_OFF = BAR_OFF + NBARS * 8;
    static constexpr uint32_t BYTES = TMEM_SLOT_OFF + 16;
    static constexpr size_t SMEM = BYTES + 1024;  // + alignment slack
    // Each M tile's accumulator(s) start on a 128-column boundary; TMEM is allocated
    // in powers of two columns (>= 32)
    static constexpr uint32_t ACC_STRIDE = (NB * BN + 127) / 128 * 128;
    static constexpr uint32_t ACC_COLS = MT == 1 ? NB * BN : MT * ACC_STRIDE;
    static constexpr uint32_t TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                          : ACC_COLS <= 256 ? 256 : 512;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(ACC_COLS <= 512, "TMEM budget");
    // 96-column tiles (single operand, Q8_0) fill one wave where 128 would leave SMs idle
    static_assert((BN % 64 == 0 && BN <= 256) || (BN == 96 && !SPLIT && !Q4K), "BN");
    static_assert(Q4K || (B8_OFF % 1024 == 0 && B8_BYTES % 1024 == 0), "64B-swizzled raw tiles start on swizzle atoms");
    static_assert(B8_OFF % 128 == 0 && B8_BYTES % 128 == 0, "TMA destinations");
    static_assert(SA * MT * A_BYTES >= 8u * 32u * 36u * 4u, "epilogue staging lives in the activation ring");
};

// 16 int8 weights (uint4) times scale -> 16 operand elements: hi[8] words (and
// lo[8] when split).
template <bool BF16, bool SPLIT>
__device__ __forceinline__ void dequant16(const uint4 q, uint16_t dbits, uint32_t (&hi)[8], uint32_t (&lo)[8]) {
    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
    const __half dh = __ushort_as_half(dbits);
    if constexpr (!BF16) {
        // byte u = q + 128 -> fp16 bits 0x6400 | u = 1024 + u; minus 1152 gives q exactly
        const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));
        const __half2 d2 = __half2half2(dh);
        const bool fast = !SPLIT || fabsf(__half2float(dh)) < 0.25f;  // keeps 2^11 * q * d in fp16 range
        if (fast) {
            const __half2 d2s = __hmul2(d2, __half2half2(__float2half_rn(2048.0f)));
            const __half2 m2048 = __half2half2(__float2half_rn(-2048.0f));
#pragma unroll
            for (int j = 0; j < 4; j++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    uint32_t pb = __byte_perm(w[j], 0x64646464u, e ? 0x4342 : 0x4140);
                    const __half2 qh = __hsub2(*reinterpret_cast<__half2*>(&pb), bias);
                    const __half2 h2 = __hmul2(qh, d2);  // RN(q*d)
                    hi[2 * j + e] = *reinterpret_cast<const uint32_t*>(&h2);
                    if (SPLIT) {
                        const __half2 l2 = __hfma2(qh, d2s, __hmul2(h2, m2048));  // RN(2^11 (q*d - hi)), exact
                        lo[2 * j + e] = *reinterpret_cast<const uint32_t*>(&l2);
                    }
                }
            }
            return;
        }
    }
    // fp32 route: bf16 operands, or a split block with |d| >= 0.25
    const float d = __half2float(dh);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float f[4];
        f[0] = __int_as_float(__byte_perm(w[j], 0x4B000000u, 0x7650)) - 8388736.0f;
        f[1] = __int_as_float(__byte_perm(w[j], 0x4B000000u, 0x7651)) - 8388736.0f;
        f[2] = __int_as_float(__byte_perm(w[j], 0x4B000000u, 0x7652)) - 8388736.0f;
        f[3] = __int_as_float(__byte_perm(w[j], 0x4B000000u, 0x7653)) - 8388736.0f;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float w0 = __fmul_rn(f[2 * e], d), w1 = __fmul_rn(f[2 * e + 1], d);  // exact
            if constexpr (BF16) {
                __nv_bfloat162 h = __floats2bfloat162_rn(w0, w1);
                hi[2 * j + e] = *reinterpret_cast<uint32_t*>(&h);
            } else {
                __half2 h = __floats2half2_rn(w0, w1);
                hi[2 * j + e] = *reinterpret_cast<uint32_t*>(&h);
                if (SPLIT) {
                    const float2 hf = __half22float2(h);
                    __half2 lh = __floats2half2_rn(__fmul_rn(__fsub_rn(w0, hf.x), 2048.0f),
                                                   __fmul_rn(__fsub_rn(w1, hf.y), 2048.0f));
                    lo[2 * j + e] = *reinterpret_cast<uint32_t*>(&lh);
                }
            }
        }
    }
}

// 16 Q4_K weights from the nibbles of 16 quant bytes (low nibbles, or high when
// `high`): w = sl * q - ml with sl = d sc and ml = dmin m of their sub-block,
// each operation rounded once as in the reference's dequantisation; then the
// operand type (fp16 hi, and lo = RN(2^11 (w - hi)) when split).
template <bool SPLIT>
__device__ __forceinline__ void dequant16_q4k(const uint4 q, bool high, float sl, float ml, uint32_t (&hi)[8],
                                              uint32_t (&lo)[8]) {
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t v = high ? (w4[j] >> 4) : w4[j];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float q0 = (float)((v >> (16 * e)) & 0xFu), q1 = (float)((v >> (16 * e + 8)) & 0xFu);
            const float w0 = __fsub_rn(__fmul_rn(sl, q0), ml), w1 = __fsub_rn(__fmul_rn(sl, q1), ml);
            const __half2 h = __floats2half2_rn(w0, w1);
            hi[2 * j + e] = *reinterpret_cast<const uint32_t*>(&h);
            if (SPLIT) {
                const float2 hf = __half22float2(h);
                const __half2 l = __floats2half2_rn(__fmul_rn(__fsub_rn(w0, hf.x), 2048.0f),
                                                    __fmul_rn(__fsub_rn(w1, hf.y), 2048.0f));
                lo[2 * j + e] = *reinterpret_cast<const uint32_t*>(&l);
            }
        }
    }
}

// Sub-block j's 6-bit scale and min from a superblock's 12 scale bytes
// (q4k_dequant.h:43-60).
__device__ __forceinline__ void q4k_scale_min_tc(int j, const uint8_t* sc, int& s, int& m) {
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

// Writes the 16-element chunk c (K elements 16c..16c+15) of row rr into a
// K-major 128B-swizzled tile: 16-byte unit u of row rr sits at unit u ^ (rr & 7).
__device__ __forceinline__ void store_chunk(uint8_t* tile, int rr, int c, const uint32_t (&w)[8]) {
    uint8_t* row = tile + (rr >> 3) * 1024 + (rr & 7) * 128;
    *reinterpret_cast<uint4*>(row + (((2 * c) ^ (rr & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(row + (((2 * c + 1) ^ (rr & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
}

// Tensor maps of activation K blocks held in separate buffers (see TcOptions).
constexpr int kMaxABlocks = 8;
struct alignas(64) ABlockMaps {
    CUtensorMap m[kMaxABlocks];
    int n;  // 0: the activations are tm_a
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kDeqThreads) : "memory"); }

// Prefill preprocessing of this CTA's q / k / v head groups (PrepEpilogue), on
// the 8 epilogue warps once the plain epilogue is done.  Per 128-column head
// group: the fp32 tile [MT * BM][128] goes from TMEM to shared memory (raw rows
// 0..2 and the last 3 also to `edge`, rows T-4..T-1 to `win`); then warp w takes
// rows [w R/8, (w+1) R/8) and lane l columns 4l..4l+3: conv1d over the 3 rows
// above (a sliding window in registers) + SiLU, in the prep kernel's arithmetic;
// for q and k the row's L2 norm (eight rows' sums of squares share one exchange
// over the lanes), then bf16 out.
// Both named barriers run on every epilogue warp, `ok` or not.
template <int BN, int MT>
__device__ __forceinline__ void prep_epilogue(const PrepEpilogue& pe, float* S, uint32_t tmem, int n0, int64_t m0,
                                              int tile, int warp, int lane, bool ok) {
    constexpr int R = MT * BM;  // tokens per M tile
    constexpr int SP = 132;     // staged row pitch (floats): 16-byte row phases on distinct bank groups
    constexpr int RC = R / 8;   // rows per warp in the conv pass
    static_assert(RC == 16 || RC == 32, "rows per warp");
    const int q = warp & 3, half = (warp - kDeqWarp0) >> 2, wi = warp - kDeqWarp0;
    for (int hg = 0; hg < BN / 128; hg++) {
        const int hc0 = n0 + hg * 128;  // channel of the head group's column 0
        if (hc0 >= pe.qkv) break;       // z columns: the plain epilogue
        epi_bar();                      // the staging area is free
        if (ok) {
            const int mt = MT == 2 ? half : 0;
            const int c_lo = MT == 2 ? 0 : half * 64, c_hi = MT == 2 ? 128 : c_lo + 64;
            const int row = mt * BM + q * 32 + lane;
            const int64_t tok = m0 + row;
            const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(mt * BN + hg * 128);
            float* edge_row = nullptr;
            if (tok < pe.T && row < 3) edge_row = pe.edge + ((int64_t)tile * 6 + row) * pe.qkv + hc0;
            if (tok < pe.T && row >= R - 3) edge_row = pe.edge + ((int64_t)tile * 6 + 3 + row - (R - 3)) * pe.qkv + hc0;
            float* win_row = (tok < pe.T && tok >= pe.T - 4) ? pe.win + (tok - (pe.T - 4)) * pe.qkv + hc0 : nullptr;
            for (int c = c_lo; c < c_hi; c += 32) {
                uint32_t v[32];
                tmem_load_32x32b_x32(tb + (uint32_t)c, v);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const uint4 u = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    *reinterpret_cast<uint4*>(S + row * SP + c + j) = u;
                    if (edge_row != nullptr) *reinterpret_cast<uint4*>(edge_row + c + j) = u;
                    if (win_row != nullptr) *reinterpret_cast<uint4*>(win_row + c + j) = u;
                }
            }
        }
        epi_bar();
        if (ok) {
            const int c4 = 4 * lane, ch = hc0 + c4, hidx = hc0 / 128;
            __nv_bfloat16* dst;
            if (hidx < pe.hk) dst = pe.qn + (int64_t)hidx * pe.Tp * 128;
            else if (hidx < 2 * pe.hk) dst = pe.kn + (int64_t)(hidx - pe.hk) * pe.Tp * 128;
            else dst = pe.vb + (int64_t)(hidx - 2 * pe.hk) * pe.Tp * 128;
            dst += c4;
            const bool l2 = hidx < 2 * pe.hk, conv = pe.conv_w != nullptr;
            float4 wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                wv[i] = conv ? __ldg(reinterpret_cast<const float4*>(pe.conv_w) + ch + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            const int r0 = wi * RC;
            const float* col = S + c4;
            // One pass over the warp's rows, eight at a time, with a branch-free body:
            // rows 0..2 of the tile, whose window lies in the previous tile, are
            // computed from clamped rows and not stored (the edge kernel's).  SiLU's
            // 1/2 is folded into the taps (exact: a power of two), and for q and k
            // the eight rows' sums of squares over the 32 lanes share one exchange
            // that halves the values each lane holds at every step.
            float4 w2[4];
#pragma unroll
            for (int c = 0; c < 4; c++)
                w2[c] = make_float4(0.5f * wv[c].x, 0.5f * wv[c].y, 0.5f * wv[c].z, 0.5f * wv[c].w);
            auto rows = [&](auto l2_tag, auto conv_tag) {
                constexpr bool L2 = decltype(l2_tag)::value, CONV = decltype(conv_tag)::value;
                float4 h0 = *reinterpret_cast<const float4*>(col + max(r0 - 3, 0) * SP);
                float4 h1 = *reinterpret_cast<const float4*>(col + max(r0 - 2, 0) * SP);
                float4 h2 = *reinterpret_cast<const float4*>(col + max(r0 - 1, 0) * SP);
#pragma unroll 1
                for (int g = 0; g < RC; g += 8) {
                    float o[8][4], ss[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float4 x = *reinterpret_cast<const float4*>(col + (r0 + g + i) * SP);
                        o[i][0] = x.x;
                        o[i][1] = x.y;
                        o[i][2] = x.z;
                        o[i][3] = x.w;
                        if constexpr (CONV) {
                            const float a0[4] = {h0.x, h0.y, h0.z, h0.w}, a1[4] = {h1.x, h1.y, h1.z, h1.w};
                            const float a2[4] = {h2.x, h2.y, h2.z, h2.w};
#pragma unroll
                            for (int c = 0; c < 4; c++) {
                                float hh = w2[c].x * a0[c];  // (w . window) / 2
                                hh = fmaf(w2[c].y, a1[c], hh);
                                hh = fmaf(w2[c].z, a2[c], hh);
                                hh = fmaf(w2[c].w, o[i][c], hh);
                                o[i][c] = fmaf(hh, tanh_hw(hh), hh);  // SiLU
                            }
                        }
                        h0 = h1;
                        h1 = h2;
                        h2 = x;
                        ss[i] = fmaf(o[i][0], o[i][0], fmaf(o[i][1], o[i][1], fmaf(o[i][2], o[i][2], o[i][3] * o[i][3])));
                    }
                    if constexpr (L2) {
                        // after the xor-16, -8, -4 halvings and two butterflies lane l holds
                        // row (l >> 2) & 7's sum in ss[0]
#pragma unroll
                        for (int st = 16, nv = 8; st >= 4; st >>= 1, nv >>= 1) {
                            const bool up = (lane & st) != 0;
#pragma unroll
                            for (int i = 0; i < nv / 2; i++) {
                                const float send = up ? ss[i] : ss[i + nv / 2];
                                const float keep = up ? ss[i + nv / 2] : ss[i];
                                ss[i] = keep + __shfl_xor_sync(0xffffffffu, send, st);
                            }
                        }
                        ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], 2);
                        ss[0] += __shfl_xor_sync(0xffffffffu, ss[0], 1);
                        const float inv_mine = inv_l2(ss[0]);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const float inv = __shfl_sync(0xffffffffu, inv_mine, 4 * i);
#pragma unroll
                            for (int c = 0; c < 4; c++) o[i][c] *= inv;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int64_t t = m0 + r0 + g + i;
                        __nv_bfloat162 a = __floats2bfloat162_rn(o[i][0], o[i][1]);
                        __nv_bfloat162 b = __floats2bfloat162_rn(o[i][2], o[i][3]);
                        uint2 val = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
                        if (t >= pe.T) val = make_uint2(0u, 0u);
                        if (r0 + g + i >= 3 && t < pe.Tp) *reinterpret_cast<uint2*>(dst + t * 128) = val;
                    }
                }
            };
            using T1 = std::true_type;
            using F0 = std::false_type;
            if (l2) {
                if (conv) rows(T1(), T1());
                else rows(T1(), F0());
            } else {
                if (conv) rows(F0(), T1());
                else rows(F0(), F0());
            }
        }
    }
}

template <int BN, int MT, int SA, int S16, int S8, bool BF16, bool SPLIT, bool Q4K = false>
__global__ void __launch_bounds__(kThreads, 1)
    q8_0_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ ABlockMaps am, const uint16_t* __restrict__ dsc, int n, int k, int m,
                        float* __restrict__ y, int64_t ldy, int kt_per_split, int a_blk_k, int a_row0,
                        const PrepEpilogue pe, uint32_t* __restrict__ err) {
    using L = TcLayout<BN, MT, SA, S16, S8, SPLIT, Q4K>;
    static_assert(!Q4K || !BF16, "Q4_K operands are fp16");
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + L::BAR_OFF;
    auto a_full = [&](int s) { return bar0 + 8u * s; };
    auto a_empty = [&](int s) { return bar0 + 8u * (SA + s); };
    auto b16_full = [&](int s) { return bar0 + 8u * (2 * SA + s); };
    auto b16_empty = [&](int s) { return bar0 + 8u * (2 * SA + S16 + s); };
    auto b8_full = [&](int s) { return bar0 + 8u * (2 * SA + 2 * S16 + s); };
    auto b8_empty = [&](int s) { return bar0 + 8u * (2 * SA + 2 * S16 + S8 + s); };
    const uint32_t accf_bar = bar0 + 8u * (2 * SA + 2 * S16 + 2 * S8);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * (BM * MT);
    const int KT_total = k / BK;
    const int kt0 = blockIdx.z * kt_per_split;
    const int KT = min(kt_per_split, KT_total - kt0);  // k-tiles of this CTA (>= 1 by construction)

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < SA; s++) {
            mbar_init(a_full(s), 1);
            mbar_init(a_empty(s), 1);
        }
        for (int s = 0; s < S16; s++) {
            mbar_init(b16_full(s), kDeqWarps);
            mbar_init(b16_empty(s), 1);
        }
        for (int s = 0; s < S8; s++) {
            mbar_init(b8_full(s), 1);
            mbar_init(b8_empty(s), kDeqWarps);
        }
        mbar_init(accf_bar, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), L::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 || warp == 2) {
        // ---- producers: warp 0 streams activation tiles, warp 2 int8 weight tiles
        if (lane == 0) {
            const bool is_a = (warp == 0);
            // The weights never come from an earlier kernel, so their stream starts at
            // once; the activations wait for the predecessor (programmatic launch).
            if (is_a) pdl_wait();
            const int depth = is_a ? SA : S8;
            const int nload = (is_a || !Q4K) ? KT : KT / kQ4kTiles;  // k-tiles, or superblocks
            int issued = 0;
            bool ok = true;
            for (int t = 0; t < nload; t++) {
                const int s = t % depth, r = t / depth;
                if (t >= depth) ok = mbar_wait(is_a ? a_empty(s) : b8_empty(s), (r - 1) & 1, err);
                if (!ok) break;
                if (is_a) {
                    mbar_arrive_expect_tx(a_full(s), MT * L::A_BYTES);
                    const int kk = (kt0 + t) * BK;
#pragma unroll
                    for (int mt = 0; mt < MT; mt++) {
                        const uint32_t dst = sbase + L::A_OFF + (s * MT + mt) * L::A_BYTES;
                        if (am.n > 0)  // K block kk / a_blk_k in its own buffer (possibly a peer's)
                            tma_load_2d(dst, &am.m[kk / a_blk_k], kk % a_blk_k, a_row0 + m0 + mt * BM, a_full(s));
                        else if (a_blk_k > 0)  // activations stored as K blocks [k / a_blk_k][rows][a_blk_k]
                            tma_load_3d(dst, &tm_a, kk % a_blk_k, a_row0 + m0 + mt * BM, kk / a_blk_k, a_full(s));
                        else
                            tma_load_2d(dst, &tm_a, kk, m0 + mt * BM, a_full(s));
                    }
                } else if (Q4K) {  // superblock kt0 / 4 + t of rows n0.., bytes at x = 144 sb
                    mbar_arrive_expect_tx(b8_full(s), L::B8_BYTES);
                    tma_load_2d(sbase + L::B8_OFF + s * L::B8_BYTES, &tm_b, (kt0 / kQ4kTiles + t) * kQ4kBytes, n0,
                                b8_full(s));
                } else {
                    mbar_arrive_expect_tx(b8_full(s), L::B8_BYTES);
                    tma_load_2d(sbase + L::B8_OFF + s * L::B8_BYTES, &tm_b, (kt0 + t) * BK, n0, b8_full(s));
                }
                issued++;
            }
            if (!ok) {
                // Give the loads already issued a bounded chance to land before exit.
                for (int t = (issued > depth ? issued - depth : 0); t < issued; t++)
                    mbar_wait(is_a ? a_full(t % depth) : b8_full(t % depth), (t / depth) & 1, err);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(BM, BN, BF16);
            for (int t = 0; t < KT; t++) {
                const int sa = t % SA, s16 = t % S16;
                if (!(mbar_wait(a_full(sa), (t / SA) & 1, err) && mbar_wait(b16_full(s16), (t / S16) & 1, err)))
                    break;
                tc_fence_after();
                const uint32_t b0 = sbase + L::B16_OFF + s16 * L::NB * L::B16_BYTES;
#pragma unroll
                for (int mt = 0; mt < MT; mt++) {
                    const uint32_t a0 = sbase + L::A_OFF + (sa * MT + mt) * L::A_BYTES;
                    const uint32_t acc_col = tmem + (uint32_t)(mt * L::ACC_STRIDE);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++) {
                        const uint64_t ad = umma_desc_sw128(a0 + kk * 32);
                        const uint32_t acc = (t | kk) != 0 ? 1u : 0u;
                        mma_f16_ss(acc_col, ad, umma_desc_sw128(b0 + kk * 32), idesc, acc);
                        if (SPLIT)
                            mma_f16_ss(acc_col + BN, ad, umma_desc_sw128(b0 + L::B16_BYTES + kk * 32), idesc, acc);
                    }
                }
                mma_commit(a_empty(sa));
                mma_commit(b16_empty(s16));
            }
            mma_commit(accf_bar);
        }
    } else {
        // ---- dequant: BN rows x 4 chunks of 16 per k-tile over 256 threads
        constexpr int CPT = (BN * 4 + kDeqThreads - 1) / kDeqThreads;  // chunks of one row per thread: 1, 2 or 4
        const int i = threadIdx.x - 32 * kDeqWarp0;
        const int kb = k >> 5;
        // BN = 96 (384 units): warps 0-3 take rows 0..63 two chunks a thread, warps 4-7
        // rows 64..95 one chunk a thread (each scheduler holds one warp of either kind)
        int rr, c0, ncpt = CPT;
        if constexpr (BN * 4 % kDeqThreads == 0) {
            rr = i / (4 / CPT);
            c0 = (i % (4 / CPT)) * CPT;
        } else {
            static_assert(BN == 96 && CPT == 2, "uneven dequant split for 96-column tiles only");
            rr = i < 128 ? (i >> 1) : 64 + ((i - 128) >> 2);
            c0 = i < 128 ? (i & 1) * 2 : (i - 128) & 3;
            ncpt = i < 128 ? 2 : 1;
        }
        const int gr = n0 + rr;
        const uint16_t* drow = (!Q4K && gr < n) ? dsc + (int64_t)gr * kb + 2 * kt0 : nullptr;
        // Scales are prefetched kWin k-tiles ahead in registers when every row's
        // window is 16-byte aligned; otherwise they are read per k-tile.
        const bool windowed = (kb % 8 == 0) && (kt0 % 4 == 0);
        uint4 cur[2], nxt[2];
        auto load_win = [&](uint4 (&dst)[2], int w) {
            const int t = w * kWin;
            if (drow != nullptr && t < KT) {
                const uint4* p = reinterpret_cast<const uint4*>(drow + 2 * t);
                dst[0] = __ldg(p);
                dst[1] = (t + 4 < KT) ? __ldg(p + 1) : make_uint4(0, 0, 0, 0);
            } else {
                dst[0] = dst[1] = make_uint4(0, 0, 0, 0);
            }
        };
        if (windowed) {
            load_win(cur, 0);
            load_win(nxt, 1);
        }
        bool ok = true;
        if constexpr (Q4K) {
            // one superblock row (header + 128 quant bytes) per 4 k-tiles, kept in registers
            for (int sbl = 0; sbl < KT / kQ4kTiles && ok; sbl++) {
                const int s8 = sbl % S8;
                ok = __all_sync(0xffffffffu, mbar_wait(b8_full(s8), (sbl / S8) & 1, err));
                if (!ok) break;
                // rows are 144 bytes apart: the 8 lanes of a shared-memory phase read 8 bank groups
                const uint4* src = reinterpret_cast<const uint4*>(smem + L::B8_OFF + s8 * L::B8_BYTES + rr * kQ4kBytes);
                const uint4 hdr = src[0];
                uint4 qb[8];
#pragma unroll
                for (int j = 0; j < 8; j++) qb[j] = src[1 + j];
                fence_proxy_async_smem();  // the slot's next write is a TMA (async proxy)
                __syncwarp();
                if (lane == 0) mbar_arrive(b8_empty(s8));
                const float d = __half2float(__ushort_as_half((unsigned short)(hdr.x & 0xFFFFu)));
                const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr.x >> 16)));
                uint8_t scb[12];
                *reinterpret_cast<uint32_t*>(scb) = hdr.y;
                *reinterpret_cast<uint32_t*>(scb + 4) = hdr.z;
                *reinterpret_cast<uint32_t*>(scb + 8) = hdr.w;
#pragma unroll
                for (int cq = 0; cq < kQ4kTiles; cq++) {  // sub-blocks 2 cq (weights 0..31) and 2 cq + 1 (32..63)
                    const int t = sbl * kQ4kTiles + cq, s16 = t % S16;
                    int sa, ma, sb, mb;
                    q4k_scale_min_tc(2 * cq, scb, sa, ma);
                    q4k_scale_min_tc(2 * cq + 1, scb, sb, mb);
                    const float slo = __fmul_rn(d, (float)sa), mlo = __fmul_rn(dmin, (float)ma);
                    const float shi = __fmul_rn(d, (float)sb), mhi = __fmul_rn(dmin, (float)mb);
                    if (t >= S16) ok = __all_sync(0xffffffffu, mbar_wait(b16_empty(s16), ((t / S16) - 1) & 1, err));
                    if (!ok) break;
                    uint8_t* bhi = smem + L::B16_OFF + s16 * L::NB * L::B16_BYTES;
#pragma unroll
                    for (int cc = 0; cc < CPT; cc++) {
                        // chunk c: weights 16c..16c+15 = nibbles of quant bytes 32 cq + 16 (c & 1) ..,
                        // low for c < 2 (sub-block 2 cq), high for c >= 2 (2 cq + 1); rows past n
                        // arrive as zeros from the TMA (d = dmin = 0), so their weights are 0
                        const int c = c0 + cc;
                        uint32_t hi[8], lo[8];
                        const bool high = c >= 2;
                        dequant16_q4k<SPLIT>((c & 1) ? qb[2 * cq + 1] : qb[2 * cq], high, high ? shi : slo,
                                             high ? mhi : mlo, hi, lo);
                        store_chunk(bhi, rr, c, hi);
                        if (SPLIT) store_chunk(bhi + L::B16_BYTES, rr, c, lo);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(b16_full(s16));
                }
            }
        }
        for (int w = 0; !Q4K && w * kWin < KT && ok; w++) {
            if (windowed && w > 0) {
                cur[0] = nxt[0];
                cur[1] = nxt[1];
                load_win(nxt, w + 1);
            }
#pragma unroll
            for (int u = 0; u < kWin; u++) {
                const int t = w * kWin + u;
                if (t >= KT) break;
                const int s8 = t % S8, s16 = t % S16;
                ok = __all_sync(0xffffffffu, mbar_wait(b8_full(s8), (t / S8) & 1, err));
                if (!ok) break;
                // raw int8 chunks of this thread -> registers; the slot is released at once.
                // The tile arrives 64B-swizzled: 16-byte chunk u of row rr sits at
                // u ^ ((rr >> 1) & 3), so the 8 lanes of each shared-memory phase
                // (rows rr..rr+7, or 4 rows x 2 chunks) hit 8 different bank groups.
                const uint4* src = reinterpret_cast<const uint4*>(smem + L::B8_OFF + s8 * L::B8_BYTES + rr * BK);
                uint4 raw[CPT];
#pragma unroll
                for (int cc = 0; cc < CPT; cc++)
                    if (cc < ncpt) raw[cc] = src[(c0 + cc) ^ ((rr >> 1) & 3)];
                // The next write to this slot is a TMA (async proxy): the generic
                // reads above must be ordered before it by a proxy fence, or the
                // refill can overtake a late read (one weight row goes stale).
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(b8_empty(s8));
                uint32_t sc2;
                if (windowed) {
                    const uint4 v = cur[u >> 2];
                    sc2 = (u & 3) == 0 ? v.x : (u & 3) == 1 ? v.y : (u & 3) == 2 ? v.z : v.w;
                } else {
                    sc2 = drow != nullptr ? __ldg(reinterpret_cast<const uint32_t*>(drow + 2 * t)) : 0u;
                }
                if (t >= S16) ok = __all_sync(0xffffffffu, mbar_wait(b16_empty(s16), ((t / S16) - 1) & 1, err));
                if (!ok) break;
                uint8_t* bhi = smem + L::B16_OFF + s16 * L::NB * L::B16_BYTES;
#pragma unroll
                for (int cc = 0; cc < CPT; cc++) {
                    if (cc >= ncpt) break;
                    const int c = c0 + cc;
                    uint32_t hi[8], lo[8];
                    dequant16<BF16, SPLIT>(raw[cc], (uint16_t)(c < 2 ? (sc2 & 0xFFFFu) : (sc2 >> 16)), hi, lo);
                    store_chunk(bhi, rr, c, hi);
                    if (SPLIT) store_chunk(bhi + L::B16_BYTES, rr, c, lo);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(b16_full(s16));
            }
        }
        // ---- epilogue: warp quadrant q reads TMEM lanes [32q, 32q+32); the two
        // warps of a quadrant take alternate 32-column groups.  Each 32 x 32 block
        // goes through a per-warp staging tile in the (drained) activation ring so
        // that global stores write whole 128-byte row segments, 4 rows per store.
        if (ok) ok = mbar_wait(accf_bar, 0, err);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
        tc_fence_after();
        const int q = warp & 3;
        const int half = (warp - kDeqWarp0) >> 2;
        float* ybase = y + (int64_t)blockIdx.z * (int64_t)m * ldy;  // split-K partial slice
        const bool vec_ok = ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
        constexpr int kPitch = 36;  // floats per staged row: 16-byte aligned, conflict-free
        float* stg = reinterpret_cast<float*>(smem + L::A_OFF) + (warp - kDeqWarp0) * (32 * kPitch);
        const int sr = lane >> 3, sc = (lane & 7) * 4;  // store phase: row within a group of 4, column
        if (ok) {
#pragma unroll 1
            for (int mt = 0; mt < MT; mt++) {
                const int row0 = m0 + mt * BM + q * 32;
                const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(mt * L::ACC_STRIDE);
#pragma unroll 1
                for (int cg = half * 32; cg < BN; cg += 64) {
                    if (!SPLIT && pe.enabled && n0 + cg < pe.qkv) continue;  // fused preprocessing below
                    uint32_t v[32];
                    tmem_load_32x32b_x32(tbase + (uint32_t)cg, v);
                    if (SPLIT) {
                        uint32_t vl[32];
                        tmem_load_32x32b_x32(tbase + (uint32_t)(BN + cg), vl);
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            v[j] = __float_as_uint(fmaf(__uint_as_float(vl[j]), 1.0f / 2048.0f, __uint_as_float(v[j])));
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<uint4*>(stg + lane * kPitch + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    __syncwarp();
                    const int col = n0 + cg + sc;
#pragma unroll
                    for (int it = 0; it < 8; it++) {
                        const int r = it * 4 + sr;
                        if (row0 + r < m) {
                            const float4 f = *reinterpret_cast<const float4*>(stg + r * kPitch + sc);
                            float* yr = ybase + (int64_t)(row0 + r) * ldy + col;
                            if (vec_ok && col + 4 <= n) {
                                *reinterpret_cast<float4*>(yr) = f;
                            } else {
                                if (col < n) yr[0] = f.x;
                                if (col + 1 < n) yr[1] = f.y;
                                if (col + 2 < n) yr[2] = f.z;
                                if (col + 3 < n) yr[3] = f.w;
                            }
                        }
                    }
                    __syncwarp();
                }
            }
        }
        if constexpr (!SPLIT && BN % 128 == 0) {
            static_assert(SPLIT || (uint32_t)MT * BM * 132 * 4 <= L::B8_OFF, "preprocessing stage fits the rings");
            if (pe.enabled)
                prep_epilogue<BN, MT>(pe, reinterpret_cast<float*>(smem), tmem, n0, m0, (int)blockIdx.y, warp, lane, ok);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

// y[r][c] = sum_z part[z][r][c], z in order (deterministic split-K reduction).
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t m, int64_t n,
                                     float* __restrict__ y, int64_t ldy) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m * n) return;
    const int64_t r = i / n, c = i - r * n;
    float s = 0.0f;
    for (int z = 0; z < splits; z++) s += part[(int64_t)z * m * n + i];
    y[r * ldy + c] = s;
}

template <typename OutT>
__global__ void convert_kernel(const void* __restrict__ x, int dtype, OutT* __restrict__ out, int64_t count) {
    pdl_trigger();
    pdl_wait();
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float v = load_act(x, dtype, i);
    if constexpr (std::is_same<OutT, __half>::value) out[i] = __float2half_rn(v);
    else out[i] = __float2bfloat16_rn(v);
}

// 8 elements per thread: 16-byte loads (two for fp32 input) and one 16-byte store.
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
        f[2 * j] = v.x;
        f[2 * j + 1] = v.y;
    }
}
__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        f[2 * j] = v.x;
        f[2 * j + 1] = v.y;
    }
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <typename InT, typename OutT>
__global__ void convert8_kernel(const InT* __restrict__ x, OutT* __restrict__ out, int64_t n8) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        float f[8];
        load8(x + 8 * i, f);
        OutT* tag = nullptr;
        *reinterpret_cast<uint4*>(out + 8 * i) =
            make_uint4(pack2(f[0], f[1], tag), pack2(f[2], f[3], tag), pack2(f[4], f[5], tag), pack2(f[6], f[7], tag));
    }
}

template <typename OutT>
int launch_convert8(const void* x, int dtype, OutT* out, int64_t n8, cudaStream_t s) {
    const unsigned g = (unsigned)std::min<int64_t>((n8 + 255) / 256, (int64_t)sm_count() * 8);
    if (dtype == GDN_DTYPE_F32)
        return launch_pdl("convert8_kernel", convert8_kernel<float, OutT>, dim3(g), dim3(256), 0, s,
                          static_cast<const float*>(x), out, n8);
    if (dtype == GDN_DTYPE_BF16)
        return launch_pdl("convert8_kernel", convert8_kernel<__nv_bfloat16, OutT>, dim3(g), dim3(256), 0, s,
                          static_cast<const __nv_bfloat16*>(x), out, n8);
    return launch_pdl("convert8_kernel", convert8_kernel<__half, OutT>, dim3(g), dim3(256), 0, s,
                      static_cast<const __half*>(x), out, n8);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode(EncodeTiledFn* out) {
    static EncodeTiledFn fn = nullptr;
    if (fn == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
            return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    *out = fn;
    return GDN_OK;
}

}  // namespace

int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
    EncodeTiledFn enc;
    int st = get_encode(&enc);
    if (st) return st;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GDN_OK;
}

// 3-D map of activations stored as K blocks: [nblk][rows][blk_k], 128B-swizzled
// boxes of BK x BM x 1.
int make_map_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t blk_k, uint64_t rows,
                uint64_t nblk, uint64_t row_bytes, uint64_t blk_bytes, uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn enc;
    int st = get_encode(&enc);
    if (st) return st;
    const cuuint64_t dims[3] = {blk_k, rows, nblk};
    const cuuint64_t strides[2] = {row_bytes, blk_bytes};
    const cuuint32_t box[3] = {box_inner, box_outer, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GDN_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return GDN_OK;
}

namespace {

struct ALayout {
    int64_t blk_k = 0, rows = 0, row0 = 0;  // see TcOptions
    const void* const* block_ptrs = nullptr;
    int nblocks = 0;
};

template <int BN, int MT, int SA, int S16, int S8, bool BF16, bool SPLIT, bool Q4K = false>
int run_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* a, int64_t m, float* out,
           int64_t ld_out, int splits, int kt_per, const ALayout& al, cudaStream_t s,
           const PrepEpilogue& pe = PrepEpilogue()) {
    using L = TcLayout<BN, MT, SA, S16, S8, SPLIT, Q4K>;
    CUtensorMap ma, mb;
    const CUtensorMapDataType adt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    ABlockMaps am;
    memset(&am, 0, sizeof(am));
    int st = GDN_OK;
    if (al.nblocks > 0) {
        for (int g = 0; g < al.nblocks && !st; g++)
            st = make_map_2d(&am.m[g], adt, al.block_ptrs[g], (uint64_t)al.blk_k, (uint64_t)al.rows,
                             (uint64_t)al.blk_k * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
        am.n = al.nblocks;
        ma = am.m[0];  // a valid map for the prologue's prefetch
    } else {
        st = al.blk_k > 0 ? make_map_3d(&ma, adt, a, (uint64_t)al.blk_k, (uint64_t)al.rows, (uint64_t)(k / al.blk_k),
                                        (uint64_t)al.blk_k * 2, (uint64_t)al.rows * al.blk_k * 2, BK, BM)
                          : make_map_2d(&ma, adt, a, (uint64_t)k, (uint64_t)m, (uint64_t)k * 2, BK, BM,
                                        CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (st) return st;
    if (Q4K)  // raw superblock rows: n x (k / 256) x 144 bytes, one superblock per box
        st = make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, qs, (uint64_t)(k / 256 * kQ4kBytes), (uint64_t)n,
                         (uint64_t)(k / 256 * kQ4kBytes), kQ4kBytes, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    else
        st = make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, qs, (uint64_t)k, (uint64_t)n, (uint64_t)k, BK, BN,
                         CU_TENSOR_MAP_SWIZZLE_64B);
    if (st) return st;
    auto kern = q8_0_gemm_tc_kernel<BN, MT, SA, S16, S8, BF16, SPLIT, Q4K>;
    GDN_CUDA(cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM));
    const dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM * MT - 1) / (BM * MT)), (unsigned)splits);
    return launch_pdl("q8_0_gemm_tc_kernel", kern, grid, dim3(kThreads), L::SMEM, s, ma, mb, am, d, (int)n, (int)k,
                      (int)m, out, ld_out, kt_per, (int)al.blk_k, (int)al.row0, pe, device_error_word());
}

}  // namespace

int launch_convert(const void* x, int x_dtype, void* out, bool to_bf16, int64_t count, cudaStream_t s) {
    if (count == 0) return GDN_OK;
    if (count % 8 == 0 && aligned(x, 16) && aligned(out, 16)) {
        if (to_bf16) return launch_convert8(x, x_dtype, static_cast<__nv_bfloat16*>(out), count / 8, s);
        return launch_convert8(x, x_dtype, static_cast<__half*>(out), count / 8, s);
    }
    const unsigned g = (unsigned)((count + 255) / 256);
    if (to_bf16)
        return launch_pdl("convert_kernel", convert_kernel<__nv_bfloat16>, dim3(g), dim3(256), 0, s, x, x_dtype,
                          static_cast<__nv_bfloat16*>(out), count);
    return launch_pdl("convert_kernel", convert_kernel<__half>, dim3(g), dim3(256), 0, s, x, x_dtype,
                      static_cast<__half*>(out), count);
}

size_t gemm_tc_workspace_bytes(int64_t m, int64_t n, int splits) {
    return splits > 1 ? (size_t)splits * m * n * sizeof(float) : 0;
}

int launch_q8_0_gemm_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* a, bool a_bf16,
                        int64_t m, float* y, int64_t ldy, const TcOptions& opt, cudaStream_t s) {
    if (k % BK != 0 || k <= 0) return fail(GDN_ERR_SHAPE, "tensor-core GEMM needs k %% 64 == 0 (k=%lld)", (long long)k);
    if (n <= 0 || m <= 0) return GDN_OK;
    if (n > INT32_MAX || m > INT32_MAX || k > INT32_MAX) return fail(GDN_ERR_SHAPE, "GEMM dims exceed int32");
    if (ldy < n) return fail(GDN_ERR_SHAPE, "ldy < n");
    if (!aligned(a, 16) || !aligned(qs, 16) || !aligned(d, 4))
        return fail(GDN_ERR_ARG, "tensor-core GEMM operands must be 16-byte aligned (scales 4-byte)");
    const int KT = (int)(k / BK);
    int splits = opt.splits < 1 ? 1 : opt.splits;
    int kt_per = (KT + splits - 1) / splits;
    if (splits > 1) kt_per = (kt_per + kWin - 1) / kWin * kWin;  // keep scale windows aligned
    splits = (KT + kt_per - 1) / kt_per;
    float* out = y;
    int64_t ld_out = ldy;
    if (splits > 1) {
        if (opt.workspace == nullptr || opt.workspace_bytes < gemm_tc_workspace_bytes(m, n, splits))
            return fail(GDN_ERR_ARG, "split-K workspace too small");
        out = static_cast<float*>(opt.workspace);
        ld_out = n;
    }
    if (opt.partials_only && (y != opt.workspace || ldy != n))
        return fail(GDN_ERR_ARG, "partials_only: y must be the workspace with ldy = n");
    // Two M tiles per CTA share each dequantised weight tile once m > 128.
    // Ring depths <SA, S16, S8> fill ~224 KB of shared memory.
    if (opt.split_precision && a_bf16)
        return fail(GDN_ERR_TYPE, "split-precision tensor-core GEMM takes fp16 activations");
    if (opt.split_precision && opt.prep != nullptr && opt.prep->enabled)
        return fail(GDN_ERR_ARG, "fused preprocessing runs on the single-operand GEMM only");
    ALayout al;
    if (opt.a_nblocks > 0) {
        if (opt.a_nblocks > kMaxABlocks || opt.a_block_ptrs == nullptr || opt.a_blk_k * opt.a_nblocks != k)
            return fail(GDN_ERR_SHAPE, "K blocks: %d buffers of %lld must cover k=%lld (at most %d)", opt.a_nblocks,
                        (long long)opt.a_blk_k, (long long)k, kMaxABlocks);
        for (int g = 0; g < opt.a_nblocks; g++)
            if (opt.a_block_ptrs[g] == nullptr || !aligned(opt.a_block_ptrs[g], 16))
                return fail(GDN_ERR_ARG, "K block %d: NULL or not 16-byte aligned", g);
        al.block_ptrs = opt.a_block_ptrs;
        al.nblocks = opt.a_nblocks;
    }
    if (opt.a_blk_k > 0) {
        if (opt.a_blk_k % BK != 0 || k % opt.a_blk_k != 0)
            return fail(GDN_ERR_SHAPE, "K blocks must be a multiple of 64 that divides k");
        if (opt.a_row0 < 0 || opt.a_row0 + m > opt.a_rows || opt.a_rows > INT32_MAX)
            return fail(GDN_ERR_SHAPE, "rows [%lld, %lld) outside the %lld stored rows", (long long)opt.a_row0,
                        (long long)(opt.a_row0 + m), (long long)opt.a_rows);
        al.blk_k = opt.a_blk_k;
        al.rows = opt.a_rows;
        al.row0 = opt.a_row0;
    }
    const bool two = m > BM;
    int st;
    if (opt.split_precision) {
        // Two M tiles per CTA share each dequantised tile -- unless the weight has
        // a single column tile (the gate rows) and one-M-tile CTAs still fit one
        // wave: then twice the CTAs split the same work.
        const int64_t mt1 = (m + BM - 1) / BM * splits;
        const bool pair = two && !(n <= 128 && mt1 <= sm_count());
        st = pair ? run_tc<128, 2, 4, 2, 4, false, true>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s)
                  : run_tc<128, 1, 6, 3, 4, false, true>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s);
    } else {
        // One operand: 256-column tiles halve the activation traffic per MMA, as long
        // as the grid still covers at least half of the SMs.
        const int64_t tiles256 = (n + 255) / 256 * ((m + 2 * BM - 1) / (2 * BM)) * splits;
        const bool wide = two && tiles256 * 2 >= sm_count();
        PrepEpilogue pe;
        if (opt.prep != nullptr && opt.prep->enabled) {
            const PrepEpilogue& p = *opt.prep;
            if (splits != 1 || p.qkv <= 0 || p.qkv % 128 != 0 || p.qkv > n || p.hk < 0 || 2 * p.hk * 128 > p.qkv ||
                p.T != m || p.Tp < m || !p.qn || !p.kn || !p.vb || !p.edge || !p.win ||
                (p.conv_w && !aligned(p.conv_w, 16)))
                return fail(GDN_ERR_ARG, "fused preprocessing: inconsistent options");
            opt.prep->rows = two ? 2 * BM : BM;
            pe = *opt.prep;
        }
        // One M tile (m <= 128): a grid short of one wave leaves SMs idle while each CTA
        // streams BN weight rows, so take the narrowest tile whose grid still fits one
        // wave (fewest rows per SM; 12288 rows: 96 columns, 128 CTAs; the decode step at
        // 16-63 sequences 10-15% faster).  Paired M tiles keep theirs: every CTA reads all
        // 256 activation rows per k-tile whatever its width, and 128 CTAs of 96 columns
        // measured slower than 96 of 128 (decode step at 256 sequences 253 vs 246-250 us).
        // The fused preprocessing keeps its tiles.
        const int64_t mtiles = (m + BM - 1) / BM;
        auto ctas = [&](int64_t bn) { return (n + bn - 1) / bn * mtiles * splits; };
        int bn = !two || wide ? 256 : 128;
        if (!two && !pe.enabled && ctas(bn) < sm_count())
            for (const int c : {128, 96})
                if (c < bn && ctas(c) <= sm_count()) bn = c;
        if (a_bf16) {
            st = !two ? (bn == 256   ? run_tc<256, 1, 4, 3, 4, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe)
                         : bn == 128 ? run_tc<128, 1, 6, 4, 8, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe)
                                     : run_tc<96, 1, 6, 4, 12, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe))
                      : (bn == 256 ? run_tc<256, 2, 3, 3, 2, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe)
                                   : run_tc<128, 2, 4, 3, 6, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe));
        } else {
            st = !two ? (bn == 256   ? run_tc<256, 1, 4, 3, 4, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe)
                         : bn == 128 ? run_tc<128, 1, 6, 4, 8, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe)
                                     : run_tc<96, 1, 6, 4, 12, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe))
                      : (bn == 256 ? run_tc<256, 2, 3, 3, 2, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe)
                                   : run_tc<128, 2, 4, 3, 6, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, al, s, pe));
        }
    }
    if (opt.splits_used != nullptr) *opt.splits_used = splits;
    if (st || splits == 1 || opt.partials_only) return st;
    const int64_t cnt = m * n;
    st = launch_pdl("splitk_reduce_kernel", splitk_reduce_kernel, dim3((unsigned)((cnt + 255) / 256)), dim3(256), 0,
                    s, (const float*)out, splits, m, n, y, ldy);
    if (st) return st;
    return GDN_OK;
}

int launch_q4_k_gemm_tc(const void* blocks, int64_t n, int64_t k, const void* a, int64_t m, float* y, int64_t ldy,
                        const TcOptions& opt, cudaStream_t s) {
    if (k % 256 != 0 || k <= 0) return fail(GDN_ERR_SHAPE, "Q4_K tensor-core GEMM needs k %% 256 == 0 (k=%lld)", (long long)k);
    if (n <= 0 || m <= 0) return GDN_OK;
    if (n > INT32_MAX || m > INT32_MAX || k > INT32_MAX) return fail(GDN_ERR_SHAPE, "GEMM dims exceed int32");
    if (ldy < n) return fail(GDN_ERR_SHAPE, "ldy < n");
    if (!aligned(a, 16) || !aligned(blocks, 16))
        return fail(GDN_ERR_ARG, "Q4_K tensor-core GEMM operands must be 16-byte aligned");
    if (opt.a_blk_k > 0 || opt.a_nblocks > 0) return fail(GDN_ERR_ARG, "Q4_K tensor-core GEMM: plain activations only");
    const int KT = (int)(k / BK);
    int splits = opt.splits < 1 ? 1 : opt.splits;
    int kt_per = (KT + splits - 1) / splits;
    kt_per = (kt_per + kWin - 1) / kWin * kWin;  // whole superblocks and scale windows per split
    splits = (KT + kt_per - 1) / kt_per;
    float* out = y;
    int64_t ld_out = ldy;
    if (splits > 1) {
        if (opt.workspace == nullptr || opt.workspace_bytes < gemm_tc_workspace_bytes(m, n, splits))
            return fail(GDN_ERR_ARG, "split-K workspace too small");
        out = static_cast<float*>(opt.workspace);
        ld_out = n;
    }
    // exact weights (hi + lo fp16 operands); fp16 activations
    const int8_t* q = static_cast<const int8_t*>(blocks);
    ALayout al;
    const int st = m > BM ? run_tc<128, 2, 3, 2, 2, false, true, true>(q, nullptr, n, k, a, m, out, ld_out, splits,
                                                                       kt_per, al, s)
                          : run_tc<128, 1, 4, 3, 3, false, true, true>(q, nullptr, n, k, a, m, out, ld_out, splits,
                                                                       kt_per, al, s);
    if (st || splits == 1) return st;
    const int64_t cnt = m * n;
    return launch_pdl("splitk_reduce_kernel", splitk_reduce_kernel, dim3((unsigned)((cnt + 255) / 256)), dim3(256), 0,
                      s, (const float*)out, splits, m, n, y, ldy);
}

}  // namespace gdn
