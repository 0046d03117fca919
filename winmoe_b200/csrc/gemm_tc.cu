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
//   split:   w = w_hi + w_lo * 2^-S with w_lo = round((w - w_hi) * 2^S)
//            (S = 11 for fp16, 8 for bf16), two MMAs into two TMEM
//            accumulators, y = acc_hi + acc_lo * 2^-S.  w_hi + w_lo*2^-S equals w
//            (fp16) or carries 16 of its bits (bf16), so the product differs
//            from an fp32 GEMV only by summation order -- the decode path
//            uses it to meet the 1e-3 parity bound.
//
// One CTA computes one BM x BN output tile (BM = 128 tokens, BN = 128/256
// weight rows) over its K range in BK = 64 steps, through a STAGES-deep ring:
//   warp 0     TMA producer: a tile (128B swizzle) + int8 weight tile
//   warp 1     TMEM allocator; lane 0 issues tcgen05.mma (M=128, N=BN, K=16)
//   warps 2-5  dequant int8 -> operand type into the swizzled B tile(s), then
//              the epilogue (tcgen05.ld TMEM -> registers -> global fp32)
// Barriers: full[s] (TMA bytes landed), deq[s] (128 dequant arrivals),
// empty[s] (MMA done reading stage s, via tcgen05.commit), accf (all MMAs done).
// Split-K (grid.z > 1) writes fp32 partials that a second kernel sums in a
// fixed order, so results do not depend on scheduling.
#include <cuda.h>
#include <type_traits>
#include "gdn_common.cuh"
#include "ptx_sm100.cuh"
#include "quant.cuh"

namespace gdn {

using namespace sm100;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kWin = 8;  // k-tiles per scale window (16 fp16 scales = 32 bytes per row)

template <int BN, int STAGES, bool SPLIT>
struct TcLayout {
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B16_BYTES = BN * BK * 2;
    static constexpr uint32_t B8_BYTES = BN * BK;
    static constexpr int NB = SPLIT ? 2 : 1;
    static constexpr uint32_t A_OFF = 0;
    static constexpr uint32_t B16_OFF = A_OFF + STAGES * A_BYTES;
    static constexpr uint32_t B8_OFF = B16_OFF + STAGES * NB * B16_BYTES;
    static constexpr uint32_t BAR_OFF = B8_OFF + STAGES * B8_BYTES;
    static constexpr uint32_t NBARS = 3 * STAGES + 1;
    static constexpr uint32_t TMEM_SLOT_OFF = BAR_OFF + NBARS * 8;
    static constexpr uint32_t BYTES = TMEM_SLOT_OFF + 16;
    static constexpr size_t SMEM = BYTES + 1024;  // + alignment slack
    static constexpr uint32_t TMEM_COLS = NB * BN;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(TMEM_COLS <= 512, "TMEM budget");
};

template <bool BF16>
struct OperandType;

template <>
struct OperandType<false> {  // fp16
    static constexpr float LO_SCALE = 2048.0f;
    static constexpr float LO_INV = 1.0f / 2048.0f;
    __device__ __forceinline__ static uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static float2 unpack(uint32_t u) {
        return __half22float2(*reinterpret_cast<__half2*>(&u));
    }
};

template <>
struct OperandType<true> {  // bf16
    static constexpr float LO_SCALE = 256.0f;
    static constexpr float LO_INV = 1.0f / 256.0f;
    __device__ __forceinline__ static uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static float2 unpack(uint32_t u) {
        return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
    }
};

// float of the four signed bytes of w (exact; see quant.cu).
__device__ __forceinline__ void i8x4_f32(uint32_t w, float* f) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
    f[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
    f[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
    f[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// 16 int8 weights times scale d -> operand words: hi[8] (and lo[8] when split).
template <bool BF16, bool SPLIT>
__device__ __forceinline__ void dequant16(const uint4 q, float d, uint32_t (&hi)[8], uint32_t (&lo)[8]) {
    using T = OperandType<BF16>;
    float f[16];
    i8x4_f32(q.x, f);
    i8x4_f32(q.y, f + 4);
    i8x4_f32(q.z, f + 8);
    i8x4_f32(q.w, f + 12);
#pragma unroll
    for (int p = 0; p < 8; p++) {
        const float w0 = __fmul_rn(f[2 * p], d), w1 = __fmul_rn(f[2 * p + 1], d);  // exact
        hi[p] = T::pack(w0, w1);
        if (SPLIT) {
            const float2 h = T::unpack(hi[p]);
            // both the difference and the power-of-two scaling are exact
            lo[p] = T::pack(__fmul_rn(__fsub_rn(w0, h.x), T::LO_SCALE), __fmul_rn(__fsub_rn(w1, h.y), T::LO_SCALE));
        }
    }
}

// Writes the 16-element chunk j (K elements 16j..16j+15) of row rr into a
// K-major 128B-swizzled tile: 16-byte unit u of row rr sits at unit u ^ (rr & 7).
__device__ __forceinline__ void store_chunk(uint8_t* tile, int rr, int j, const uint32_t (&w)[8]) {
    uint8_t* row = tile + (rr >> 3) * 1024 + (rr & 7) * 128;
    *reinterpret_cast<uint4*>(row + (((2 * j) ^ (rr & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(row + (((2 * j + 1) ^ (rr & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
}

template <int BN, int STAGES, bool BF16, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    q8_0_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const uint16_t* __restrict__ dsc, int n, int k, int m, float* __restrict__ y, int64_t ldy,
                        int kt_per_split, uint32_t* __restrict__ err) {
    using L = TcLayout<BN, STAGES, SPLIT>;
    using T = OperandType<BF16>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    auto full_bar = [&](int s) { return sbase + L::BAR_OFF + 8u * s; };
    auto deq_bar = [&](int s) { return sbase + L::BAR_OFF + 8u * (STAGES + s); };
    auto empty_bar = [&](int s) { return sbase + L::BAR_OFF + 8u * (2 * STAGES + s); };
    const uint32_t accf_bar = sbase + L::BAR_OFF + 8u * (3 * STAGES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::TMEM_SLOT_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int KT_total = k / BK;
    const int kt0 = blockIdx.z * kt_per_split;
    const int KT = min(kt_per_split, KT_total - kt0);  // k-tiles of this CTA (>= 1 by construction)

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(deq_bar(s), 128);
            mbar_init(empty_bar(s), 1);
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

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            bool ok = true;
            for (int t = 0; t < KT && ok; t++) {
                const int s = t % STAGES, r = t / STAGES;
                if (t >= STAGES) ok = mbar_wait(empty_bar(s), (r - 1) & 1, err);
                if (!ok) break;
                mbar_arrive_expect_tx(full_bar(s), L::A_BYTES + L::B8_BYTES);
                tma_load_2d(sbase + L::A_OFF + s * L::A_BYTES, &tm_a, (kt0 + t) * BK, m0, full_bar(s));
                tma_load_2d(sbase + L::B8_OFF + s * L::B8_BYTES, &tm_b, (kt0 + t) * BK, n0, full_bar(s));
                issued++;
            }
            if (!ok) {
                // Give the loads already issued a bounded chance to land before exit.
                for (int t = (issued > STAGES ? issued - STAGES : 0); t < issued; t++)
                    mbar_wait(full_bar(t % STAGES), (t / STAGES) & 1, err);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(BM, BN, BF16);
            for (int t = 0; t < KT; t++) {
                const int s = t % STAGES, r = t / STAGES;
                // the A tile (TMA) and the dequantised B tile(s) of this stage
                if (!(mbar_wait(full_bar(s), r & 1, err) && mbar_wait(deq_bar(s), r & 1, err))) break;
                tc_fence_after();
                const uint32_t a0 = sbase + L::A_OFF + s * L::A_BYTES;
                const uint32_t b0 = sbase + L::B16_OFF + s * L::NB * L::B16_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    const uint64_t ad = umma_desc_sw128(a0 + kk * 32);
                    const uint32_t acc = (t | kk) != 0 ? 1u : 0u;
                    mma_f16_ss(tmem, ad, umma_desc_sw128(b0 + kk * 32), idesc, acc);
                    if (SPLIT) mma_f16_ss(tmem + BN, ad, umma_desc_sw128(b0 + L::B16_BYTES + kk * 32), idesc, acc);
                }
                mma_commit(empty_bar(s));
            }
            mma_commit(accf_bar);
        }
    } else {
        // ---- dequant: thread i owns weight rows i (and i+128 when BN = 256)
        constexpr int R = BN / 128;
        const int i = threadIdx.x - 64;
        const int kb = k >> 5;
        const uint16_t* drow[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            const int gr = n0 + i + 128 * j;
            drow[j] = gr < n ? dsc + (int64_t)gr * kb + 2 * kt0 : nullptr;
        }
        // Scales are prefetched kWin k-tiles ahead in registers when every row's
        // window is 16-byte aligned; otherwise they are read per stage.
        const bool windowed = (kb % 8 == 0) && (kt0 % 4 == 0);
        uint4 cur[R][2], nxt[R][2];
        auto load_win = [&](uint4 (&dst)[R][2], int w) {
#pragma unroll
            for (int j = 0; j < R; j++) {
                const int t = w * kWin;
                if (drow[j] != nullptr && t < KT) {
                    const uint4* p = reinterpret_cast<const uint4*>(drow[j] + 2 * t);
                    dst[j][0] = __ldg(p);
                    dst[j][1] = (t + 4 < KT) ? __ldg(p + 1) : make_uint4(0, 0, 0, 0);
                } else {
                    dst[j][0] = dst[j][1] = make_uint4(0, 0, 0, 0);
                }
            }
        };
        if (windowed) {
            load_win(cur, 0);
            load_win(nxt, 1);
        }
        bool ok = true;
        for (int w = 0; w * kWin < KT && ok; w++) {
            if (windowed && w > 0) {
#pragma unroll
                for (int j = 0; j < R; j++) {
                    cur[j][0] = nxt[j][0];
                    cur[j][1] = nxt[j][1];
                }
                load_win(nxt, w + 1);
            }
#pragma unroll
            for (int u = 0; u < kWin; u++) {
                const int t = w * kWin + u;
                if (t >= KT) break;
                const int s = t % STAGES, r = t / STAGES;
                ok = mbar_wait(full_bar(s), r & 1, err);
                if (!ok) break;
                const uint8_t* b8 = smem + L::B8_OFF + s * L::B8_BYTES;
                uint8_t* bhi = smem + L::B16_OFF + s * L::NB * L::B16_BYTES;
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const int rr = i + 128 * j;
                    uint32_t sc2;
                    if (windowed) {
                        const uint4 v = cur[j][u >> 2];
                        sc2 = (u & 3) == 0 ? v.x : (u & 3) == 1 ? v.y : (u & 3) == 2 ? v.z : v.w;
                    } else {
                        sc2 = drow[j] != nullptr ? __ldg(reinterpret_cast<const uint32_t*>(drow[j] + 2 * t)) : 0u;
                    }
                    const float d0 = fp16_bits_to_float((uint16_t)(sc2 & 0xFFFFu));
                    const float d1 = fp16_bits_to_float((uint16_t)(sc2 >> 16));
                    const uint4* src = reinterpret_cast<const uint4*>(b8 + rr * BK);
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        uint32_t hi[8], lo[8];
                        dequant16<BF16, SPLIT>(src[c], c < 2 ? d0 : d1, hi, lo);
                        store_chunk(bhi, rr, c, hi);
                        if (SPLIT) store_chunk(bhi + L::B16_BYTES, rr, c, lo);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(deq_bar(s));
            }
        }
        // ---- epilogue: warp quadrant q reads TMEM lanes [32q, 32q+32)
        if (ok) ok = mbar_wait(accf_bar, 0, err);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
        tc_fence_after();
        const int q = warp & 3;
        const int row = m0 + q * 32 + lane;
        float* ybase = y + (int64_t)blockIdx.z * (int64_t)m * ldy;  // split-K partial slice
        const bool vec_ok = ((ldy & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
        if (ok) {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
                if (SPLIT) {
                    uint32_t vl[32];
                    tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), vl);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        v[j] = __float_as_uint(fmaf(__uint_as_float(vl[j]), T::LO_INV, __uint_as_float(v[j])));
                } else {
                    tmem_ld_wait();
                }
                if (row < m) {
                    float* yr = ybase + (int64_t)row * ldy + n0 + c0;
                    if (vec_ok && n0 + c0 + 32 <= n) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4*>(yr + j) =
                                make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                            __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (n0 + c0 + j < n) yr[j] = __uint_as_float(v[j]);
                    }
                }
            }
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
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m * n) return;
    const int64_t r = i / n, c = i - r * n;
    float s = 0.0f;
    for (int z = 0; z < splits; z++) s += part[(int64_t)z * m * n + i];
    y[r * ldy + c] = s;
}

template <typename OutT>
__global__ void convert_kernel(const void* __restrict__ x, int dtype, OutT* __restrict__ out, int64_t count) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float v = load_act(x, dtype, i);
    if constexpr (std::is_same<OutT, __half>::value) out[i] = __float2half_rn(v);
    else out[i] = __float2bfloat16_rn(v);
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

template <int BN, int STAGES, bool BF16, bool SPLIT>
int run_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* a, int64_t m, float* out,
           int64_t ld_out, int splits, int kt_per, cudaStream_t s) {
    using L = TcLayout<BN, STAGES, SPLIT>;
    CUtensorMap ma, mb;
    int st = make_map_2d(&ma, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, (uint64_t)k,
                         (uint64_t)m, (uint64_t)k * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, qs, (uint64_t)k, (uint64_t)n, (uint64_t)k, BK, BN,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    auto kern = q8_0_gemm_tc_kernel<BN, STAGES, BF16, SPLIT>;
    GDN_CUDA(cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM));
    const dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM), (unsigned)splits);
    kern<<<grid, kThreads, L::SMEM, s>>>(ma, mb, d, (int)n, (int)k, (int)m, out, ld_out, kt_per,
                                         device_error_word());
    GDN_LAUNCH_CHECK("q8_0_gemm_tc_kernel");
    return GDN_OK;
}

}  // namespace

int launch_convert(const void* x, int x_dtype, void* out, bool to_bf16, int64_t count, cudaStream_t s) {
    if (count == 0) return GDN_OK;
    const unsigned g = (unsigned)((count + 255) / 256);
    if (to_bf16) convert_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(x, x_dtype, static_cast<__nv_bfloat16*>(out), count);
    else convert_kernel<__half><<<g, 256, 0, s>>>(x, x_dtype, static_cast<__half*>(out), count);
    GDN_LAUNCH_CHECK("convert_kernel");
    return GDN_OK;
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
    int st;
    if (opt.split_precision) {
        st = a_bf16 ? run_tc<128, 4, true, true>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, s)
                    : run_tc<128, 4, false, true>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, s);
    } else {
        const int64_t tiles256 = ((n + 255) / 256) * ((m + BM - 1) / BM) * splits;
        if (tiles256 >= 148)
            st = a_bf16 ? run_tc<256, 3, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, s)
                        : run_tc<256, 3, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, s);
        else
            st = a_bf16 ? run_tc<128, 4, true, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, s)
                        : run_tc<128, 4, false, false>(qs, d, n, k, a, m, out, ld_out, splits, kt_per, s);
    }
    if (st || splits == 1) return st;
    const int64_t cnt = m * n;
    splitk_reduce_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, s>>>(out, splits, m, n, y, ldy);
    GDN_LAUNCH_CHECK("splitk_reduce_kernel");
    return GDN_OK;
}

}  // namespace gdn
