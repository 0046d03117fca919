// Q8_0 dequant-GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
//   y[m][n] = sum_k a[m][k] * W[n][k]
//   a: fp16 [m][k] activations (tokens / sequences), row-major
//   W: Q8_0 planes qs [n][k] int8 and d [n][k/32] fp16 (see gdn_q8_0_repack)
//
// This is the batched form of quant_matvec type 8 (engine/runtime/transformer.h
// :157-194; the reference GPU kernel is engine/runtime/gpu_offload.cu:152-199).
// The weights are never materialised in HBM: each int8 tile arrives in shared
// memory by TMA and is dequantised there to fp16 (d*q rounded once) straight
// into the MMA operand layout.
//
// One CTA computes one BM x BN output tile (BM = 128 tokens, BN = 128/256
// weight rows) over K in BK = 64 steps, through a STAGES-deep ring:
//   warp 0     TMA producer: a tile (128B swizzle) + int8 weight tile
//   warp 1     TMEM allocator; lane 0 issues tcgen05.mma (M=128, N=BN, K=16) x4
//   warps 2-5  dequant int8 -> fp16 into the swizzled B tile, then the
//              epilogue (tcgen05.ld TMEM -> registers -> global fp32)
// Barriers: full[s] (TMA bytes landed), deq[s] (128 dequant arrivals),
// empty[s] (MMA done reading stage s, via tcgen05.commit), accf (all MMAs done).
#include <cuda.h>
#include "gdn_common.cuh"
#include "ptx_sm100.cuh"
#include "quant.cuh"

namespace gdn {

using namespace sm100;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;

template <int BN, int STAGES>
struct TcLayout {
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B16_BYTES = BN * BK * 2;
    static constexpr uint32_t B8_BYTES = BN * BK;
    static constexpr uint32_t A_OFF = 0;
    static constexpr uint32_t B16_OFF = A_OFF + STAGES * A_BYTES;
    static constexpr uint32_t B8_OFF = B16_OFF + STAGES * B16_BYTES;
    static constexpr uint32_t BAR_OFF = B8_OFF + STAGES * B8_BYTES;
    static constexpr uint32_t NBARS = 3 * STAGES + 1;
    static constexpr uint32_t TMEM_SLOT_OFF = BAR_OFF + NBARS * 8;
    static constexpr uint32_t BYTES = TMEM_SLOT_OFF + 16;
    static constexpr size_t SMEM = BYTES + 1024;  // + alignment slack
};

// 16 int8 weights (one uint4) times scale -> 16 fp16 in two uint4 (8 each).
// Each byte q becomes fp16(1024 + (q+128)) - 1152 = q exactly, then one
// correctly rounded fp16 multiply by d.
__device__ __forceinline__ void dequant16(const uint4 q, __half2 d2, uint4& lo, uint4& hi) {
    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480));  // 1152
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint32_t p0 = __byte_perm(w[j], 0x64646464u, 0x4140);
        uint32_t p1 = __byte_perm(w[j], 0x64646464u, 0x4342);
        __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&p0), bias), d2);
        __half2 h1 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&p1), bias), d2);
        o[2 * j] = *reinterpret_cast<uint32_t*>(&h0);
        o[2 * j + 1] = *reinterpret_cast<uint32_t*>(&h1);
    }
    lo = make_uint4(o[0], o[1], o[2], o[3]);
    hi = make_uint4(o[4], o[5], o[6], o[7]);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    q8_0_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const uint16_t* __restrict__ dsc, int n, int k, int m, float* __restrict__ y,
                        uint32_t* __restrict__ err) {
    using L = TcLayout<BN, STAGES>;
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
    const int KT = k / BK;

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
        tmem_alloc(smem_u32(tmem_slot), BN);
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
            for (int kt = 0; kt < KT && ok; kt++) {
                const int s = kt % STAGES, r = kt / STAGES;
                if (kt >= STAGES) ok = mbar_wait(empty_bar(s), (r - 1) & 1, err);
                if (!ok) break;
                mbar_arrive_expect_tx(full_bar(s), L::A_BYTES + L::B8_BYTES);
                tma_load_2d(sbase + L::A_OFF + s * L::A_BYTES, &tm_a, kt * BK, m0, full_bar(s));
                tma_load_2d(sbase + L::B8_OFF + s * L::B8_BYTES, &tm_b, kt * BK, n0, full_bar(s));
                issued++;
            }
            if (!ok) {
                // Give the loads already issued a bounded chance to land before exit.
                for (int kt = (issued > STAGES ? issued - STAGES : 0); kt < issued; kt++)
                    mbar_wait(full_bar(kt % STAGES), (kt / STAGES) & 1, err);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(BM, BN, false);
            bool ok = true;
            for (int kt = 0; kt < KT; kt++) {
                const int s = kt % STAGES, r = kt / STAGES;
                // the A tile (TMA) and the dequantised B tile of this stage
                ok = mbar_wait(full_bar(s), r & 1, err) && mbar_wait(deq_bar(s), r & 1, err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a0 = sbase + L::A_OFF + s * L::A_BYTES;
                const uint32_t b0 = sbase + L::B16_OFF + s * L::B16_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)
                    mma_f16_ss(tmem, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), idesc,
                               (kt | kk) != 0 ? 1u : 0u);
                mma_commit(empty_bar(s));
            }
            mma_commit(accf_bar);
        }
    } else {
        // ---- dequant: thread i owns weight rows i (and i+128 when BN = 256)
        const int i = threadIdx.x - 64;
        const int kb = k >> 5;
        bool ok = true;
        for (int kt = 0; kt < KT; kt++) {
            const int s = kt % STAGES, r = kt / STAGES;
            ok = mbar_wait(full_bar(s), r & 1, err);
            if (!ok) break;
            const uint8_t* b8 = smem + L::B8_OFF + s * L::B8_BYTES;
            uint8_t* b16 = smem + L::B16_OFF + s * L::B16_BYTES;
#pragma unroll
            for (int rr0 = 0; rr0 < BN; rr0 += 128) {
                const int rr = rr0 + i;
                const int gr = n0 + rr;
                uint32_t sc2 = 0;
                if (gr < n) sc2 = __ldg(reinterpret_cast<const uint32_t*>(dsc + (int64_t)gr * kb + 2 * kt));
                const __half2 dlo = __half2half2(__ushort_as_half((unsigned short)(sc2 & 0xFFFFu)));
                const __half2 dhi = __half2half2(__ushort_as_half((unsigned short)(sc2 >> 16)));
                const uint4* src = reinterpret_cast<const uint4*>(b8 + rr * BK);
                uint8_t* dst = b16 + (rr >> 3) * 1024 + (rr & 7) * 128;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint4 lo, hi;
                    dequant16(src[j], j < 2 ? dlo : dhi, lo, hi);
                    *reinterpret_cast<uint4*>(dst + (((2 * j) ^ (rr & 7)) << 4)) = lo;
                    *reinterpret_cast<uint4*>(dst + (((2 * j + 1) ^ (rr & 7)) << 4)) = hi;
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(deq_bar(s));
        }
        // ---- epilogue: warp quadrant q reads TMEM lanes [32q, 32q+32)
        if (ok) ok = mbar_wait(accf_bar, 0, err);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
        tc_fence_after();
        const int q = warp & 3;
        const int row = m0 + q * 32 + lane;
        const bool vec_ok = ((n & 3) == 0) && ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
        if (ok) {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
                tmem_ld_wait();
                if (row < m) {
                    float* yr = y + (int64_t)row * n + n0 + c0;
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
        tmem_dealloc(tmem, BN);
    }
}

__global__ void to_f16_kernel(const void* __restrict__ x, int dtype, __half* __restrict__ out, int64_t count) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) out[i] = __float2half_rn(load_act(x, dtype, i));
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

template <int BN, int STAGES>
int run_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const __half* a, int64_t m, float* y,
           cudaStream_t s) {
    using L = TcLayout<BN, STAGES>;
    CUtensorMap ma, mb;
    int st = make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, (uint64_t)k, (uint64_t)m, (uint64_t)k * 2, BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, qs, (uint64_t)k, (uint64_t)n, (uint64_t)k, BK, BN,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    GDN_CUDA(cudaFuncSetAttribute((const void*)q8_0_gemm_tc_kernel<BN, STAGES>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::SMEM));
    const dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
    q8_0_gemm_tc_kernel<BN, STAGES><<<grid, kThreads, L::SMEM, s>>>(ma, mb, d, (int)n, (int)k, (int)m, y,
                                                                    device_error_word());
    GDN_LAUNCH_CHECK("q8_0_gemm_tc_kernel");
    return GDN_OK;
}

}  // namespace

int launch_to_f16(const void* x, int x_dtype, __half* out, int64_t count, cudaStream_t s) {
    if (count == 0) return GDN_OK;
    to_f16_kernel<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(x, x_dtype, out, count);
    GDN_LAUNCH_CHECK("to_f16_kernel");
    return GDN_OK;
}

int launch_q8_0_gemm_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const __half* a, int64_t m,
                        float* y, cudaStream_t s) {
    if (k % BK != 0) return fail(GDN_ERR_SHAPE, "tensor-core GEMM needs k %% 64 == 0 (k=%lld)", (long long)k);
    if (n <= 0 || m <= 0) return GDN_OK;
    if (n > INT32_MAX || m > INT32_MAX || k > INT32_MAX) return fail(GDN_ERR_SHAPE, "GEMM dims exceed int32");
    if (!aligned(a, 16) || !aligned(qs, 16) || !aligned(d, 4))
        return fail(GDN_ERR_ARG, "tensor-core GEMM operands must be 16-byte aligned (scales 4-byte)");
    const int64_t tiles256 = ((n + 255) / 256) * ((m + BM - 1) / BM);
    if (tiles256 >= 148) return run_tc<256, 3>(qs, d, n, k, a, m, y, s);
    return run_tc<128, 4>(qs, d, n, k, a, m, y, s);
}

}  // namespace gdn
