// Glue of a stack of DeltaNet layers: residual add + RMSNorm of the hidden
// states between layers,
//   x[t] <- x[t] + add[t]             (winmoe_inference.c:1652, hidden = residual + o_out)
//   y[t]  = (x[t] * scale) * w        (attention.h:29-44, rmsnorm before each layer,
//   scale = 1 / sqrtf(float(sum x^2 / H) + 1e-6), the sum in double)
// One block per token row; y in fp32, bf16 or fp16 (the next layer's input),
// written to one buffer or broadcast to several (every rank's copy of the
// next layer's input, over NVLink).
#include "gdn_common.cuh"
#include "stack.cuh"

namespace gdn {

namespace {

constexpr int kNormThreads = 256;

template <typename E>
__device__ __forceinline__ E to_elem(float v);
template <>
__device__ __forceinline__ float to_elem<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_elem<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half to_elem<__half>(float v) { return __float2half_rn(v); }

// Four consecutive outputs as one store (16 B of fp32, 8 B of bf16 / fp16).
template <typename E>
__device__ __forceinline__ void store4(E* p, const float (&v)[4]) {
    if constexpr (sizeof(E) == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        union { E e[4]; uint2 u; } pk;
#pragma unroll
        for (int j = 0; j < 4; j++) pk.e[j] = to_elem<E>(v[j]);
        *reinterpret_cast<uint2*>(p) = pk.u;
    }
}

// y rows go to every destination: dst.ptr[b] + dst.col0 + row * dst.ld (a
// broadcast; with peers' buffers, plain stores over NVLink).  vec: hidden % 4
// == 0 and every base 16-byte aligned, so each thread moves 4 columns at once.
template <typename E, bool vec>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ add,
                                                                   const float* __restrict__ w, const RowDest dst,
                                                                   int64_t hidden) {
    pdl_trigger();
    pdl_wait();
    __shared__ double part[kNormThreads / 32];
    const int64_t row = blockIdx.x;
    float* xr = x + row * hidden;
    const float* ar = add != nullptr ? add + row * hidden : nullptr;
    constexpr int V = vec ? 4 : 1;
    double ss = 0.0;
    for (int64_t i = (int64_t)threadIdx.x * V; i < hidden; i += (int64_t)blockDim.x * V) {
        float v[V];
        if constexpr (vec) {
            const float4 a4 = *reinterpret_cast<const float4*>(xr + i);
            v[0] = a4.x, v[1] = a4.y, v[2] = a4.z, v[3] = a4.w;
        } else {
            v[0] = xr[i];
        }
        if (ar != nullptr) {
#pragma unroll
            for (int j = 0; j < V; j++) v[j] = __fadd_rn(v[j], ar[i + j]);
#pragma unroll
            for (int j = 0; j < V; j++) xr[i + j] = v[j];
        }
#pragma unroll
        for (int j = 0; j < V; j++) ss += (double)v[j] * (double)v[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; i++) tot += part[i];
    const float scale = 1.0f / sqrtf((float)(tot / (double)hidden) + 1e-6f);
    for (int64_t i = (int64_t)threadIdx.x * V; i < hidden; i += (int64_t)blockDim.x * V) {
        float v[4];
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = __fmul_rn(__fmul_rn(xr[i + j], scale), w != nullptr ? w[i + j] : 1.0f);
        for (int b = 0; b < dst.n; b++) {
            E* yr = static_cast<E*>(dst.ptr[b]) + dst.col0 + row * dst.ld + i;
            if constexpr (vec) store4<E>(yr, v);
            else yr[0] = to_elem<E>(v[0]);
        }
    }
}

template <typename E>
int launch_typed(float* x, const float* add, const float* w, const RowDest& dst, int64_t T, int64_t hidden,
                 cudaStream_t s) {
    bool vec = hidden % 4 == 0 && aligned(x, 16) && (add == nullptr || aligned(add, 16)) &&
               (w == nullptr || aligned(w, 16)) && (dst.col0 * (int64_t)sizeof(E)) % 16 == 0 &&
               (dst.ld * (int64_t)sizeof(E)) % 16 == 0 && hidden / 4 >= 1;
    for (int b = 0; b < dst.n; b++) vec = vec && aligned(dst.ptr[b], 16);
    if (vec)
        return launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel<E, true>, dim3((unsigned)T), dim3(kNormThreads), 0,
                          s, x, add, w, dst, hidden);
    return launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel<E, false>, dim3((unsigned)T), dim3(kNormThreads), 0, s,
                      x, add, w, dst, hidden);
}

}  // namespace

int launch_add_rmsnorm(float* x, const float* add, const float* w, const RowDest& y, int y_dtype, int64_t T,
                       int64_t hidden, cudaStream_t s) {
    if (T == 0) return GDN_OK;
    if (y_dtype == GDN_DTYPE_BF16) return launch_typed<__nv_bfloat16>(x, add, w, y, T, hidden, s);
    if (y_dtype == GDN_DTYPE_F16) return launch_typed<__half>(x, add, w, y, T, hidden, s);
    return launch_typed<float>(x, add, w, y, T, hidden, s);
}

}  // namespace gdn
