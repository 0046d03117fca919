// Glue of a stack of DeltaNet layers: residual add + RMSNorm of the hidden
// states between layers,
//   x[t] <- x[t] + add[t]             (winmoe_inference.c:1652, hidden = residual + o_out)
//   y[t]  = (x[t] * scale) * w        (attention.h:29-44, rmsnorm before each layer,
//   scale = 1 / sqrtf(float(sum x^2 / H) + 1e-6), the sum in double)
// One block per token row; y in fp32, bf16 or fp16 (the next layer's input).
#include "gdn_common.cuh"
#include "stack.cuh"

namespace gdn {

namespace {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ add,
                                                                   const float* __restrict__ w, void* __restrict__ y,
                                                                   int y_dtype, int64_t hidden) {
    pdl_trigger();
    pdl_wait();
    __shared__ double part[kNormThreads / 32];
    const int64_t row = blockIdx.x;
    float* xr = x + row * hidden;
    const float* ar = add != nullptr ? add + row * hidden : nullptr;
    double ss = 0.0;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v = xr[i];
        if (ar != nullptr) {
            v = __fadd_rn(v, ar[i]);
            xr[i] = v;
        }
        ss += (double)v * (double)v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; i++) tot += part[i];
    const float scale = 1.0f / sqrtf((float)(tot / (double)hidden) + 1e-6f);
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(xr[i], scale), w != nullptr ? w[i] : 1.0f);
        const int64_t o = row * hidden + i;
        if (y_dtype == GDN_DTYPE_BF16) static_cast<__nv_bfloat16*>(y)[o] = __float2bfloat16_rn(v);
        else if (y_dtype == GDN_DTYPE_F16) static_cast<__half*>(y)[o] = __float2half_rn(v);
        else static_cast<float*>(y)[o] = v;
    }
}

}  // namespace

int launch_add_rmsnorm(float* x, const float* add, const float* w, void* y, int y_dtype, int64_t T, int64_t hidden,
                       cudaStream_t s) {
    if (T == 0) return GDN_OK;
    return launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel, dim3((unsigned)T), dim3(kNormThreads), 0, s, x, add,
                      w, y, y_dtype, hidden);
}

}  // namespace gdn
