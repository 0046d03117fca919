// Shared definitions of the sm_100a Gated DeltaNet library: status plumbing,
// dtype loads, and the device error word that bounded waits report through.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/winmoe_gdn.h"

namespace gdn {

// Sets the thread-local error string; returns `st` so call sites can write
// `return fail(GDN_ERR_SHAPE, "...")`.
int fail(int st, const char* fmt, ...);
// Maps a CUDA error to GDN_ERR_CUDA with its name; GDN_OK if none.
int cuda_status(cudaError_t e, const char* what);

#define GDN_CUDA(call)                                                  \
    do {                                                                \
        cudaError_t e__ = (call);                                       \
        if (e__ != cudaSuccess) return ::gdn::cuda_status(e__, #call);  \
    } while (0)

// After a launch: reports configuration errors (not asynchronous faults).
#define GDN_LAUNCH_CHECK(name)                                          \
    do {                                                                \
        cudaError_t e__ = cudaGetLastError();                           \
        if (e__ != cudaSuccess) return ::gdn::cuda_status(e__, name);   \
    } while (0)

// Device error word: bit 0 = a bounded wait gave up.  Kernels OR into it and
// return; gdn_check_device_error reads and clears it.
enum : uint32_t { DEV_ERR_TIMEOUT = 1u, DEV_ERR_BOUNDS = 2u };
uint32_t* device_error_word();  // per-device __device__ word, looked up once per device
int sm_count();                  // SMs of the current device (cached per device)

// Where a kernel writes row t of a [T][width] output: token slice r = t / rows
// (rows = T for one destination) goes to ptr[r] + (t - r rows) ld + col0, in
// elements.  With the ptr[r] of other GPUs (CUDA IPC) the writes are plain
// peer stores over NVLink: a producer kernel scatters its rows to the ranks
// that consume them, and every byte crosses the link once.
constexpr int kMaxRowDest = 8;
struct RowDest {
    void* ptr[kMaxRowDest];
    int64_t rows;  // rows per destination
    int64_t ld;    // row pitch, elements
    int64_t col0;  // first column, elements
    int n;
    template <typename E>
    __device__ __forceinline__ E* row(int64_t t) const {
        const int64_t r = t / rows;
        return static_cast<E*>(pick(r)) + (t - r * rows) * ld + col0;
    }
    // ptr[r] by a chain of constant-index selects: a dynamic index into the
    // kernel parameter's array would go through local memory on every call.
    __device__ __forceinline__ void* pick(int64_t r) const {
        void* p = ptr[0];
#pragma unroll
        for (int i = 1; i < kMaxRowDest; i++)
            if (r == i) p = ptr[i];
        return p;
    }
};

// Programmatic dependent launch.  Kernels started with launch_pdl may be
// scheduled while their predecessor in the stream is still running: each kernel
// calls pdl_trigger() on entry (its own dependents may then be scheduled once
// every CTA has started) and pdl_wait() before it touches any global memory that
// an earlier kernel writes or reads (it returns once the predecessor has completed
// and its writes are visible; without PDL it returns at once).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
int launch_pdl(const char* name, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
               Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    return e == cudaSuccess ? 0 : cuda_status(e, name);
}

__device__ __forceinline__ float tanh_hw(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// SiLU(x) = x sigmoid(x) = x (1 + tanh(x / 2)) / 2: one special-function op.
__device__ __forceinline__ float silu_fast(float x) {
    const float h = 0.5f * x;
    return fmaf(h, tanh_hw(h), h);
}

// 1 / (sqrt(ss) + 1e-6), the L2 normalisation of q and k (deltanet_impl.h:89),
// branch-free: above ss = 1e-4 the epsilon moves the result by under 1e-4
// relative and one rsqrt is as good; below it sqrt(ss) = ss rsqrt(ss) (0 at 0)
// and a fast reciprocal, within a few ulp of the exact expression.
__device__ __forceinline__ float inv_l2(float ss) {
    const float r = rsqrtf(ss);
    const float root = ss > 0.0f ? ss * r : 0.0f;
    return ss > 1e-4f ? r : __fdividef(1.0f, root + 1e-6f);
}

// Spin limit of bounded waits, in SM clock cycles (~1 s at 1.9 GHz).
constexpr long long kWaitCycles = 2000000000LL;

__device__ __forceinline__ float load_act(const void* p, int dtype, size_t i) {
    if (dtype == GDN_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    if (dtype == GDN_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
    return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ float fp16_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace gdn
