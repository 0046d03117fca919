// Warp-level bf16 tensor-core fragments (mma.sync m16n8k16, ldmatrix) for the
// small per-chunk products of the chunked prefill, plus 16-byte cp.async.
//
// Fragment layouts (lane = threadIdx.x % 32, g = lane / 4, q = lane % 4):
//   A 16x16 (row-major): a0 = (g, 2q..2q+1), a1 = (g+8, 2q..), a2 = (g, 8+2q..), a3 = (g+8, 8+2q..)
//   B 16x8  ("col"):      b0 = (k 2q..2q+1, n g), b1 = (k 8+2q.., n g)
//   C 16x8 fp32:          c0,c1 = (g, 2q..2q+1), c2,c3 = (g+8, 2q..2q+1)
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace gdn {
namespace wmma16 {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(saddr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(saddr(p)));
}

// D += A * B, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A tile (rows r0..r0+15, cols c0..c0+15) of a row-major matrix M[m][k] (ld elements).
__device__ __forceinline__ void load_a(uint32_t (&a)[4], const bf16* M, int ld, int r0, int c0) {
    const int t = threadIdx.x & 31;
    ldsm_x4(a, M + (r0 + (t & 15)) * ld + c0 + ((t >> 4) << 3));
}

// A tile where A[m][k] = M[k][m], M row-major (ld elements): rows r0.. of A, cols c0.. of A.
__device__ __forceinline__ void load_a_t(uint32_t (&a)[4], const bf16* M, int ld, int r0, int c0) {
    const int t = threadIdx.x & 31, j = t >> 3;
    ldsm_x4_t(a, M + (c0 + (t & 7) + ((j >> 1) << 3)) * ld + r0 + ((j & 1) << 3));
}

// Two B tiles (k0..k0+15; n0..n0+7 and n0+8..n0+15) with B[k][n] = M[n][k], M row-major:
// b[0], b[1] for the first n8 tile, b[2], b[3] for the second.
__device__ __forceinline__ void load_b_nk(uint32_t (&b)[4], const bf16* M, int ld, int k0, int n0) {
    const int t = threadIdx.x & 31, j = t >> 3;
    ldsm_x4(b, M + (n0 + (t & 7) + ((j >> 1) << 3)) * ld + k0 + ((j & 1) << 3));
}

// Two B tiles with B[k][n] = M[k][n], M row-major.
__device__ __forceinline__ void load_b_kn(uint32_t (&b)[4], const bf16* M, int ld, int k0, int n0) {
    const int t = threadIdx.x & 31, j = t >> 3;
    ldsm_x4_t(b, M + (k0 + (t & 7) + ((j & 1) << 3)) * ld + n0 + ((j >> 1) << 3));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// 16-byte global -> shared copy through the async-copy unit (L2 only).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace wmma16
}  // namespace gdn
