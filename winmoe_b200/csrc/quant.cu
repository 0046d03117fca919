// GGUF Q8_0 / Q4_K kernels on CUDA cores: repack, bit-exact dequant, and the
// dequant-in-registers GEMV used for small activation batches (decode B=1..63,
// the Q4_K projection sweep).  The tensor-core path for large batches lives in
// gemm_tc.cu.
//
// Reference semantics:
//   Q8_0 block {fp16 d; int8 qs[32]}          engine/runtime/q8_dequant.h:15-18
//   Q8_0 dequant w = d*q                       engine/runtime/q8_dequant.h:116-126
//   Q8_0 GEMV, fp32 activations                engine/runtime/gpu_offload.cu:152-199
//   Q4_K block {d; dmin; scales[12]; qs[128]}  engine/runtime/q4k_dequant.h:28-33
//   Q4_K scale/min decode                      engine/runtime/gpu_offload.cu:90-98
//   Q4_K dequant (d*sc)*q - dmin*m, GGML nibble layout
//                                              engine/runtime/gpu_offload.cu:237-250
#include "gdn_common.cuh"
#include "quant.cuh"
#include <algorithm>
#include <string.h>

namespace gdn {

// ------------------------------------------------------------------ helpers

// float(q) for the four signed bytes of `w`: sets each byte (biased by 128) as
// the low mantissa bits of 2^23 and subtracts 2^23+128.  Exact.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float f[4]) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
    f[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
    f[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
    f[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
}

// float of the 4-bit values 0..15 in the low nibbles of the four bytes of `w`.
__device__ __forceinline__ void u4x4_to_f32(uint32_t w, float f[4]) {
    const uint32_t u = w & 0x0F0F0F0Fu;
    f[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388608.0f;
    f[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388608.0f;
    f[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388608.0f;
    f[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388608.0f;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------ Q8_0 planes

__global__ void q8_0_repack_kernel(const uint8_t* __restrict__ blocks, int8_t* __restrict__ qs,
                                   uint16_t* __restrict__ d, int64_t nblocks) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint8_t* b = blocks + i * 34;
    d[i] = (uint16_t)(b[0] | (b[1] << 8));
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; j++)
        w[j] = (uint32_t)b[2 + 4 * j] | ((uint32_t)b[3 + 4 * j] << 8) | ((uint32_t)b[4 + 4 * j] << 16) |
               ((uint32_t)b[5 + 4 * j] << 24);
    uint4* dst = reinterpret_cast<uint4*>(qs + i * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// One thread per 16 weights.  out = float(d) * float(q), a single rounding,
// as q8_dequant_row computes it.
__global__ void q8_0_dequant_kernel(const int8_t* __restrict__ qs, const uint16_t* __restrict__ d,
                                    float* __restrict__ out, int64_t n16) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n16) return;
    const uint4 q = reinterpret_cast<const uint4*>(qs)[i];
    const float s = fp16_bits_to_float(d[i >> 1]);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    float4* o = reinterpret_cast<float4*>(out + i * 16);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float f[4];
        i8x4_to_f32(qw[j], f);
        o[j] = make_float4(__fmul_rn(s, f[0]), __fmul_rn(s, f[1]), __fmul_rn(s, f[2]), __fmul_rn(s, f[3]));
    }
}

// Activation rows staged in shared memory as fp32: xs[m][k].
__device__ __forceinline__ void stage_x(float* xs, const void* x, int dtype, int64_t m0, int mb,
                                        int64_t k) {
    const int64_t n = (int64_t)mb * k;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) xs[i] = load_act(x, dtype, m0 * k + i);
}

// The same with 4 floats of padding after every 16 (row length kp = k * 5 / 4):
// 16-element chunks that consecutive lanes read start on distinct bank groups.
__device__ __forceinline__ int64_t padded(int64_t i) { return i + ((i >> 4) << 2); }
__device__ __forceinline__ void stage_x_padded(float* xs, const void* x, int dtype, int64_t m0, int mb,
                                               int64_t k) {
    const int64_t kp = k + (k >> 2);
    for (int j = 0; j < mb; j++)
        for (int64_t e = threadIdx.x; e < k; e += blockDim.x)
            xs[j * kp + padded(e)] = load_act(x, dtype, (m0 + j) * k + e);
}

// Q8_0 GEMV: each warp owns one weight row at a time; lane l reads the 16-byte
// chunks l, l+32, ... of the row's int8 plane (coalesced 512 B per warp load)
// and the fp16 scale of the 32-block each chunk belongs to.  The block sum
// sum(q*x) is scaled by d once per 16-chunk.  The MB activation rows of block
// row blockIdx.y share every weight load.  Weight loads run one batch (four
// chunks per lane) ahead: the first batch is issued before the activations are
// staged, and each next batch -- of this row or of the warp's next row --
// before the current one is reduced, so HBM latency overlaps the staging, the
// arithmetic and the row sums.
template <int MB>
__global__ void __launch_bounds__(256) q8_0_gemv_kernel(const int8_t* __restrict__ qs,
                                                       const uint16_t* __restrict__ dsc,
                                                       int64_t n_rows, int64_t k, const void* x,
                                                       int x_dtype, int64_t m, float* __restrict__ y,
                                                       int64_t ldy, int rows_per_block) {
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int64_t nchunk = k >> 4;
    const int64_t row0 = (int64_t)blockIdx.x * rows_per_block;
    const int64_t row_end = min(row0 + rows_per_block, n_rows);
    uint4 qv[4];
    uint16_t sv[4];
    auto load = [&](int64_t r, int64_t c0) {  // batch of chunks c0 + 32u of row r
        const uint4* qrow = reinterpret_cast<const uint4*>(qs + r * k);
        const uint16_t* drow = dsc + r * (k >> 5);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t c = c0 + 32 * u;
            if (c < nchunk) {
                qv[u] = __ldg(qrow + c);
                sv[u] = __ldg(drow + (c >> 1));
            }
        }
    };
    int64_t r = row0 + warp, c0 = lane;
    bool have = r < row_end;
    if (have) load(r, c0);  // weights never come from an earlier kernel: before the wait
    pdl_wait();
    extern __shared__ float xs[];  // [mb][k * 5 / 4], padded (lane l reads chunk l)
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    const int64_t kp = k + (k >> 2);
    stage_x_padded(xs, x, x_dtype, m0, mb, k);
    __syncthreads();
    float acc[MB];
#pragma unroll
    for (int j = 0; j < MB; j++) acc[j] = 0.0f;
    while (have) {
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t c = c0 + 32 * u;
            if (c >= nchunk) break;
            const float s = fp16_bits_to_float(sv[u]);
            float f[16];
            i8x4_to_f32(qv[u].x, f);
            i8x4_to_f32(qv[u].y, f + 4);
            i8x4_to_f32(qv[u].z, f + 8);
            i8x4_to_f32(qv[u].w, f + 12);
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (j < mb) {
                    const float4* xv = reinterpret_cast<const float4*>(xs + (int64_t)j * kp + c * 20);
                    float bs = 0.0f;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float4 v = xv[e];
                        bs = fmaf(f[4 * e + 0], v.x, bs);
                        bs = fmaf(f[4 * e + 1], v.y, bs);
                        bs = fmaf(f[4 * e + 2], v.z, bs);
                        bs = fmaf(f[4 * e + 3], v.w, bs);
                    }
                    acc[j] = fmaf(s, bs, acc[j]);
                }
            }
        }
        const bool row_done = c0 + 4 * 32 >= nchunk;
        const int64_t nr = row_done ? r + nwarps : r, nc0 = row_done ? (int64_t)lane : c0 + 4 * 32;
        const bool next = nr < row_end;
        if (next) load(nr, nc0);
        if (row_done) {
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (j < mb) {
                    const float v = warp_sum(acc[j]);
                    if (lane == 0) y[(m0 + j) * ldy + r] = v;
                }
                acc[j] = 0.0f;
            }
        }
        r = nr;
        c0 = nc0;
        have = next;
    }
}

// ---------------------------------------------- reference-exact projection
//
// quant_matvec type 8 exactly as the reference's CPU computes it
// (engine/runtime/transformer.h:157-194 -> q8_matvec, q8_dequant.h:63-113):
//   k >= 256 and n >= 128: x -> Q8_K per 256 values (quantize_block_q8_K,
//     q8k_quant.h:32-93: d = amax / 127, q = RNE(x * (1/d)) clamped to +-127),
//     every 32-block term (fp16(d_w) * d_a) * float(sum q_w q_a) (q8_dot_q8k,
//     q8_dequant.h:35-61; the integer sum is exact); as in the reference
//     (q8_dequant.h:75-79, 88-101) only the blocks of whole 256-value groups
//     enter this branch's sum;
//   otherwise: per 32-block, 16 lanes of two fused products, the
//     _mm512_reduce_add_ps tree, times d_w (q8_dot_block, q8_dequant.h:21-32).
// The row sum adds the block terms strictly in block order, as the reference's
// loop does, so every output is bit-identical to the CPU's.

// Q8_K block of 256 activations in shared memory: d, then qs.
struct Q8KSmem {
    float d;
    int8_t qs[256];
};

// One warp quantises 256 values (quantize_block_q8_K); lane l holds x[8l..8l+7].
__device__ __forceinline__ void quantize_q8_K_warp(const float (&v)[8], int lane, float& d_out, int8_t (&q)[8]) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (amax < 1e-10f) {
        d_out = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) q[j] = 0;
        return;
    }
    const float d = amax / 127.0f;  // correctly rounded division and reciprocal, as the CPU's
    const float id = 1.0f / d;
    d_out = d;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int v8 = __float2int_rn(__fmul_rn(v[j], id));  // cvtps_epi32: round to nearest even
        v8 = v8 < -127 ? -127 : (v8 > 127 ? 127 : v8);
        q[j] = (int8_t)v8;
    }
}

// GGUF block_q8_K {float d; int8 qs[256]; int16 bsums[16]} (292 bytes) per 256 values.
__global__ void quantize_q8_K_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
    pdl_trigger();
    pdl_wait();
    const int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (blk >= nblocks) return;
    const int lane = threadIdx.x & 31;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = x[blk * 256 + lane * 8 + j];
    float d;
    int8_t q[8];
    quantize_q8_K_warp(v, lane, d, q);
    uint8_t* ob = out + blk * 292;
    int s = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        ob[4 + lane * 8 + j] = (uint8_t)q[j];
        s += q[j];
    }
    s += __shfl_down_sync(0xffffffffu, s, 1);  // the 16-value group of lanes 2g, 2g+1
    if ((lane & 1) == 0) {
        const int16_t bs = (int16_t)s;
        memcpy(ob + 4 + 256 + lane, &bs, 2);
    }
    if (lane == 0) memcpy(ob, &d, 4);
}

// The _mm512_reduce_add_ps tree over 16 lanes.
__device__ __forceinline__ float hsum16_tree(const float (&a)[16]) {
    float t3[8], t6[4];
#pragma unroll
    for (int i = 0; i < 8; i++) t3[i] = __fadd_rn(a[8 + i], a[i]);
#pragma unroll
    for (int i = 0; i < 4; i++) t6[i] = __fadd_rn(t3[4 + i], t3[i]);
    return __fadd_rn(__fadd_rn(t6[0], t6[2]), __fadd_rn(t6[1], t6[3]));
}

// One warp per weight row, MB activation rows per block row (grid.y).  Lane l
// forms the terms of blocks l, l+32, ...; the row sum replays them in order.
constexpr int kRefMaxBlocksPerLane = 8;  // k <= 8192

template <int MB>
__global__ void __launch_bounds__(256) q8_0_gemv_ref_kernel(const int8_t* __restrict__ qs,
                                                           const uint16_t* __restrict__ dsc, int64_t n_rows,
                                                           int64_t k, const float* __restrict__ x, int64_t m,
                                                           float* __restrict__ y, int64_t ldy, int use_q8k) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ uint8_t sm_raw[];
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int64_t nk = k >> 8;
    const int64_t nb = use_q8k ? nk * 8 : k >> 5;  // blocks that enter the sum
    Q8KSmem* xq = reinterpret_cast<Q8KSmem*>(sm_raw);  // [mb][nk] when use_q8k
    float* xf = reinterpret_cast<float*>(sm_raw);      // [mb][k] otherwise
    if (use_q8k) {
        for (int64_t qb = warp; qb < (int64_t)mb * nk; qb += nwarps) {
            const int64_t j = qb / nk, kb = qb % nk;
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = x[(m0 + j) * k + kb * 256 + lane * 8 + e];
            float d;
            int8_t q[8];
            quantize_q8_K_warp(v, lane, d, q);
            Q8KSmem& b = xq[qb];
#pragma unroll
            for (int e = 0; e < 8; e++) b.qs[lane * 8 + e] = q[e];
            if (lane == 0) b.d = d;
        }
    } else {
        for (int64_t i = threadIdx.x; i < (int64_t)mb * k; i += blockDim.x) xf[i] = x[m0 * k + i];
    }
    __syncthreads();
    for (int64_t r = (int64_t)blockIdx.x * nwarps + warp; r < n_rows; r += (int64_t)gridDim.x * nwarps) {
        const int8_t* wrow = qs + r * k;
        const uint16_t* drow = dsc + r * (k >> 5);
        for (int j = 0; j < mb; j++) {
            float t[kRefMaxBlocksPerLane];
#pragma unroll
            for (int u = 0; u < kRefMaxBlocksPerLane; u++) {
                const int64_t b = lane + 32 * u;
                t[u] = 0.0f;
                if (b >= nb) continue;
                const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(wrow + b * 32));
                const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(wrow + b * 32 + 16));
                const float dw = fp16_bits_to_float(__ldg(drow + b));  // drow: k / 32 scales per row
                if (use_q8k) {
                    const Q8KSmem& xb = xq[j * nk + (b >> 3)];
                    const int* a4 = reinterpret_cast<const int*>(xb.qs + (b & 7) * 32);
                    const int wv[8] = {(int)w0.x, (int)w0.y, (int)w0.z, (int)w0.w,
                                       (int)w1.x, (int)w1.y, (int)w1.z, (int)w1.w};
                    int isum = 0;
#pragma unroll
                    for (int e = 0; e < 8; e++) isum = __dp4a(wv[e], a4[e], isum);
                    t[u] = __fmul_rn(__fmul_rn(dw, xb.d), (float)isum);
                } else {
                    const float* xv = xf + (int64_t)j * k + b * 32;
                    const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    float f[32];
#pragma unroll
                    for (int e = 0; e < 8; e++) i8x4_to_f32(wv[e], f + 4 * e);
                    float acc[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[i] = fmaf(f[i], xv[i], 0.0f);
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[i] = fmaf(f[16 + i], xv[16 + i], acc[i]);
                    t[u] = __fmul_rn(dw, hsum16_tree(acc));
                }
            }
            float sum = 0.0f;  // block order, as the reference's loop
            for (int64_t b = 0; b < nb; b++) {
                float tb = 0.0f;
#pragma unroll
                for (int u = 0; u < kRefMaxBlocksPerLane; u++)
                    if ((b >> 5) == u) tb = __shfl_sync(0xffffffffu, t[u], (int)(b & 31));
                sum = __fadd_rn(sum, tb);
            }
            if (lane == 0) y[(m0 + j) * ldy + r] = sum;
        }
    }
}

// ------------------------------------------------------------------- Q4_K

__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* sc, int& s, int& m) {
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

// One thread per (superblock, chunk c, 16-byte half): 32 weights out.
__global__ void q4_k_dequant_kernel(const uint8_t* __restrict__ blocks, float* __restrict__ out,
                                    int64_t nsb) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nsb * 8) return;
    const int64_t sb = t >> 3;
    const int c = (int)(t & 7) >> 1, half = (int)(t & 1);
    const uint8_t* blk = blocks + sb * 144;
    const float d = fp16_bits_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = fp16_bits_to_float((uint16_t)(blk[2] | (blk[3] << 8)));
    int s_lo, m_lo, s_hi, m_hi;
    q4k_scale_min(2 * c, blk + 4, s_lo, m_lo);
    q4k_scale_min(2 * c + 1, blk + 4, s_hi, m_hi);
    const float sl = __fmul_rn(d, (float)s_lo), ml = __fmul_rn(dmin, (float)m_lo);
    const float sh = __fmul_rn(d, (float)s_hi), mh = __fmul_rn(dmin, (float)m_hi);
    const uint4 q = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c + 16 * half);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    float* o_lo = out + sb * 256 + 64 * c + 16 * half;
    float* o_hi = o_lo + 32;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        float lo[4], hi[4];
        u4x4_to_f32(qw[j], lo);
        u4x4_to_f32(qw[j] >> 4, hi);
        reinterpret_cast<float4*>(o_lo)[j] =
            make_float4(__fsub_rn(__fmul_rn(sl, lo[0]), ml), __fsub_rn(__fmul_rn(sl, lo[1]), ml),
                        __fsub_rn(__fmul_rn(sl, lo[2]), ml), __fsub_rn(__fmul_rn(sl, lo[3]), ml));
        reinterpret_cast<float4*>(o_hi)[j] =
            make_float4(__fsub_rn(__fmul_rn(sh, hi[0]), mh), __fsub_rn(__fmul_rn(sh, hi[1]), mh),
                        __fsub_rn(__fmul_rn(sh, hi[2]), mh), __fsub_rn(__fmul_rn(sh, hi[3]), mh));
    }
}

// One thread per (superblock, chunk c, 16-byte half) of a Q5_K tensor (176-byte
// superblocks: d, dmin, 12 scale bytes, qh[32], qs[128]): 32 weights out, the
// nibble of qs[32c + j] with bit 2c (low) / 2c + 1 (high) of qh[j] as the fifth
// bit (engine/runtime/gpu_offload.cu:302-309), w = (d*sc)*q - (dmin*m) with
// each operation rounded once.
__global__ void q5_k_dequant_kernel(const uint8_t* __restrict__ blocks, float* __restrict__ out, int64_t nsb) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nsb * 8) return;
    const int64_t sb = t >> 3;
    const int c = (int)(t & 7) >> 1, half = (int)(t & 1);
    const uint8_t* blk = blocks + sb * 176;
    const float d = fp16_bits_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = fp16_bits_to_float((uint16_t)(blk[2] | (blk[3] << 8)));
    int s_lo, m_lo, s_hi, m_hi;
    q4k_scale_min(2 * c, blk + 4, s_lo, m_lo);
    q4k_scale_min(2 * c + 1, blk + 4, s_hi, m_hi);
    const float sl = __fmul_rn(d, (float)s_lo), ml = __fmul_rn(dmin, (float)m_lo);
    const float sh = __fmul_rn(d, (float)s_hi), mh = __fmul_rn(dmin, (float)m_hi);
    const uint8_t* qh = blk + 16 + 16 * half;
    const uint8_t* qs = blk + 48 + 32 * c + 16 * half;
    float* o_lo = out + sb * 256 + 64 * c + 16 * half;
    float* o_hi = o_lo + 32;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const int ql = (qs[j] & 0x0F) | (((qh[j] >> (2 * c)) & 1) << 4);
        const int qv = (qs[j] >> 4) | (((qh[j] >> (2 * c + 1)) & 1) << 4);
        o_lo[j] = __fsub_rn(__fmul_rn(sl, (float)ql), ml);
        o_hi[j] = __fsub_rn(__fmul_rn(sh, (float)qv), mh);
    }
}

// Q4_K GEMV (quant_matvec type 12 with fp32 activations; the reference GPU
// kernel is engine/runtime/gpu_offload.cu:237-250).  A sub-block's contribution
// is (d sc) sum(q x) - (dmin m) sum(x); the MB activation rows of block row
// blockIdx.y share every weight load.
template <int MB>
__global__ void __launch_bounds__(256) q4_k_gemv_kernel(const uint8_t* __restrict__ blocks,
                                                       int64_t n_rows, int64_t k, const void* x,
                                                       int x_dtype, int64_t m, float* __restrict__ y,
                                                       int64_t ldy, int rows_per_block) {
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int64_t nsb = k >> 8;
    // A warp walks one row's superblocks; lane l takes the 4 quant bytes
    // 32c + 4g .. +3 (c = l / 8, g = l % 8): low nibbles are weights 64c + 4g + e
    // (sub-block 2c), high nibbles weights 64c + 32 + 4g + e (sub-block 2c + 1).
    // The warp reads the 128 quant bytes as one line and each quarter-warp reads
    // 128 contiguous bytes of x.  w = (d sc) q - dmin m is summed as
    // (d sc) sum(q x) - (dmin m) sum(x) per lane.  Loads run one batch (four
    // superblocks) ahead: the first before the activations are staged, each next
    // one -- of this row or the warp's next -- before the current is reduced.
    const int c = lane >> 3, g = lane & 7;
    const int64_t row0 = (int64_t)blockIdx.x * rows_per_block;
    const int64_t row_end = min(row0 + rows_per_block, n_rows);
    uint4 hv[4];
    uint32_t qv[4];
    auto load = [&](int64_t r, int64_t sb0) {
        const uint8_t* row = blocks + r * nsb * 144;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            if (sb0 + u < nsb) {
                const uint8_t* blk = row + (sb0 + u) * 144;
                hv[u] = __ldg(reinterpret_cast<const uint4*>(blk));
                qv[u] = __ldg(reinterpret_cast<const uint32_t*>(blk + 16 + 32 * c + 4 * g));
            }
        }
    };
    int64_t r = row0 + warp, sb0 = 0;
    bool have = r < row_end;
    if (have) load(r, sb0);  // weights never come from an earlier kernel: before the wait
    pdl_wait();
    extern __shared__ float xs[];  // [mb][k]
    const int64_t m0 = (int64_t)blockIdx.y * MB;
    const int mb = (int)min((int64_t)MB, m - m0);
    stage_x(xs, x, x_dtype, m0, mb, k);
    __syncthreads();
    float acc[MB];
#pragma unroll
    for (int j = 0; j < MB; j++) acc[j] = 0.0f;
    while (have) {
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t sb = sb0 + u;
            if (sb >= nsb) break;
            const uint4 hdr = hv[u];
            const uint32_t qw = qv[u];
            const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hdr);
            const float d = fp16_bits_to_float((uint16_t)(hdr.x & 0xFFFFu));
            const float dmin = fp16_bits_to_float((uint16_t)(hdr.x >> 16));
            int s_lo, m_lo, s_hi, m_hi;
            q4k_scale_min(2 * c, hb + 4, s_lo, m_lo);
            q4k_scale_min(2 * c + 1, hb + 4, s_hi, m_hi);
            const float sl = d * (float)s_lo, ml = dmin * (float)m_lo;
            const float sh = d * (float)s_hi, mh = dmin * (float)m_hi;
            float lo[4], hi[4];
            u4x4_to_f32(qw, lo);
            u4x4_to_f32(qw >> 4, hi);
            const int64_t klo = sb * 256 + 64 * c + 4 * g;
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (j < mb) {
                    const float4 xl = *reinterpret_cast<const float4*>(xs + (int64_t)j * k + klo);
                    const float4 xh = *reinterpret_cast<const float4*>(xs + (int64_t)j * k + klo + 32);
                    const float al = fmaf(lo[3], xl.w, fmaf(lo[2], xl.z, fmaf(lo[1], xl.y, lo[0] * xl.x)));
                    const float ah = fmaf(hi[3], xh.w, fmaf(hi[2], xh.z, fmaf(hi[1], xh.y, hi[0] * xh.x)));
                    const float sxl = (xl.x + xl.y) + (xl.z + xl.w);
                    const float sxh = (xh.x + xh.y) + (xh.z + xh.w);
                    acc[j] += (sl * al - ml * sxl) + (sh * ah - mh * sxh);
                }
            }
        }
        const bool row_done = sb0 + 4 >= nsb;
        const int64_t nr = row_done ? r + nwarps : r, nsb0 = row_done ? 0 : sb0 + 4;
        const bool next = nr < row_end;
        if (next) load(nr, nsb0);
        if (row_done) {
#pragma unroll
            for (int j = 0; j < MB; j++) {
                if (j < mb) {
                    const float v = warp_sum(acc[j]);
                    if (lane == 0) y[(m0 + j) * ldy + r] = v;
                }
                acc[j] = 0.0f;
            }
        }
        r = nr;
        sb0 = nsb0;
        have = next;
    }
}

// -------------------------------------------------------------- launchers

static int smem_optin(const void* fn, size_t bytes) {
    if (bytes <= 48 * 1024) return GDN_OK;
    GDN_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return GDN_OK;
}

int launch_q8_0_repack(const void* blocks, int8_t* qs, uint16_t* d, int64_t rows, int64_t cols,
                       cudaStream_t s) {
    const int64_t nb = rows * (cols / 32);
    if (nb == 0) return GDN_OK;
    q8_0_repack_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(static_cast<const uint8_t*>(blocks), qs,
                                                                     d, nb);
    GDN_LAUNCH_CHECK("q8_0_repack_kernel");
    return GDN_OK;
}

int launch_q8_0_dequant(const int8_t* qs, const uint16_t* d, float* out, int64_t rows, int64_t cols,
                        cudaStream_t s) {
    const int64_t n16 = rows * cols / 16;
    if (n16 == 0) return GDN_OK;
    q8_0_dequant_kernel<<<(unsigned)((n16 + 255) / 256), 256, 0, s>>>(qs, d, out, n16);
    GDN_LAUNCH_CHECK("q8_0_dequant_kernel");
    return GDN_OK;
}

// Weight rows per block (a multiple of the 8 warps, at most 32): fewer when
// the grid would otherwise leave SMs idle (few weight rows, e.g. the gates).
static int rows_per_block(int64_t n, int64_t groups, int mb) {
    // one activation row per block: x staging is trivial, so aim for ~8 resident
    // blocks per SM (one weight row per warp in flight); with more rows, larger
    // blocks amortise the staging
    const int64_t want = (mb == 1 ? 8 : 2) * (int64_t)sm_count();
    int rpb = 32;
    while (rpb > 8 && ((n + rpb - 1) / rpb) * groups < want) rpb -= 8;
    return rpb;
}

// Activation rows per block (a template size: 1, 2, 4 or 8): the smallest one
// that covers min(m, 8) rows, halved while the staged rows overflow shared memory.
static int pick_mb(int64_t m, int64_t floats_per_row) {
    int mb = m >= 5 ? 8 : m >= 3 ? 4 : m >= 2 ? 2 : 1;
    while (mb > 1 && (size_t)mb * floats_per_row * 4 > 200 * 1024) mb >>= 1;
    return mb;
}

template <int MB>
static int run_q8_gemv(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* x, int dt,
                       int64_t m, float* y, int64_t ldy, cudaStream_t s) {
    const size_t smem = (size_t)MB * (k + k / 4) * sizeof(float);
    int st = smem_optin((const void*)q8_0_gemv_kernel<MB>, smem);
    if (st) return st;
    const int rpb = rows_per_block(n, (m + MB - 1) / MB, MB);
    const dim3 grid((unsigned)((n + rpb - 1) / rpb), (unsigned)((m + MB - 1) / MB));
    return launch_pdl("q8_0_gemv_kernel", q8_0_gemv_kernel<MB>, grid, dim3(256), smem, s, qs, d, n, k, x, dt, m, y,
                      ldy, rpb);
}

int launch_q8_0_gemv(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* x, int dt,
                     int64_t m, float* y, int64_t ldy, cudaStream_t s) {
    if ((size_t)(k + k / 4) * 4 > 200 * 1024) return fail(GDN_ERR_SHAPE, "q8_0 gemv: k=%lld too large", (long long)k);
    if (m <= 0 || n <= 0) return GDN_OK;
    if ((m + 7) / 8 > 65535) return fail(GDN_ERR_SHAPE, "q8_0 gemv: m=%lld too large", (long long)m);
    if (gemv_stream_fits(0, qs, d, k, m)) return launch_gemv_stream(0, qs, d, n, k, x, dt, m, y, ldy, s);
    switch (pick_mb(m, k + k / 4)) {
        case 1: return run_q8_gemv<1>(qs, d, n, k, x, dt, m, y, ldy, s);
        case 2: return run_q8_gemv<2>(qs, d, n, k, x, dt, m, y, ldy, s);
        case 4: return run_q8_gemv<4>(qs, d, n, k, x, dt, m, y, ldy, s);
        default: return run_q8_gemv<8>(qs, d, n, k, x, dt, m, y, ldy, s);
    }
}

int launch_quantize_q8_K(const float* x, void* out, int64_t n, cudaStream_t s) {
    if (n % 256 != 0) return fail(GDN_ERR_SHAPE, "quantize_q8_K: the length must be a multiple of 256");
    const int64_t nb = n / 256;
    if (nb == 0) return GDN_OK;
    return launch_pdl("quantize_q8_K_kernel", quantize_q8_K_kernel, dim3((unsigned)((nb + 7) / 8)), dim3(256), 0, s,
                      x, static_cast<uint8_t*>(out), nb);
}

template <int MB>
static int run_q8_gemv_ref(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const float* x, int64_t m,
                           float* y, int64_t ldy, bool q8k, cudaStream_t s) {
    const size_t smem = q8k ? (size_t)MB * (k / 256) * sizeof(Q8KSmem) : (size_t)MB * k * sizeof(float);
    int st = smem_optin((const void*)q8_0_gemv_ref_kernel<MB>, smem);
    if (st) return st;
    const int64_t blocks_x = std::min<int64_t>((n + 7) / 8, (int64_t)sm_count() * 4);
    const dim3 grid((unsigned)blocks_x, (unsigned)((m + MB - 1) / MB));
    return launch_pdl("q8_0_gemv_ref_kernel", q8_0_gemv_ref_kernel<MB>, grid, dim3(256), smem, s, qs, d, n, k, x, m,
                      y, ldy, q8k ? 1 : 0);
}

int launch_q8_0_gemv_ref(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const float* x, int64_t m,
                         float* y, int64_t ldy, cudaStream_t s) {
    if (k % 32 != 0 || k <= 0 || k / 32 > 32 * kRefMaxBlocksPerLane)
        return fail(GDN_ERR_SHAPE, "reference-exact q8_0 gemv: k=%lld must be a multiple of 32 up to 8192",
                    (long long)k);
    if (m <= 0 || n <= 0) return GDN_OK;
    if ((m + 7) / 8 > 65535) return fail(GDN_ERR_SHAPE, "reference-exact q8_0 gemv: m too large");
    const bool q8k = k >= 256 && n >= 128;  // q8_matvec's Q8_K branch (q8_dequant.h:75-79)
    if (!q8k && (size_t)8 * k * 4 > 200 * 1024) return run_q8_gemv_ref<1>(qs, d, n, k, x, m, y, ldy, q8k, s);
    return m >= 8 ? run_q8_gemv_ref<8>(qs, d, n, k, x, m, y, ldy, q8k, s)
                  : run_q8_gemv_ref<1>(qs, d, n, k, x, m, y, ldy, q8k, s);
}

int launch_q4_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, cudaStream_t s) {
    const int64_t nsb = rows * cols / 256;
    if (nsb == 0) return GDN_OK;
    q4_k_dequant_kernel<<<(unsigned)((nsb * 8 + 255) / 256), 256, 0, s>>>(static_cast<const uint8_t*>(blocks),
                                                                         out, nsb);
    GDN_LAUNCH_CHECK("q4_k_dequant_kernel");
    return GDN_OK;
}

template <int MB>
static int run_q4_gemv(const void* w, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
                       int64_t ldy, cudaStream_t s) {
    const size_t smem = (size_t)MB * k * sizeof(float);
    int st = smem_optin((const void*)q4_k_gemv_kernel<MB>, smem);
    if (st) return st;
    const int rpb = rows_per_block(n, (m + MB - 1) / MB, MB);
    const dim3 grid((unsigned)((n + rpb - 1) / rpb), (unsigned)((m + MB - 1) / MB));
    return launch_pdl("q4_k_gemv_kernel", q4_k_gemv_kernel<MB>, grid, dim3(256), smem, s,
                      static_cast<const uint8_t*>(w), n, k, x, dt, m, y, ldy, rpb);
}

int launch_q5_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, cudaStream_t s) {
    const int64_t nsb = rows * (cols / 256);
    if (nsb == 0) return GDN_OK;
    q5_k_dequant_kernel<<<(unsigned)((nsb * 8 + 255) / 256), 256, 0, s>>>(static_cast<const uint8_t*>(blocks), out,
                                                                        nsb);
    GDN_LAUNCH_CHECK("q5_k_dequant_kernel");
    return GDN_OK;
}

// Q5_K GEMV: the streamed kernels only (there is no row-per-warp Q5_K GEMV).
int launch_q5_k_gemv(const void* w, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y, int64_t ldy,
                     cudaStream_t s) {
    if (m <= 0 || n <= 0) return GDN_OK;
    if (!gemv_stream_fits(2, w, nullptr, k, m))
        return fail(GDN_ERR_SHAPE, "q5_k gemv: k=%lld must be a multiple of 256 (16-byte aligned blocks)",
                    (long long)k);
    return launch_gemv_stream(2, w, nullptr, n, k, x, dt, m, y, ldy, s);
}

int launch_q4_k_gemv(const void* w, int64_t n, int64_t k, const void* x, int dt, int64_t m, float* y,
                     int64_t ldy, cudaStream_t s) {
    if ((size_t)k * 4 > 200 * 1024) return fail(GDN_ERR_SHAPE, "q4_k gemv: k=%lld too large", (long long)k);
    if (m <= 0 || n <= 0) return GDN_OK;
    if ((m + 7) / 8 > 65535) return fail(GDN_ERR_SHAPE, "q4_k gemv: m=%lld too large", (long long)m);
    if (gemv_stream_fits(1, w, nullptr, k, m)) return launch_gemv_stream(1, w, nullptr, n, k, x, dt, m, y, ldy, s);
    switch (pick_mb(m, k)) {
        case 1: return run_q4_gemv<1>(w, n, k, x, dt, m, y, ldy, s);
        case 2: return run_q4_gemv<2>(w, n, k, x, dt, m, y, ldy, s);
        case 4: return run_q4_gemv<4>(w, n, k, x, dt, m, y, ldy, s);
        default: return run_q4_gemv<8>(w, n, k, x, dt, m, y, ldy, s);
    }
}

}  // namespace gdn
