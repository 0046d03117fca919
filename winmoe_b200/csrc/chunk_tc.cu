// The chunked WY recurrence on the 5th-generation tensor cores (tcgen05, TMEM).
//
// Per value head h and chunk c of C = 64 tokens (prefill.cu derives W', U',
// E = diag(e) K and the decays; the reference's sequential recurrence these
// reproduce is engine/runtime/deltanet_impl.h:279-348):
//   D_c     = U'_c - W'_c S_c                       (the chunk's deltas)
//   S_{c+1} = gam_c S_c + E_c^T D_c                 (the state carry)
//   O_c     = scale (diag(gam) Q_c S_c + P_c D_c)   (outputs; P the decayed, masked Q K^T)
// Both kernels work in the transposed form, with the value index v as the MMA's
// M = 128 (a full tile):
//   D^T = U'^T - S^T W'^T,   S^T <- gam S^T + D^T E,   O^T = S^T Q^T (x gam) + D^T P^T.
// Every operand is then K-major: S^T [v][k], W' [t][k], D^T [v][t], E^T [k][t],
// Q [t][k], P [t][t'].  They travel as "images" (img_off: the 128-byte-swizzle
// UMMA layout), written by their producer so that a consumer fetches each with
// one bulk copy into 1024-byte aligned shared memory.
//
//  chunk_scan_tc_kernel: one CTA per head, sequential over the chunks.  S^T
//    lives in TMEM as fp32 (128 lanes = v, 128 columns = k) for the whole
//    prompt; per chunk the CTA reads it once (bf16 copy -> the A operand of
//    MMA1 and the chunk's start-state image for chunk_out; gam * S^T back to
//    TMEM), MMA1 puts S^T W'^T into a second TMEM accumulator, the threads form
//    D^T = U'^T - that (bf16 image: MMA2's A operand and chunk_out's), and MMA2
//    accumulates D^T E onto gam S^T.  The images of the next chunks stream in
//    behind (a three-deep ring of bulk copies).
//  chunk_out_tc_kernel: one CTA per (chunk, head).  P = mask(exp(G_i - G_j)
//    q_i . k_j) on mma.sync (64 x 64, in registers, then into its image); the
//    two products on tcgen05 into two TMEM accumulators; the epilogue (one
//    thread per v) applies gam, the scale, the per-token RMSNorm over v (a
//    warp transpose-reduction plus four warp partials), the norm weight and the
//    SiLU(z) gate (deltanet_impl.h:350-371) and stores the fp16 out_proj operand.
#include "gdn_common.cuh"
#include "ptx_sm100.cuh"
#include "warp_mma.cuh"
#include "chunk_tc.cuh"

namespace gdn {

using namespace sm100;
using wmma16::bf16;

namespace {

constexpr int HD = 128;
constexpr int CH = 64;
constexpr uint32_t kImgWBytes = CH * HD * 2;   // [64][128] images: W', Q, K
constexpr uint32_t kImgEBytes = HD * CH * 2;   // [128][64] images: E^T, U'^T, D^T
constexpr uint32_t kImgSBytes = HD * HD * 2;   // [128][128] image: S^T

__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return wmma16::pack_bf16(lo, hi); }

// ------------------------------------------------------------------ scan

// The per-chunk images stream through a kRing-deep ring, requested kRing - 1
// chunks ahead of their use.
constexpr int kRing = 3;
constexpr int kScanChunksInSmem = 1024;  // chunk decays staged in shared memory (T up to 64K)

// A head's value rows are split over two CTAs (kVRows = 64 each, M = 64 MMA
// tiles): the images a CTA moves per chunk are its halves of U'^T, S^T and D^T
// plus the full W' and E^T -- 64 KB instead of 96 KB through one SM, which is
// what bounds a chunk step -- and the chain of steps runs on twice the SMs.
constexpr int kVRows = 64;
constexpr uint32_t kHalfUBytes = kVRows * CH * 2;  // U'^T / D^T rows of one CTA: [64 v][64 t]
constexpr uint32_t kHalfSBytes = kVRows * HD * 2;  // S^T rows of one CTA: [64 v][128 k] (two K blocks of 8 KB)

struct ScanTcSmem {
    uint8_t w[kRing][kImgWBytes];   // W' images [64 t][128 k]        (B of MMA1)
    uint8_t e[kRing][kImgEBytes];   // E^T images [128 k][64 t]       (B of MMA2)
    uint8_t u[kRing][kHalfUBytes];  // this CTA's U'^T rows [64 v][64 t]
    uint8_t s[kHalfSBytes];         // S^T rows [64 v][128 k]         (A of MMA1; the chunk's start state)
    uint8_t d[kHalfUBytes];         // D^T rows [64 v][64 t]          (A of MMA2; the chunk's deltas)
    float gc[kScanChunksInSmem];
    uint64_t full[kRing];          // a chunk's three images landed
    uint64_t mma_d, mma_s;         // MMA1 / MMA2 of a chunk completed
    uint64_t s_half[2], d_half[2]; // a column half of the S^T / D^T image written (128 arrivals)
    uint64_t s_free, d_free;       // the previous S^T / D^T image's bulk store has read it
    uint64_t drain;
    uint32_t tmem_slot;
};
static_assert(offsetof(ScanTcSmem, e) % 1024 == 0 && offsetof(ScanTcSmem, u) % 1024 == 0 &&
              offsetof(ScanTcSmem, s) % 1024 == 0 && offsetof(ScanTcSmem, d) % 1024 == 0, "images 1024-aligned");

constexpr uint32_t kScanTmemCols = 256;  // S^T: columns 0..127; D^T: 128..191
constexpr int kScanThreads = 256;

// One CTA per (head, half of the value rows); 256 threads.  With M = 64 the
// accumulator row i (local value row) sits in TMEM lane 32 (i / 16) + i % 16:
// lanes 0..15 of each warp carry a row, lanes 16..31 only take part in the
// warp-wide TMEM instructions.  Warps w and w + 4 share TMEM lanes
// 32 (w % 4) .. and split the columns into halves: warps 0..3 take S^T columns
// 0..63 (the image's first K block) and D^T columns 0..31, warps 4..7 the rest.
// No block barrier sits on the chain of a chunk: each half announces its part
// of an image on an mbarrier, and thread 0 issues the MMAs of that K block as
// soon as it is complete (MMA1 per K block of S^T, MMA2 per half of the
// chunk's tokens).  Thread 32 moves the images: the requests kRing - 1 chunks
// ahead, and the bulk stores of each chunk's start state and deltas (their
// completions -- "the image may be rewritten" -- on s_free / d_free).
__global__ void __launch_bounds__(kScanThreads, 1) chunk_scan_tc_kernel(const uint8_t* __restrict__ wimg,
                                                                        const uint8_t* __restrict__ eimg,
                                                                        const uint8_t* __restrict__ uimg,
                                                                        const float* __restrict__ gchunk,
                                                                        float* __restrict__ S,
                                                                        uint8_t* __restrict__ simg,
                                                                        uint8_t* __restrict__ dimg, int64_t nc,
                                                                        uint32_t* __restrict__ err) {
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    ScanTcSmem& sm = *reinterpret_cast<ScanTcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int h = blockIdx.x >> 1, vh = blockIdx.x & 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, half = warp >> 2;
    const bool row_lane = lane < 16;               // this lane holds a row of the M = 64 tiles
    const int vr = 16 * quad + (lane & 15);        // the local value row (image row)
    const int v = kVRows * vh + vr;                // ... its value column of S
    const bool issuer = tid == 0, copier = tid == 32;

    if (warp == 0) {
        tmem_alloc(smem_u32(&sm.tmem_slot), kScanTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < kRing; i++) mbar_init(smem_u32(&sm.full[i]), 1);
        mbar_init(smem_u32(&sm.mma_d), 1);
        mbar_init(smem_u32(&sm.mma_s), 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&sm.s_half[i]), kScanThreads / 2);
            mbar_init(smem_u32(&sm.d_half[i]), kScanThreads / 2);
        }
        mbar_init(smem_u32(&sm.s_free), 1);
        mbar_init(smem_u32(&sm.d_free), 1);
        mbar_init(smem_u32(&sm.drain), 1);
        fence_barrier_init();
    }
    pdl_wait();  // W', E, U' and the decays come from chunk_local
    const bool gc_smem = nc <= kScanChunksInSmem;
    if (gc_smem)
        for (int64_t i = tid; i < nc; i += kScanThreads) sm.gc[i] = gchunk[(int64_t)h * nc + i];
    auto prefetch = [&](int64_t c) {
        const int buf = (int)(c % kRing);
        const uint32_t bar = smem_u32(&sm.full[buf]);
        const int64_t i = (int64_t)h * nc + c;
        mbar_arrive_expect_tx(bar, kImgWBytes + kImgEBytes + kHalfUBytes);
        bulk_load(smem_u32(sm.w[buf]), wimg + i * kImgWBytes, kImgWBytes, bar);
        bulk_load(smem_u32(sm.e[buf]), eimg + i * kImgEBytes, kImgEBytes, bar);
        // rows 64 vh .. of the [128 v][64 t] image: one contiguous 8 KB (same swizzle phase)
        bulk_load(smem_u32(sm.u[buf]), uimg + i * kImgEBytes + vh * kHalfUBytes, kHalfUBytes, bar);
    };
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    int64_t last_pref = -1;  // copier: the last chunk whose images were requested
    if (copier)
        for (int64_t j = 0; j < kRing - 1 && j < nc; j++) {
            prefetch(j);
            last_pref = j;
        }
    const uint32_t tmem = sm.tmem_slot;
    const uint32_t tS = tmem + ((uint32_t)(quad * 32) << 16) + 64 * half;        // this thread's S^T columns
    const uint32_t tD = tmem + ((uint32_t)(quad * 32) << 16) + 128 + 32 * half;  // ... D^T columns

    // S_0 -> TMEM: lane v holds row v of S^T = column v of S (coalesced over the warp)
    float* Sh = S + (int64_t)h * HD * HD;
    {
        uint32_t r[64];
#pragma unroll
        for (int i = 0; i < 64; i++) r[i] = row_lane ? __float_as_uint(Sh[(int64_t)(64 * half + i) * HD + v]) : 0u;
        tmem_store_32x32b_x64(tS, r);
    }

    constexpr uint32_t idesc1 = umma_idesc_f16(kVRows, 64, true);   // D^T = S^T W'^T
    constexpr uint32_t idesc2 = umma_idesc_f16(kVRows, 128, true);  // S^T += D^T E
    bool ok = true;
    int64_t c = 0;
    for (; c < nc && ok; c++) {
        const int buf = (int)(c % kRing);
        const uint32_t fpar = (uint32_t)((c / kRing) & 1), par = (uint32_t)(c & 1), ppar = par ^ 1u;
        // (a) S_c complete in TMEM (MMA2 of the previous chunk) and the S^T image free
        if (c > 0) {
            ok = mbar_wait(smem_u32(&sm.mma_s), ppar, err) && ok;
            ok = mbar_wait(smem_u32(&sm.s_free), ppar, err) && ok;
        }
        tc_fence_after();
        // (b) bf16 copy of this half of S_c^T into the image, gam_c S_c^T back to TMEM
        const float gam = gc_smem ? sm.gc[c] : gchunk[(int64_t)h * nc + c];
        {
            uint32_t r[64];
            tmem_load_32x32b_x64(tS, r);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const uint4 pk = make_uint4(
                    pack2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1])),
                    pack2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3])),
                    pack2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5])),
                    pack2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7])));
                if (row_lane) *reinterpret_cast<uint4*>(sm.s + img_off(kVRows, vr, 64 * half + 8 * q)) = pk;
            }
#pragma unroll
            for (int i = 0; i < 64; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * gam);
            tmem_store_32x32b_x64(tS, r);
        }
        fence_proxy_async_smem();  // the image is read by MMA1 and a bulk store (async proxy)
        tc_fence_before();
        mbar_arrive(smem_u32(&sm.s_half[half]));
        // (c) MMA1 D^T = S^T W'^T, one K block as soon as its half of the image is written
        if (issuer) {
            ok = mbar_wait(smem_u32(&sm.full[buf]), fpar, err) && ok;
            const uint32_t a0 = smem_u32(sm.s), b0 = smem_u32(sm.w[buf]);
#pragma unroll
            for (int kb = 0; kb < 2; kb++) {
                ok = mbar_wait(smem_u32(&sm.s_half[kb]), par, err) && ok;
                tc_fence_after();
                if (ok) {
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_f16_ss(tmem + 128, umma_desc_sw128(a0 + kb * (kVRows * 128) + ks * 32),
                                   umma_desc_sw128(b0 + kb * (CH * 128) + ks * 32), idesc1, (kb | ks) != 0);
                }
            }
            mma_commit(smem_u32(&sm.mma_d));
        } else if (copier) {
            // the chunk's start state leaves; the previous deltas' store has read its image
            ok = mbar_wait(smem_u32(&sm.s_half[0]), par, err) && ok;
            ok = mbar_wait(smem_u32(&sm.s_half[1]), par, err) && ok;
            if (ok) {  // this CTA's rows of each K block of the [128 v][128 k] image
                uint8_t* dst = simg + ((int64_t)h * nc + c) * kImgSBytes + vh * (kHalfSBytes / 2);
                bulk_store(dst, smem_u32(sm.s), kHalfSBytes / 2);
                bulk_store(dst + kImgSBytes / 2, smem_u32(sm.s) + kHalfSBytes / 2, kHalfSBytes / 2);
                bulk_commit();
            }
            bulk_wait_read<1>();
            mbar_arrive(smem_u32(&sm.d_free));
            // chunk c - 1's buffer is free: its MMAs completed before MMA2(c - 1)'s
            // commit, its U'^T reads before d_half(c - 1)
            if (c + kRing - 1 < nc) {
                prefetch(c + kRing - 1);
                last_pref = c + kRing - 1;
            }
        }
        // (e) D^T = U'^T - S^T W'^T for this half's tokens of row v -> the D^T image
        ok = mbar_wait(smem_u32(&sm.full[buf]), fpar, err) && ok;
        ok = mbar_wait(smem_u32(&sm.mma_d), par, err) && ok;
        ok = mbar_wait(smem_u32(&sm.d_free), par, err) && ok;
        tc_fence_after();
        {
            uint32_t r[32];
            tmem_load_32x32b_x32(tD, r);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int t8 = 32 * half + 8 * q;
                const uint4 u4 = *reinterpret_cast<const uint4*>(sm.u[buf] + img_off(kVRows, vr, t8));
                const uint32_t uw[4] = {u4.x, u4.y, u4.z, u4.w};
                uint32_t dw[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 uf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&uw[i]));
                    dw[i] = pack2(uf.x - __uint_as_float(r[8 * q + 2 * i]), uf.y - __uint_as_float(r[8 * q + 2 * i + 1]));
                }
                if (row_lane) *reinterpret_cast<uint4*>(sm.d + img_off(kVRows, vr, t8)) = make_uint4(dw[0], dw[1], dw[2], dw[3]);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(smem_u32(&sm.d_half[half]));
        // (g) MMA2 S^T += D^T E, two K steps per half of the chunk's tokens
        if (issuer) {
            const uint32_t a0 = smem_u32(sm.d), b0 = smem_u32(sm.e[buf]);
#pragma unroll
            for (int th = 0; th < 2; th++) {
                ok = mbar_wait(smem_u32(&sm.d_half[th]), par, err) && ok;
                tc_fence_after();
                if (ok) {
#pragma unroll
                    for (int ks = 2 * th; ks < 2 * th + 2; ks++)
                        mma_f16_ss(tmem, umma_desc_sw128(a0 + ks * 32), umma_desc_sw128(b0 + ks * 32), idesc2, 1u);
                }
            }
            mma_commit(smem_u32(&sm.mma_s));
        } else if (copier) {
            // the deltas leave; the start state's store has read its image
            ok = mbar_wait(smem_u32(&sm.d_half[0]), par, err) && ok;
            ok = mbar_wait(smem_u32(&sm.d_half[1]), par, err) && ok;
            if (ok) {
                bulk_store(dimg + ((int64_t)h * nc + c) * kImgEBytes + vh * kHalfUBytes, smem_u32(sm.d), kHalfUBytes);
                bulk_commit();
            }
            bulk_wait_read<1>();
            mbar_arrive(smem_u32(&sm.s_free));
        }
    }
    // every thread leaves the loop here (a timed-out wait ends the CTA's loop; the
    // waits of the others on its arrivals then time out too)
    const bool all_ok = __syncthreads_and(ok && c == nc);
    if (all_ok) {
        // the state after the prompt: S[k][v] = lane v, column k
        const bool okf = mbar_wait(smem_u32(&sm.mma_s), (uint32_t)((nc - 1) & 1), err);
        tc_fence_after();
        if (okf) {
            uint32_t r[64];
            tmem_load_32x32b_x64(tS, r);
            if (row_lane)
#pragma unroll
                for (int i = 0; i < 64; i++) Sh[(int64_t)(64 * half + i) * HD + v] = __uint_as_float(r[i]);
        }
    } else if (issuer) {
        // the error word is set: let the MMAs already issued finish (bounded)
        mma_commit(smem_u32(&sm.drain));
        mbar_wait(smem_u32(&sm.drain), 0, err);
    } else if (copier) {
        // ... and the image requests still in flight
        for (int64_t j = last_pref; j >= 0 && j > last_pref - kRing; j--)
            mbar_wait(smem_u32(&sm.full[j % kRing]), (uint32_t)((j / kRing) & 1), err);
    }
    if (copier) bulk_wait_read_all();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, kScanTmemCols);
}

// ------------------------------------------------------------------ output

struct OutTcSmem {
    uint8_t s[kImgSBytes];   // S_c^T image [128 v][128 k]   (A of the first product)
    uint8_t q[kImgWBytes];   // Q image [64 t][128 k]        (B of the first product; A of Q K^T)
    uint8_t kd[kImgWBytes];  // K image [64 t][128 k] for Q K^T, then the D_c^T image [128 v][64 t]
    uint8_t p[CH * CH * 2];  // P image [64 t][64 t']        (B of the second product)
    float G[CH], gam[CH], hn[HD];
    uint64_t ld_s, ld_d, mma;
    uint32_t tmem_slot;
};
// The epilogue's per-token partial sums live in the S^T image, dead by then.
struct OutTcRed {
    float red[4][CH];
    float inv[CH];
};
static_assert(offsetof(OutTcSmem, q) % 1024 == 0 && offsetof(OutTcSmem, kd) % 1024 == 0 &&
              offsetof(OutTcSmem, p) % 1024 == 0, "images 1024-aligned");

constexpr uint32_t kOutTmemCols = 128;  // S^T Q^T: columns 0..63; D^T P^T: 64..127

// Sums over the warp's 32 lanes of 32 per-lane values: after five halving
// exchanges lane l holds the sum of value l.
__device__ __forceinline__ float warp_token_sums(const float (&x)[32], int lane) {
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const bool hi = lane & 16;
        const float keep = hi ? x[16 + i] : x[i], send = hi ? x[i] : x[16 + i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float b[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const bool hi = lane & 8;
        const float keep = hi ? a[8 + i] : a[i], send = hi ? a[i] : a[8 + i];
        b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float c4[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const bool hi = lane & 4;
        const float keep = hi ? b[4 + i] : b[i], send = hi ? b[i] : b[4 + i];
        c4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    float d2[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const bool hi = lane & 2;
        const float keep = hi ? c4[2 + i] : c4[i], send = hi ? c4[i] : c4[2 + i];
        d2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    const bool hi = lane & 1;
    const float keep = hi ? d2[1] : d2[0], send = hi ? d2[0] : d2[1];
    return keep + __shfl_xor_sync(0xffffffffu, send, 1);
}

// Three CTAs per SM (72 KB of shared memory each): the D^T image reuses the K
// image's buffer once P is formed, and the z inputs arrive in two halves (the
// first during the products, the second during the epilogue's reduction).
// (All loads issued at once with two CTAs per SM measured slower: 135 against
// 103 us at T = 4096.)  The epilogue loops over the two 32-token halves without
// unrolling: one copy of its body keeps the kernel's code small enough for the
// instruction cache (fully unrolled, instruction fetch stalls dominated).
__global__ void __launch_bounds__(128, 3) chunk_out_tc_kernel(const bf16* __restrict__ qn, const bf16* __restrict__ kn,
                                                              const uint8_t* __restrict__ simg,
                                                              const uint8_t* __restrict__ dimg,
                                                              const float* __restrict__ gcum,
                                                              const float* __restrict__ proj, int64_t ldp,
                                                              const float* __restrict__ head_norm,
                                                              __half* __restrict__ gated, const RowDest dst, int64_t T,
                                                              int64_t Tp, int hk, int hv, int qkv, int head_map,
                                                              uint32_t* __restrict__ err) {
    pdl_trigger();
    extern __shared__ uint8_t smem_raw[];
    OutTcSmem& sm = *reinterpret_cast<OutTcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int c = blockIdx.x, h = blockIdx.y;
    const int g = head_map ? (h % hk) : (h / (hv / hk));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, qq = lane & 3;
    const int64_t t0 = (int64_t)c * CH;
    const int64_t nc = Tp / CH;
    const int v = tid;

    if (warp == 0) {
        tmem_alloc(smem_u32(&sm.tmem_slot), kOutTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(smem_u32(&sm.ld_s), 1);
        mbar_init(smem_u32(&sm.ld_d), 1);
        mbar_init(smem_u32(&sm.mma), 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_wait();  // S^T and D^T images come from chunk_scan
    if (tid == 0) {
        mbar_arrive_expect_tx(smem_u32(&sm.ld_s), kImgSBytes);
        bulk_load(smem_u32(sm.s), simg + ((int64_t)h * nc + c) * kImgSBytes, kImgSBytes, smem_u32(&sm.ld_s));
    }
    {  // Q and K rows [t][128] -> their images (16-byte chunks to their swizzled places)
        const bf16* qc = qn + ((int64_t)g * Tp + t0) * HD;
        const bf16* kc = kn + ((int64_t)g * Tp + t0) * HD;
        for (int i = tid; i < CH * HD / 8; i += 128) {
            const int r = i >> 4, j = i & 15;
            wmma16::cp_async16(sm.q + img_off(CH, r, 8 * j), qc + r * HD + 8 * j);
            wmma16::cp_async16(sm.kd + img_off(CH, r, 8 * j), kc + r * HD + 8 * j);
        }
        wmma16::cp_async_commit();
    }
    if (tid < CH) {
        const float G = gcum[(int64_t)h * Tp + t0 + tid];
        sm.G[tid] = G;
        sm.gam[tid] = expf(G);
    }
    sm.hn[tid] = head_norm != nullptr ? head_norm[tid] : 1.0f;
    wmma16::cp_async_wait<0>();
    __syncthreads();

    // ---- P = mask(exp(G_i - G_j) Q K^T): warp w token rows 16w .. 16w+15, all 64 columns
    {
        float pacc[CH / 8][4] = {};
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            uint32_t a[4];
            {
                const int r = 16 * warp + (lane & 15), col = 16 * kk + ((lane >> 4) << 3);
                wmma16::ldsm_x4(a, sm.q + img_off(CH, r, col));
            }
#pragma unroll
            for (int np2 = 0; np2 < CH / 16; np2++) {
                uint32_t b[4];
                const int j = lane >> 3;
                const int n = 16 * np2 + (lane & 7) + ((j >> 1) << 3), col = 16 * kk + ((j & 1) << 3);
                wmma16::ldsm_x4(b, sm.kd + img_off(CH, n, col));
                wmma16::mma(pacc[2 * np2], a, b[0], b[1]);
                wmma16::mma(pacc[2 * np2 + 1], a, b[2], b[3]);
            }
        }
        const int rA = 16 * warp + gq, rB = rA + 8;
#pragma unroll
        for (int n = 0; n < CH / 8; n++) {
            const int j = 8 * n + 2 * qq;
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int i = (e >> 1) ? rB : rA, jj = j + (e & 1);
                pv[e] = (jj <= i) ? __expf(sm.G[i] - sm.G[jj]) * pacc[n][e] : 0.0f;
            }
            *reinterpret_cast<uint32_t*>(sm.p + img_off(CH, rA, j)) = pack2(pv[0], pv[1]);
            *reinterpret_cast<uint32_t*>(sm.p + img_off(CH, rB, j)) = pack2(pv[2], pv[3]);
        }
    }
    // The gate inputs z of this thread's column for tokens 0..31, loaded now so
    // that they are in flight during the products (tokens 32..63 follow during
    // the epilogue's reduction).
    const float* zcol = proj + qkv + (int64_t)h * HD + v;
    float z0[32];
#pragma unroll
    for (int i = 0; i < 32; i++) z0[i] = (t0 + i < T) ? zcol[(t0 + i) * ldp] : 0.0f;
    fence_proxy_async_smem();  // P and Q (generic writes) are read by the MMAs; K's buffer is refilled
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_slot;
    bool ok = true;  // thread 0: both images landed
    if (warp == 0) {  // lane 0 issues; the warp waits for it (no lane spins beside it)
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(128, 64, true);
            mbar_arrive_expect_tx(smem_u32(&sm.ld_d), kImgEBytes);
            bulk_load(smem_u32(sm.kd), dimg + ((int64_t)h * nc + c) * kImgEBytes, kImgEBytes, smem_u32(&sm.ld_d));
            ok = mbar_wait(smem_u32(&sm.ld_s), 0, err);
            if (ok) {
                const uint32_t a0 = smem_u32(sm.s), b0 = smem_u32(sm.q);
#pragma unroll
                for (int kb = 0; kb < 2; kb++)
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_f16_ss(tmem, umma_desc_sw128(a0 + kb * (HD * 128) + ks * 32),
                                   umma_desc_sw128(b0 + kb * (CH * 128) + ks * 32), idesc, (kb | ks) != 0);
                ok = mbar_wait(smem_u32(&sm.ld_d), 0, err);
                if (ok) {
                    const uint32_t a1 = smem_u32(sm.kd), b1 = smem_u32(sm.p);
#pragma unroll
                    for (int ks = 0; ks < 4; ks++)
                        mma_f16_ss(tmem + 64, umma_desc_sw128(a1 + ks * 32), umma_desc_sw128(b1 + ks * 32), idesc,
                                   ks != 0);
                }
            }
            mma_commit(smem_u32(&sm.mma));  // arrives once every MMA issued above has completed
        }
        __syncwarp();
    }
    ok = mbar_wait(smem_u32(&sm.mma), 0, err) && ok;
    tc_fence_after();
    ok = __syncthreads_and(ok);
    OutTcRed& rd = *reinterpret_cast<OutTcRed*>(sm.s);

    // ---- epilogue: o[t] = scale (gam_t acc1 + acc2) for this thread's value column v,
    // read from TMEM twice: for the per-token sums of squares, then for the outputs
    const float scale = 1.0f / sqrtf((float)HD);
    const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int half = 0; half < 2; half++) {
        uint32_t a1[32], a2[32];
        tmem_load_32x32b_x32(tl + 32 * half, a1);
        tmem_load_32x32b_x32(tl + 64 + 32 * half, a2);
        float sq[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const float o = scale * fmaf(sm.gam[32 * half + i], __uint_as_float(a1[i]), __uint_as_float(a2[i]));
            sq[i] = o * o;
        }
        rd.red[warp][32 * half + lane] = warp_token_sums(sq, lane);
    }
    float z1[32];
#pragma unroll
    for (int i = 0; i < 32; i++) z1[i] = (t0 + 32 + i < T) ? zcol[(t0 + 32 + i) * ldp] : 0.0f;
    __syncthreads();
    if (tid < CH) {
        const float ss = (rd.red[0][tid] + rd.red[1][tid]) + (rd.red[2][tid] + rd.red[3][tid]);
        rd.inv[tid] = 1.0f / sqrtf(ss / (float)HD + 1e-6f);
    }
    __syncthreads();
    if (ok) {
        const float hnv = head_norm != nullptr ? sm.hn[v] : 1.0f;
        // this chunk's output rows: base + t * pitch when they lie in one buffer
        // (always with `gated`; with `dst`, unless the chunk straddles two slices)
        __half* base = nullptr;
        int64_t pitch = 0;
        if (gated != nullptr) {
            base = gated + t0 * (int64_t)hv * HD + h * HD + v;
            pitch = (int64_t)hv * HD;
        } else if (t0 / dst.rows == min(t0 + CH - 1, T - 1) / dst.rows) {
            base = dst.row<__half>(t0) + h * HD + v;
            pitch = dst.ld;
        }
#pragma unroll 1
        for (int half = 0; half < 2; half++) {
            uint32_t a1[32], a2[32];
            tmem_load_32x32b_x32(tl + 32 * half, a1);
            tmem_load_32x32b_x32(tl + 64 + 32 * half, a2);
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const int t = 32 * half + i;
                const int64_t tok = t0 + t;
                if (tok >= T) continue;
                const float o = scale * fmaf(sm.gam[t], __uint_as_float(a1[i]), __uint_as_float(a2[i]));
                const float zv = fminf(fmaxf(half ? z1[i] : z0[i], -88.0f), 88.0f);
                const float nv = (o * rd.inv[t]) * hnv;
                __half* out = base != nullptr ? base + t * pitch : dst.row<__half>(tok) + h * HD + v;
                *out = __float2half_rn(nv * silu_fast(zv));
            }
        }
    }
    if (!ok && tid == 0) {  // a load timed out: give the bulk copies a bounded chance to land
        mbar_wait(smem_u32(&sm.ld_s), 0, err);
        mbar_wait(smem_u32(&sm.ld_d), 0, err);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, kOutTmemCols);
}

template <typename K>
int set_smem(K kern, size_t bytes) {
    GDN_CUDA(cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return GDN_OK;
}

}  // namespace

size_t chunk_img_w_bytes() { return kImgWBytes; }
size_t chunk_img_e_bytes() { return kImgEBytes; }
size_t chunk_img_s_bytes() { return kImgSBytes; }

int launch_chunk_scan_tc(const uint8_t* wimg, const uint8_t* eimg, const uint8_t* uimg, const float* gchunk, float* S,
                         uint8_t* simg, uint8_t* dimg, int hv, int64_t nc, cudaStream_t s) {
    const size_t smem = sizeof(ScanTcSmem) + 1024;
    int st = set_smem(chunk_scan_tc_kernel, smem);
    if (st) return st;
    return launch_pdl("chunk_scan_tc_kernel", chunk_scan_tc_kernel, dim3((unsigned)(2 * hv)), dim3(kScanThreads), smem, s,
                      wimg, eimg, uimg, gchunk, S, simg, dimg, nc, device_error_word());
}

int launch_chunk_out_tc(const bf16* qn, const bf16* kn, const uint8_t* simg, const uint8_t* dimg, const float* gcum,
                        const float* proj, int64_t ldp, const float* head_norm, __half* gated, const RowDest& dst,
                        int64_t T, int64_t Tp, int hk, int hv, int qkv, int head_map, cudaStream_t s) {
    const size_t smem = sizeof(OutTcSmem) + 1024;
    int st = set_smem(chunk_out_tc_kernel, smem);
    if (st) return st;
    return launch_pdl("chunk_out_tc_kernel", chunk_out_tc_kernel, dim3((unsigned)(Tp / CH), (unsigned)hv), dim3(128),
                      smem, s, qn, kn, simg, dimg, gcum, proj, ldp, head_norm, gated, dst, T, Tp, hk, hv, qkv,
                      head_map, device_error_word());
}

}  // namespace gdn
