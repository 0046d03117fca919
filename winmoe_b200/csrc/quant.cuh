// Launchers of the GGUF quant kernels (quant.cu) and the tensor-core GEMM
// (gemm_tc.cu).  All are stream-ordered and return a gdn_status.
#pragma once
#include "gdn_common.cuh"

namespace gdn {

int launch_q8_0_repack(const void* blocks, int8_t* qs, uint16_t* d, int64_t rows, int64_t cols, cudaStream_t s);
int launch_q8_0_dequant(const int8_t* qs, const uint16_t* d, float* out, int64_t rows, int64_t cols,
                        cudaStream_t s);
// y[m][ldy] = x[m][:] . W[n][:] on CUDA cores, dequantising in registers.
// quant_matvec type 8 exactly as the reference's CPU computes it (Q8_K
// activations when k % 256 == 0 and n >= 128, else fp32 block dots), bit for bit.
int launch_q8_0_gemv_ref(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const float* x, int64_t m,
                         float* y, int64_t ldy, cudaStream_t s);
// quantize_row_q8_K: n fp32 values -> n / 256 GGUF block_q8_K (292 bytes each).
int launch_quantize_q8_K(const float* x, void* out, int64_t n, cudaStream_t s);
int launch_q8_0_gemv(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* x, int x_dtype,
                     int64_t m, float* y, int64_t ldy, cudaStream_t s);
// Streamed GEMV (gemv_stream.cu), fmt 0 = Q8_0 planes (wd = the fp16 scale
// plane), 1 = Q4_K blocks: k a multiple of 512 (Q8_0) or 256 (Q4_K) and
// 16-byte aligned weights; gemv_stream_fits says whether a call qualifies.
// Options (the expert FFN's fusions).  nseg > 0: the n = nseg * seg_rows
// weight rows come from nseg Q4_K / Q5_K matrices seg[s] (row r from matrix
// r / seg_rows), the CTAs split evenly over the matrices; matrix s's input is
// the activations offset by s * x_seg elements within each row, rows ldx
// elements apart (0: the input length).  swiglu: fp32 activation rows hold
// [g | u] (2 k values) and the input is (g * sigmoid(g)) * u.  kseg > 0 (with
// swiglu, K-quants): the k axis is kseg matrices seg[s] side by side, each
// [n][k / kseg]; activation rows hold [s][g | u] per segment and segment s's
// inputs are scaled by kscale[s] (y = sum_s W_s (kscale_s a_s)).  y = alpha *
// result, or with accumulate y += alpha * result.
constexpr int kGemvMaxSeg = 16;
struct GemvOpts {
    int nseg = 0;
    const uint8_t* seg[kGemvMaxSeg] = {};
    int64_t seg_rows = 0;
    int64_t x_seg = 0;
    int64_t ldx = 0;
    int swiglu = 0;
    int kseg = 0;
    float kscale[kGemvMaxSeg] = {};
    int accumulate = 0;
    float alpha = 1.0f;
};
bool gemv_stream_fits(int fmt, const void* wq, const void* wd, int64_t k, int64_t m);
int launch_gemv_stream(int fmt, const void* wq, const void* wd, int64_t n, int64_t k, const void* x, int x_dtype,
                       int64_t m, float* y, int64_t ldy, cudaStream_t s, const GemvOpts& o = GemvOpts());
int launch_q4_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, cudaStream_t s);
int launch_q5_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, cudaStream_t s);
int launch_q5_k_gemv(const void* blocks, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m, float* y,
                     int64_t ldy, cudaStream_t s);
// The expert FFN (expert.cu): out[m][hidden] (+)= sum_e weight_e * down_e(SwiGLU(gate_e x, up_e x))
// over n_experts <= kMaxExpertsPerCall experts (one expert: gdn_expert_ffn).
constexpr int kMaxExpertsPerCall = kGemvMaxSeg / 2;
size_t experts_ffn_workspace_bytes(int n_experts, int64_t m, int64_t hidden, int64_t inter);
int launch_experts_ffn(int n_experts, const void* const* w_gate, const void* const* w_up, const void* const* w_down,
                       int gate_type, int down_type, int64_t hidden, int64_t inter, const void* x, int x_dtype,
                       int64_t m, const float* weights, float* out, int accumulate, void* workspace,
                       size_t workspace_bytes, cudaStream_t s);
int launch_q4_k_gemv(const void* blocks, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m, float* y,
                     int64_t ldy, cudaStream_t s);

// Prefill preprocessing fused into the tensor-core GEMM's epilogue (the single
// fp16-operand path): output columns [0, qkv) are the q, k, v channels of the
// input projection, 128 per head (heads 0..hk-1 q, hk..2hk-1 k, then v).  For
// each M tile of `rows` tokens, rows 3.. leave as conv1d + SiLU (+ L2 norm for q
// and k) in bf16 [head][Tp][128]; rows 0..2 need the previous tile's raw rows and
// are finished by the prefill's edge kernel from `edge` (per tile: raw rows 0..2
// and rows-3..rows-1).  Raw rows T-4..T-1 go to `win` (the next conv window).
// Columns >= qkv take the plain fp32 epilogue.
struct PrepEpilogue {
    int enabled = 0;
    int qkv = 0, hk = 0;
    int rows = 0;                  // set by the launcher: tokens per M tile (128 or 256)
    int64_t T = 0, Tp = 0;         // tokens, and rows of the bf16 outputs (T rounded up; zeros past T)
    const float* conv_w = nullptr; // [qkv][4], or none: no conv, no SiLU
    __nv_bfloat16 *qn = nullptr, *kn = nullptr, *vb = nullptr;
    float* edge = nullptr;         // [ceil(T / rows)][6][qkv]
    float* win = nullptr;          // [4][qkv]: raw row t at slot t - (T - 4)
};

// Options of the tensor-core GEMM.
struct TcOptions {
    bool split_precision = false;  // weights as hi + lo operands (two MMAs): fp32-GEMV accuracy
    int splits = 1;                // split-K factor (partials in `workspace`, then a fixed-order sum)
    void* workspace = nullptr;
    size_t workspace_bytes = 0;
    // Activations stored as K blocks a[k / a_blk_k][a_rows][a_blk_k] (0: plain
    // [m][k]); the GEMM's m rows are rows a_row0 .. a_row0 + m - 1 of every block.
    int64_t a_blk_k = 0, a_rows = 0, a_row0 = 0;
    // ... or the K blocks in separate buffers (this GPU's or peers' memory over
    // NVLink, each [a_rows][a_blk_k]): a_block_ptrs[k / a_blk_k], a_nblocks <= 8
    const void* const* a_block_ptrs = nullptr;
    int a_nblocks = 0;
    PrepEpilogue* prep = nullptr;  // single-operand path only; `rows` is filled in
    // Leave the split-K partials [splits][m][n] for the caller to sum (y must then
    // be `workspace` with ldy = n: with one split the product lands there as
    // [1][m][n]); the split count used is written to *splits_used.
    bool partials_only = false;
    int* splits_used = nullptr;
};
size_t gemm_tc_workspace_bytes(int64_t m, int64_t n, int splits);

// Tensor-core (tcgen05) Q8_0 GEMM: y[m][ldy] = a[m][:] . W[n][:], a fp16 or
// bf16 [m][k] row-major (k % 64 == 0, 16-byte aligned), fp32 out.
int launch_q8_0_gemm_tc(const int8_t* qs, const uint16_t* d, int64_t n, int64_t k, const void* a, bool a_bf16,
                        int64_t m, float* y, int64_t ldy, const TcOptions& opt, cudaStream_t s);
// The same for GGUF Q4_K blocks [n][k / 256] (144 bytes each), fp16 activations,
// exact weights (hi + lo operands): the fp32 product up to summation order.
int launch_q4_k_gemm_tc(const void* blocks, int64_t n, int64_t k, const void* a, int64_t m, float* y, int64_t ldy,
                        const TcOptions& opt, cudaStream_t s);
// fp32 / bf16 / fp16 activations -> fp16 or bf16 (the tensor-core operand).
int launch_convert(const void* x, int x_dtype, void* out, bool to_bf16, int64_t count, cudaStream_t s);

}  // namespace gdn
