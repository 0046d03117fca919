// The gdn_* C ABI (include/winmoe_gdn.h): argument checks, error strings, the
// device error word, and dispatch to the kernels.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "gdn_common.cuh"
#include "quant.cuh"
#include "decode.cuh"
#include "prefill.cuh"
#include "stack.cuh"

namespace gdn {

static thread_local char g_errbuf[512] = "";

int fail(int st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_errbuf, sizeof(g_errbuf), fmt, ap);
    va_end(ap);
    return st;
}

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return GDN_OK;
    snprintf(g_errbuf, sizeof(g_errbuf), "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return GDN_ERR_CUDA;
}

// One error word per device, a __device__ variable (no allocation).
__device__ uint32_t g_device_error_word;

uint32_t* device_error_word() {
    static uint32_t* ptrs[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (ptrs[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<uint32_t*>(p);
    }
    return ptrs[dev];
}

int sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (counts[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev] = n;
    }
    return counts[dev];
}

static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

static int check_act_dtype(int dt) {
    if (dt == GDN_DTYPE_F32 || dt == GDN_DTYPE_BF16 || dt == GDN_DTYPE_F16) return GDN_OK;
    return fail(GDN_ERR_TYPE, "activation dtype %d is not supported (0=f32, 1=bf16, 2=f16)", dt);
}

}  // namespace gdn

using namespace gdn;

extern "C" {

const char* gdn_last_error(void) { return g_errbuf; }

int gdn_abi_version(void) { return 100; }

int gdn_check_device_error(void* stream) {
    GDN_CUDA(cudaStreamSynchronize(as_stream(stream)));
    uint32_t w = 0;
    GDN_CUDA(cudaMemcpyFromSymbol(&w, g_device_error_word, sizeof(w)));
    if (w == 0) return GDN_OK;
    const uint32_t zero = 0;
    GDN_CUDA(cudaMemcpyToSymbol(g_device_error_word, &zero, sizeof(zero)));
    if (w & DEV_ERR_TIMEOUT) return fail(GDN_ERR_TIMEOUT, "a bounded device-side wait timed out (word 0x%x)", w);
    return fail(GDN_ERR_SHAPE, "a device-side bounds check failed (word 0x%x)", w);
}

int gdn_q8_0_repack(const void* blocks, int8_t* qs, uint16_t* d, int64_t rows, int64_t cols, void* stream) {
    if (rows < 0 || cols < 0 || cols % 32 != 0) return fail(GDN_ERR_SHAPE, "q8_0 repack: cols %% 32 != 0");
    if (!blocks || !qs || !d) return fail(GDN_ERR_ARG, "q8_0 repack: NULL pointer");
    if (!aligned(qs, 16) || !aligned(d, 2)) return fail(GDN_ERR_ARG, "q8_0 repack: qs must be 16-byte aligned");
    return launch_q8_0_repack(blocks, qs, d, rows, cols, as_stream(stream));
}

int gdn_q8_0_dequant(const int8_t* qs, const uint16_t* d, float* out, int64_t rows, int64_t cols, void* stream) {
    if (rows < 0 || cols < 0 || cols % 32 != 0) return fail(GDN_ERR_SHAPE, "q8_0 dequant: cols %% 32 != 0");
    if (!qs || !d || !out) return fail(GDN_ERR_ARG, "q8_0 dequant: NULL pointer");
    if (!aligned(qs, 16) || !aligned(out, 16)) return fail(GDN_ERR_ARG, "q8_0 dequant: qs/out must be 16-byte aligned");
    return launch_q8_0_dequant(qs, d, out, rows, cols, as_stream(stream));
}

int gdn_q8_0_gemm(const int8_t* qs, const uint16_t* d, int64_t n_rows, int64_t k, const void* x, int x_dtype,
                  int64_t m, float* y, int flags, void* stream) {
    if (n_rows < 0 || m < 0 || k <= 0 || k % 32 != 0) return fail(GDN_ERR_SHAPE, "q8_0 gemm: k must be a positive multiple of 32");
    if (!qs || !d || !x || !y) return fail(GDN_ERR_ARG, "q8_0 gemm: NULL pointer");
    int st = check_act_dtype(x_dtype);
    if (st) return st;
    if (!aligned(qs, 16)) return fail(GDN_ERR_ARG, "q8_0 gemm: qs must be 16-byte aligned");
    if (n_rows == 0 || m == 0) return GDN_OK;
    cudaStream_t s = as_stream(stream);
    if (flags == GDN_GEMM_REF_EXACT) {
        if (x_dtype != GDN_DTYPE_F32) return fail(GDN_ERR_TYPE, "q8_0 gemm: GDN_GEMM_REF_EXACT takes fp32 x");
        if (!aligned(x, 16)) return fail(GDN_ERR_ARG, "q8_0 gemm: x must be 16-byte aligned");
        return launch_q8_0_gemv_ref(qs, d, n_rows, k, static_cast<const float*>(x), m, y, n_rows, s);
    }
    if (flags != GDN_GEMM_EXACT && flags != GDN_GEMM_FAST) return fail(GDN_ERR_ARG, "q8_0 gemm: unknown flags %d", flags);
    // From 16 rows: the 35B layer's in_proj + out_proj take ~65 us (FAST, one weight operand) or ~70 us
    // (EXACT, hi + lo) at any batch up to 128, the GEMV 70 us at 16 rows and 4.3 us per further row
    const bool tc_shape = m >= 16 && k % 64 == 0 && aligned(x, 16) && aligned(d, 4);
    const bool tc = tc_shape && (flags == GDN_GEMM_FAST ? x_dtype != GDN_DTYPE_F32 : x_dtype == GDN_DTYPE_F16);
    if (tc) {
        TcOptions opt;
        opt.split_precision = (flags == GDN_GEMM_EXACT);
        return launch_q8_0_gemm_tc(qs, d, n_rows, k, x, x_dtype == GDN_DTYPE_BF16, m, y, n_rows, opt, s);
    }
    return launch_q8_0_gemv(qs, d, n_rows, k, x, x_dtype, m, y, n_rows, s);
}

int gdn_quantize_q8_K(const float* x, void* out, int64_t n, void* stream) {
    if (!x || !out) return fail(GDN_ERR_ARG, "quantize_q8_K: NULL pointer");
    if (n < 0) return fail(GDN_ERR_SHAPE, "quantize_q8_K: n < 0");
    if (!aligned(x, 16) || !aligned(out, 4)) return fail(GDN_ERR_ARG, "quantize_q8_K: x 16-byte, out 4-byte aligned");
    return launch_quantize_q8_K(x, out, n, as_stream(stream));
}

int gdn_q4_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, void* stream) {
    if (rows < 0 || cols < 0 || cols % 256 != 0) return fail(GDN_ERR_SHAPE, "q4_k dequant: cols %% 256 != 0");
    if (!blocks || !out) return fail(GDN_ERR_ARG, "q4_k dequant: NULL pointer");
    if (!aligned(blocks, 16) || !aligned(out, 16)) return fail(GDN_ERR_ARG, "q4_k dequant: pointers must be 16-byte aligned");
    return launch_q4_k_dequant(blocks, out, rows, cols, as_stream(stream));
}

// Q4_K batches from this many rows (fp16 activations) run on the tcgen05 GEMM;
// below, the fp16-MMA GEMV is faster (35B in_proj + out_proj at 16 rows: 42
// against 80 us; about even at 32).
constexpr int64_t kQ4kTcMinRows = 32;

int gdn_q4_k_gemm(const void* blocks, int64_t n_rows, int64_t k, const void* x, int x_dtype, int64_t m, float* y,
                  void* stream) {
    if (n_rows < 0 || m < 0 || k <= 0 || k % 256 != 0) return fail(GDN_ERR_SHAPE, "q4_k gemm: k must be a positive multiple of 256");
    if (!blocks || !x || !y) return fail(GDN_ERR_ARG, "q4_k gemm: NULL pointer");
    int st = check_act_dtype(x_dtype);
    if (st) return st;
    if (!aligned(blocks, 16)) return fail(GDN_ERR_ARG, "q4_k gemm: blocks must be 16-byte aligned");
    if (n_rows == 0 || m == 0) return GDN_OK;
    cudaStream_t s = as_stream(stream);
    if (x_dtype == GDN_DTYPE_F16 && m >= kQ4kTcMinRows && aligned(x, 16)) {
        // tensor cores, exact weights: the fp32 product of the fp16 activations up to
        // summation order; one split (no workspace: this entry point allocates nothing)
        return launch_q4_k_gemm_tc(blocks, n_rows, k, x, m, y, n_rows, TcOptions(), s);
    }
    return launch_q4_k_gemv(blocks, n_rows, k, x, x_dtype, m, y, n_rows, s);
}

int gdn_q5_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, void* stream) {
    if (rows < 0 || cols < 0 || cols % 256 != 0) return fail(GDN_ERR_SHAPE, "q5_k dequant: cols %% 256 != 0");
    if (!blocks || !out) return fail(GDN_ERR_ARG, "q5_k dequant: NULL pointer");
    return launch_q5_k_dequant(blocks, out, rows, cols, as_stream(stream));
}

int gdn_q5_k_gemm(const void* blocks, int64_t n_rows, int64_t k, const void* x, int x_dtype, int64_t m, float* y,
                  void* stream) {
    if (n_rows < 0 || m < 0 || k <= 0 || k % 256 != 0) return fail(GDN_ERR_SHAPE, "q5_k gemm: k must be a positive multiple of 256");
    if (!blocks || !x || !y) return fail(GDN_ERR_ARG, "q5_k gemm: NULL pointer");
    int st = check_act_dtype(x_dtype);
    if (st) return st;
    if (!aligned(blocks, 16)) return fail(GDN_ERR_ARG, "q5_k gemm: blocks must be 16-byte aligned");
    if (n_rows == 0 || m == 0) return GDN_OK;
    return launch_q5_k_gemv(blocks, n_rows, k, x, x_dtype, m, y, n_rows, as_stream(stream));
}

size_t gdn_expert_ffn_workspace_size(int64_t m, int64_t hidden, int64_t inter) {
    if (m <= 0 || hidden <= 0 || inter <= 0) return 0;
    return experts_ffn_workspace_bytes(1, m, hidden, inter);
}

size_t gdn_experts_ffn_workspace_size(int n_experts, int64_t m, int64_t hidden, int64_t inter) {
    if (n_experts <= 0 || n_experts > GDN_MAX_EXPERTS_PER_CALL || m <= 0 || hidden <= 0 || inter <= 0) return 0;
    return experts_ffn_workspace_bytes(n_experts, m, hidden, inter);
}

int gdn_experts_ffn(int n_experts, const void* const* w_gate, const void* const* w_up, const void* const* w_down,
                    int gate_type, int down_type, int64_t hidden, int64_t inter, const void* x, int x_dtype, int64_t m,
                    const float* weights, float* out, int accumulate, void* workspace, size_t workspace_bytes,
                    void* stream) {
    auto kq = [](int t) { return t == GDN_GGML_Q4_K || t == GDN_GGML_Q5_K; };
    if (!kq(gate_type) || !kq(down_type))
        return fail(GDN_ERR_TYPE, "expert ffn: weight types must be Q4_K (12) or Q5_K (13), got %d / %d", gate_type,
                    down_type);
    if (n_experts < 0 || n_experts > GDN_MAX_EXPERTS_PER_CALL)
        return fail(GDN_ERR_ARG, "expert ffn: %d experts, 0..%d per call", n_experts, GDN_MAX_EXPERTS_PER_CALL);
    if (m < 0 || hidden <= 0 || inter <= 0 || hidden % 256 != 0 || inter % 256 != 0)
        return fail(GDN_ERR_SHAPE, "expert ffn: hidden and inter must be positive multiples of 256");
    if (n_experts == 0 || m == 0) return GDN_OK;
    if (!w_gate || !w_up || !w_down || !x || !out || !workspace) return fail(GDN_ERR_ARG, "expert ffn: NULL pointer");
    for (int e = 0; e < n_experts; e++) {
        if (!w_gate[e] || !w_up[e] || !w_down[e]) return fail(GDN_ERR_ARG, "expert ffn: NULL weights of expert %d", e);
        if (!aligned(w_gate[e], 16) || !aligned(w_up[e], 16) || !aligned(w_down[e], 16))
            return fail(GDN_ERR_ARG, "expert ffn: weights of expert %d must be 16-byte aligned", e);
    }
    if (!aligned(workspace, 256)) return fail(GDN_ERR_ARG, "expert ffn: workspace must be 256-byte aligned");
    int st = check_act_dtype(x_dtype);
    if (st) return st;
    return launch_experts_ffn(n_experts, w_gate, w_up, w_down, gate_type, down_type, hidden, inter, x, x_dtype, m,
                              weights, out, accumulate, workspace, workspace_bytes, as_stream(stream));
}

int gdn_expert_ffn(const void* w_gate, const void* w_up, const void* w_down, int gate_type, int down_type,
                   int64_t hidden, int64_t inter, const void* x, int x_dtype, int64_t m, float* out, float weight,
                   int accumulate, void* workspace, size_t workspace_bytes, void* stream) {
    const float w = accumulate ? weight : 1.0f;  // stored unweighted, as gpu_expert_ffn_fused returns it
    return gdn_experts_ffn(1, &w_gate, &w_up, &w_down, gate_type, down_type, hidden, inter, x, x_dtype, m, &w, out,
                           accumulate, workspace, workspace_bytes, stream);
}

size_t gdn_decode_workspace_size(const gdn_dims* dims, int64_t batch) {
    if (dims == nullptr || batch <= 0) return 0;
    return decode_workspace_bytes(*dims, batch);
}

int gdn_decode_step(const gdn_layer* layer, int64_t batch, const void* x, int x_dtype, float* out, float* S,
                    float* conv_buf, int32_t* conv_pos, void* workspace, size_t workspace_bytes, void* stream) {
    return decode_step(layer, batch, x, x_dtype, out, S, conv_buf, conv_pos, workspace, workspace_bytes,
                       as_stream(stream));
}

// Scratch of gdn_decode_step_noalloc: a file-scope device array (one per
// device, zero-initialised storage of the module, never allocated by a call).
static __device__ __align__(256) unsigned char g_noalloc_scratch[GDN_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device, resolved once per
// device (cudaGetSymbolAddress with that device current) and cached.
static int noalloc_scratch(void** out) {
    static void* ptrs[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(GDN_ERR_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (ptrs[dev] == nullptr) {
        void* p = nullptr;
        GDN_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        if (!aligned(p, 256)) return fail(GDN_ERR_CUDA, "static scratch is not 256-byte aligned");
        ptrs[dev] = p;
    }
    *out = ptrs[dev];
    return GDN_OK;
}

int gdn_decode_step_noalloc(const gdn_layer* layer, int64_t batch, const void* x, int x_dtype, float* out, float* S,
                            float* conv_buf, int32_t* conv_pos, void* stream) {
    int st = validate_layer(layer);
    if (st) return st;
    if (batch <= 0 || batch > 65535)
        return fail(GDN_ERR_SHAPE, "batch must be in [1, 65535] (got %lld)", (long long)batch);
    const size_t need = decode_workspace_bytes_for(*layer, batch, 0, x_dtype);
    if (need > GDN_NOALLOC_SCRATCH_BYTES)
        return fail(GDN_ERR_SHAPE,
                    "gdn_decode_step_noalloc: batch %lld needs %zu bytes of scratch, more than the fixed %zu; "
                    "use gdn_decode_step with a caller workspace",
                    (long long)batch, need, (size_t)GDN_NOALLOC_SCRATCH_BYTES);
    void* ws = nullptr;
    if ((st = noalloc_scratch(&ws))) return st;
    return decode_step(layer, batch, x, x_dtype, out, S, conv_buf, conv_pos, ws, GDN_NOALLOC_SCRATCH_BYTES,
                       as_stream(stream));
}

int gdn_decode_step_ex(const gdn_layer* layer, int64_t batch, const void* x, int x_dtype, float* out, float* S,
                       float* conv_buf, int32_t* conv_pos, void* workspace, size_t workspace_bytes, int flags,
                       void* stream) {
    return decode_step(layer, batch, x, x_dtype, out, S, conv_buf, conv_pos, workspace, workspace_bytes,
                       as_stream(stream), flags);
}

size_t gdn_prefill_workspace_size(const gdn_dims* dims, int64_t T) {
    if (dims == nullptr || T <= 0) return 0;
    return prefill_workspace_bytes(*dims, T);
}

int gdn_prefill(const gdn_layer* layer, int64_t T, const void* x, int x_dtype, float* out, float* S, float* conv_buf,
                int32_t* conv_pos, void* workspace, size_t workspace_bytes, void* stream) {
    if (out == nullptr) return fail(GDN_ERR_ARG, "out must be non-NULL");
    return prefill(layer, T, x, x_dtype, out, nullptr, S, conv_buf, conv_pos, workspace, workspace_bytes,
                   as_stream(stream));
}

int gdn_prefill_gated(const gdn_layer* layer, int64_t T, const void* x, int x_dtype, uint16_t* gated, float* S,
                      float* conv_buf, int32_t* conv_pos, void* workspace, size_t workspace_bytes, void* stream) {
    if (gated == nullptr || layer == nullptr) return fail(GDN_ERR_ARG, "gated and layer must be non-NULL");
    RowDest dst{};
    dst.ptr[0] = gated;
    dst.n = 1;
    dst.rows = T;
    dst.ld = (int64_t)layer->dims.num_v_heads * 128;
    return prefill(layer, T, x, x_dtype, nullptr, &dst, S, conv_buf, conv_pos, workspace, workspace_bytes,
                   as_stream(stream));
}

int gdn_prefill_scatter(const gdn_layer* layer, int64_t T, const void* x, int x_dtype, uint16_t* const* dst, int ndst,
                        int64_t ld, int64_t col0, float* S, float* conv_buf, int32_t* conv_pos, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (dst == nullptr || layer == nullptr) return fail(GDN_ERR_ARG, "prefill scatter: NULL pointer");
    if (ndst < 1 || ndst > kMaxRowDest || T % ndst != 0)
        return fail(GDN_ERR_SHAPE, "prefill scatter: T=%lld over %d destinations (1..%d)", (long long)T, ndst,
                    kMaxRowDest);
    RowDest d{};
    for (int r = 0; r < ndst; r++) d.ptr[r] = dst[r];
    d.n = ndst;
    d.rows = T / ndst;
    d.ld = ld;
    d.col0 = col0;
    return prefill(layer, T, x, x_dtype, nullptr, &d, S, conv_buf, conv_pos, workspace, workspace_bytes,
                   as_stream(stream));
}

int gdn_out_proj_gathered(const int8_t* out_qs, const uint16_t* out_d, int64_t hidden, int64_t inner,
                          const uint16_t* gated, int blocks, int64_t T, int64_t t0, int64_t t1, float* out,
                          void* stream) {
    if (!out_qs || !out_d || !gated || !out) return fail(GDN_ERR_ARG, "out_proj gathered: NULL pointer");
    if (hidden <= 0 || inner <= 0 || inner % 64 != 0 || blocks < 1 || inner % ((int64_t)blocks * 64) != 0)
        return fail(GDN_ERR_SHAPE, "out_proj gathered: inner=%lld must split into %d blocks of a multiple of 64",
                    (long long)inner, blocks);
    if (T <= 0 || t0 < 0 || t1 > T || t0 >= t1) return fail(GDN_ERR_SHAPE, "out_proj gathered: bad token range");
    if (!aligned(gated, 16) || !aligned(out, 16) || !aligned(out_qs, 16))
        return fail(GDN_ERR_ARG, "out_proj gathered: pointers must be 16-byte aligned");
    cudaStream_t s = as_stream(stream);
    if (T < 64) {  // gdn_prefill's out_proj below 64 tokens: the CUDA-core GEMV
        if (blocks != 1) return fail(GDN_ERR_SHAPE, "out_proj gathered: T < 64 needs blocks == 1");
        return launch_q8_0_gemv(out_qs, out_d, hidden, inner, gated + t0 * inner, GDN_DTYPE_F16, t1 - t0, out,
                                hidden, s);
    }
    TcOptions opt;  // one fp16 weight operand, as gdn_prefill's out_proj
    opt.a_blk_k = inner / blocks;
    opt.a_rows = T;
    opt.a_row0 = t0;
    return launch_q8_0_gemm_tc(out_qs, out_d, hidden, inner, gated, false, t1 - t0, out, hidden, opt, s);
}

int gdn_out_proj_blocks(const int8_t* out_qs, const uint16_t* out_d, int64_t hidden, int64_t inner,
                        const uint16_t* const* blocks, int nblocks, int64_t T, int64_t t0, int64_t t1, float* out,
                        void* stream) {
    if (!out_qs || !out_d || !blocks || !out) return fail(GDN_ERR_ARG, "out_proj blocks: NULL pointer");
    if (nblocks < 1 || nblocks > 8 || inner % ((int64_t)nblocks * 64) != 0)
        return fail(GDN_ERR_SHAPE, "out_proj blocks: inner=%lld in %d blocks (1..8) of a multiple of 64",
                    (long long)inner, nblocks);
    if (T < 64 || t0 < 0 || t1 > T || t0 >= t1) return fail(GDN_ERR_SHAPE, "out_proj blocks: bad token range (T >= 64)");
    if (!aligned(out, 16) || !aligned(out_qs, 16)) return fail(GDN_ERR_ARG, "out_proj blocks: misaligned pointer");
    const void* ptrs[8];
    for (int b = 0; b < nblocks; b++) ptrs[b] = blocks[b];
    TcOptions opt;
    opt.a_blk_k = inner / nblocks;
    opt.a_rows = T;
    opt.a_row0 = t0;
    opt.a_block_ptrs = ptrs;
    opt.a_nblocks = nblocks;
    return launch_q8_0_gemm_tc(out_qs, out_d, hidden, inner, ptrs[0], false, t1 - t0, out, hidden, opt,
                               as_stream(stream));
}

int gdn_ipc_alloc(size_t bytes, void** ptr, void* handle64) {
    if (!ptr || !handle64 || bytes == 0) return fail(GDN_ERR_ARG, "ipc_alloc: bad argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    GDN_CUDA(cudaMalloc(ptr, bytes));
    const cudaError_t e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle64), *ptr);
    if (e != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return cuda_status(e, "cudaIpcGetMemHandle");
    }
    return GDN_OK;
}

int gdn_ipc_open(const void* handle64, void** ptr) {
    if (!ptr || !handle64) return fail(GDN_ERR_ARG, "ipc_open: bad argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    GDN_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return GDN_OK;
}

int gdn_ipc_close(void* ptr) {
    GDN_CUDA(cudaIpcCloseMemHandle(ptr));
    return GDN_OK;
}

int gdn_ipc_free(void* ptr) {
    GDN_CUDA(cudaFree(ptr));
    return GDN_OK;
}

int gdn_add_rmsnorm(float* x, const float* add, const float* w, void* y, int y_dtype, int64_t T, int64_t hidden,
                    void* stream) {
    if (!x || !y) return fail(GDN_ERR_ARG, "add_rmsnorm: x and y must be non-NULL");
    if (T < 0 || hidden <= 0 || T > INT32_MAX) return fail(GDN_ERR_SHAPE, "add_rmsnorm: bad shape");
    if (y_dtype != GDN_DTYPE_F32 && y_dtype != GDN_DTYPE_BF16 && y_dtype != GDN_DTYPE_F16)
        return fail(GDN_ERR_TYPE, "add_rmsnorm: y_dtype %d is not supported", y_dtype);
    RowDest d{};
    d.ptr[0] = y;
    d.n = 1;
    d.rows = T > 0 ? T : 1;
    d.ld = hidden;
    return launch_add_rmsnorm(x, add, w, d, y_dtype, T, hidden, as_stream(stream));
}

int gdn_add_rmsnorm_bcast(float* x, const float* add, const float* w, void* const* y, int ny, int y_dtype, int64_t T,
                          int64_t hidden, int64_t row0, void* stream) {
    if (!x || !y) return fail(GDN_ERR_ARG, "add_rmsnorm bcast: x and y must be non-NULL");
    if (T < 0 || hidden <= 0 || T > INT32_MAX || row0 < 0) return fail(GDN_ERR_SHAPE, "add_rmsnorm bcast: bad shape");
    if (ny < 1 || ny > kMaxRowDest) return fail(GDN_ERR_SHAPE, "add_rmsnorm bcast: %d destinations (1..%d)", ny,
                                                kMaxRowDest);
    if (y_dtype != GDN_DTYPE_F32 && y_dtype != GDN_DTYPE_BF16 && y_dtype != GDN_DTYPE_F16)
        return fail(GDN_ERR_TYPE, "add_rmsnorm bcast: y_dtype %d is not supported", y_dtype);
    RowDest d{};
    for (int r = 0; r < ny; r++) {
        if (y[r] == nullptr) return fail(GDN_ERR_ARG, "add_rmsnorm bcast: destination %d is NULL", r);
        d.ptr[r] = y[r];
    }
    d.n = ny;
    d.rows = T > 0 ? T : 1;
    d.ld = hidden;
    d.col0 = row0 * hidden;
    return launch_add_rmsnorm(x, add, w, d, y_dtype, T, hidden, as_stream(stream));
}

int gdn_profile_enable(int on) { return profile_enable(on); }

int gdn_decode_phase_ms(float* ms, int n) {
    if (ms == nullptr || n < 0) return fail(GDN_ERR_ARG, "gdn_decode_phase_ms: bad buffer");
    return phase_ms(ms, n);
}

}  // extern "C"
