/*
 * winmoe_gdn.h -- C ABI of the B200 (sm_100a) Gated DeltaNet hot path.
 *
 * Two groups of entry points, both exported by winmoe_b200/libwinmoe_gdn.so:
 *
 *  1. The reference engine's DeltaNet offload API, same names and signatures
 *     as engine/runtime/gpu_offload.h:19-53 (gpu_init ... gpu_get_ssm_out_buf),
 *     so engine/runtime/winmoe_inference.c links against this library without
 *     source changes (its call sites: 868, 938-942, 1215-1226, 1437-1440).
 *     Host pointers in, host pointers out, 0 = ok / -1 = error, one host
 *     thread, module-owned device buffers -- as in the reference.
 *
 *  2. gdn_* entry points: device pointers, a caller stream, no hidden
 *     allocation, every call returns a gdn_status.  These cover what the
 *     reference does on the CPU in deltanet_forward
 *     (engine/runtime/deltanet_impl.h:145-377) -- for a batch of sequences
 *     (decode) or a run of tokens of one sequence (chunked prefill) -- and the
 *     GGUF Q8_0 / Q4_K dequant + GEMV kernels behind quant_matvec
 *     (engine/runtime/transformer.h:157-194).
 *
 *  3. gdn_layer_forward: deltanet_forward's own argument list (raw GGUF
 *     blocks + GGML type ids, dims from gdn_dn_init_dims) for batch x T
 *     tokens; like group 1 it owns the device memory it prepares.
 *
 * Conventions: all pointers of group 2 are device pointers unless stated;
 * `stream` is a cudaStream_t (NULL = legacy default stream); every call is
 * stream-ordered and returns after enqueueing.  Shapes use int64_t.
 * No entry point aborts or exits; on error the status is returned and
 * gdn_last_error() describes it (thread-local string).
 */
#ifndef WINMOE_GDN_H
#define WINMOE_GDN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */

typedef enum gdn_status {
    GDN_OK = 0,
    GDN_ERR_CUDA = -1,    /* a CUDA call failed (the reference's CHECK_CUDA -1, gpu_offload.cu:23-29) */
    GDN_ERR_SHAPE = -2,   /* a dimension is out of range or not a multiple the kernel needs */
    GDN_ERR_TYPE = -3,    /* unsupported GGML type id or activation dtype */
    GDN_ERR_TIMEOUT = -4, /* a bounded device-side wait gave up (read with gdn_check_device_error) */
    GDN_ERR_STATE = -5,   /* not initialised / layer not uploaded (gpu_offload.cu:1078) */
    GDN_ERR_ARG = -6,     /* NULL or misaligned pointer, workspace too small */
    GDN_ERR_NOMEM = -7    /* an allocation of the legacy API failed */
} gdn_status;

/* Activation dtypes accepted by the gdn_* entry points. */
enum { GDN_DTYPE_F32 = 0, GDN_DTYPE_BF16 = 1, GDN_DTYPE_F16 = 2 };

/* GGML type ids (engine/runtime/gguf_parser.h:21-29). */
enum { GDN_GGML_F32 = 0, GDN_GGML_Q8_0 = 8, GDN_GGML_Q4_K = 12, GDN_GGML_Q5_K = 13 };

/* Head maps of the Q/K key group shared by a value head h (hpg = Hv / Hk). */
enum {
    GDN_HEAD_MAP_GROUPED = 0,    /* g = h / hpg: engine/runtime/deltanet_impl.h:280 (default) */
    GDN_HEAD_MAP_INTERLEAVED = 1 /* g = h % Hk:  engine/runtime/winmoe_inference.c:1330 */
};

/* Description of the last error on this host thread ("" if none). */
GDN_API const char* gdn_last_error(void);
/* ABI version of this library (major*100 + minor). */
GDN_API int gdn_abi_version(void);
/* Reads and clears the device error word that bounded waits set; returns
 * GDN_OK or GDN_ERR_TIMEOUT.  Synchronises `stream`. */
GDN_API int gdn_check_device_error(void* stream);

/* ------------------------------------------------------------ quant blocks */

/*
 * Q8_0 in HBM.  GGUF stores a Q8_0 row as blocks of {fp16 d; int8 qs[32]}
 * (34 bytes, engine/runtime/q8_dequant.h:15-18).  On the device the library
 * keeps the same numbers as two planes: qs [rows][cols] int8 and
 * d [rows][cols/32] fp16 bits, so that every load is 16-byte aligned and the
 * tensor-core path can move tiles with TMA.  Dequantised weights are the
 * same floats d*q either way.
 *
 * gdn_q8_0_repack: GGUF blocks (device) -> planes (device).  cols % 32 == 0.
 * Replaces the raw-block cudaMemcpy of gpu_upload_deltanet_weights
 * (engine/runtime/gpu_offload.cu:1056-1061).
 */
GDN_API int gdn_q8_0_repack(const void* blocks, int8_t* qs, uint16_t* d,
                    int64_t rows, int64_t cols, void* stream);

/* Dequantise Q8_0 planes to fp32, bit-exact with q8_dequant_row
 * (engine/runtime/q8_dequant.h:116-126): out[r][c] = float(d) * q. */
GDN_API int gdn_q8_0_dequant(const int8_t* qs, const uint16_t* d, float* out,
                     int64_t rows, int64_t cols, void* stream);

/* Precision flags of gdn_q8_0_gemm. */
enum {
    GDN_GEMM_EXACT = 0,    /* fp32-GEMV accuracy (the reference's fp32-activation projection) */
    GDN_GEMM_FAST = 1,     /* tensor cores with one fp16/bf16 weight operand */
    GDN_GEMM_REF_EXACT = 2 /* the reference CPU's quant_matvec bit for bit (fp32 x, see below) */
};

/*
 * y[m][n] = sum_k x[m][k] * W[n][k] with W Q8_0 planes [n_rows][k].
 * The quant_matvec of engine/runtime/transformer.h:157-194 (type 8) for a
 * batch of m activation rows (the reference computes one row per call, with
 * fp32 activations on its GPU route: q8_matvec_kernel,
 * engine/runtime/gpu_offload.cu:152-199).  x_dtype: F32, BF16 or F16; k % 32 == 0.
 * m >= 16, k % 64 == 0, 16-byte aligned x: tcgen05 tensor cores with fp32
 * accumulation in TMEM --
 *   GDN_GEMM_EXACT, fp16 x: each weight split into exact hi + lo fp16
 *     operands (two MMAs), so only the summation order differs from fp32;
 *   GDN_GEMM_FAST, fp16 or bf16 x: one operand, weights rounded once to the
 *     x type.
 * Every other case (m < 16, fp32 x, bf16 x with EXACT): the streamed GEMVs
 * (int8 tensor cores from 3 rows), fp32-activation arithmetic.
 */
GDN_API int gdn_q8_0_gemm(const int8_t* qs, const uint16_t* d, int64_t n_rows, int64_t k,
                  const void* x, int x_dtype, int64_t m, float* y, int flags, void* stream);
/*
 * GDN_GEMM_REF_EXACT (x_dtype F32, k % 32 == 0, k <= 8192): each y[j] is what
 * the reference's CPU quant_matvec(type 8) returns for x[j], bit for bit --
 * with k >= 256 and n_rows >= 128 the activations are quantised to Q8_K
 * (q8k_quant.h:32-104) and every 32-block term is fp16(d_w)*d_a*sum(q_w q_a)
 * (q8_dot_q8k, q8_dequant.h:35-61), over the blocks of whole 256-value groups
 * only, as the reference's branch sums them (q8_dequant.h:75-101); otherwise
 * every block is the 16-lane fp32 dot of q8_dot_block (q8_dequant.h:21-32).
 * Terms are added in block order.
 * No counterpart on the reference's GPU route, which uses fp32 activations.
 */

/* quantize_row_q8_K (engine/runtime/q8k_quant.h:99-104) on the device: n fp32
 * values (n % 256 == 0) -> n / 256 GGUF block_q8_K {float d; int8 qs[256];
 * int16 bsums[16]} (292 bytes each), bit-identical to the CPU's. */
GDN_API int gdn_quantize_q8_K(const float* x, void* out, int64_t n, void* stream);

/*
 * Q4_K: GGUF superblocks of 256 weights, {fp16 d; fp16 dmin; u8 scales[12];
 * u8 qs[128]} (144 bytes, engine/runtime/q4k_dequant.h:28-33), used as stored.
 * gdn_q4_k_dequant: fp32 weights in the GGML nibble layout with the float
 * formula of engine/runtime/gpu_offload.cu:237-250, w = (d*sc)*q - (dmin*m),
 * each operation rounded once; cols % 256 == 0.
 */
GDN_API int gdn_q4_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, void* stream);

/* y[m][n] = sum_k x[m][k] * W[n][k], W Q4_K [n_rows][k], fp32 accumulation
 * (q4k_matvec_kernel, engine/runtime/gpu_offload.cu:206-268).  x_dtype F32,
 * BF16 or F16; k % 256 == 0.  fp16 x with m >= 32 runs on the tcgen05 tensor
 * cores (superblocks by TMA, dequantised in shared memory into hi + lo fp16
 * operands: the fp32 product of those activations up to summation order);
 * otherwise the streamed GEMV, weight rows by bulk copy: m <= 2 splits the
 * activations per 32-block into three int8 levels (error below 5e-7 of the
 * block's max |x|) summed exactly by dp4a; m >= 3 splits them per 256-element
 * piece into a power-of-two scale and fp16 hi + lo parts (error about 1e-7 of
 * the piece's max |x|) against the exact fp16 weights q * sc on the fp16
 * tensor cores (mma.sync, fp32 accumulation over a superblock). */
GDN_API int gdn_q4_k_gemm(const void* blocks, int64_t n_rows, int64_t k,
                  const void* x, int x_dtype, int64_t m, float* y, void* stream);

/*
 * Q5_K: GGUF superblocks of 256 weights, {fp16 d; fp16 dmin; u8 scales[12];
 * u8 qh[32]; u8 qs[128]} (176 bytes, engine/runtime/q5k_dequant.h:19-25), used
 * as stored: weight 64c + j of a superblock is the low nibble of qs[32c + j]
 * with bit 2c of qh[j] as its fifth bit, weight 64c + 32 + j the high nibble
 * with bit 2c + 1 (engine/runtime/gpu_offload.cu:302-309).
 * gdn_q5_k_dequant: fp32 weights, w = (d*sc)*q - (dmin*m), each operation
 * rounded once; cols % 256 == 0.
 */
GDN_API int gdn_q5_k_dequant(const void* blocks, float* out, int64_t rows, int64_t cols, void* stream);

/* y[m][n] = sum_k x[m][k] * W[n][k], W Q5_K [n_rows][k], fp32 activations
 * (q5k_matvec_kernel / q5k_expert_kernel, engine/runtime/gpu_offload.cu:271-331,
 * 400-457); the streamed GEMV as gdn_q4_k_gemm's.  blocks 16-byte aligned,
 * k % 256 == 0 (GDN_ERR_SHAPE if a row's stages do not fit). */
GDN_API int gdn_q5_k_gemm(const void* blocks, int64_t n_rows, int64_t k,
                  const void* x, int x_dtype, int64_t m, float* y, void* stream);

/*
 * One MoE expert's FFN for m tokens, the reference's fused GPU route
 * (gpu_expert_ffn_fused, engine/runtime/gpu_offload.cu:718-751): gate and up
 * projections [inter][hidden] (GDN_GGML_Q4_K or GDN_GGML_Q5_K, gate_type for
 * both), a = (g * sigmoid(g)) * u (swiglu_kernel, :460-466), then the down
 * projection [hidden][inter] (down_type).  accumulate == 0: out[m][hidden] =
 * y (weight unused, as gpu_expert_ffn_fused returns it); accumulate != 0:
 * out += weight * y (gpu_expert_batch_add / weighted_add_kernel, :766-793).
 * Device pointers; x fp32, bf16 or fp16; hidden and inter multiples of 256;
 * the caller's workspace of gdn_expert_ffn_workspace_size(m, hidden, inter)
 * bytes.  The expert cache that owns the weights is the reference's.
 */
GDN_API size_t gdn_expert_ffn_workspace_size(int64_t m, int64_t hidden, int64_t inter);
GDN_API int gdn_expert_ffn(const void* w_gate, const void* w_up, const void* w_down, int gate_type, int down_type,
                  int64_t hidden, int64_t inter, const void* x, int x_dtype, int64_t m, float* out,
                  float weight, int accumulate, void* workspace, size_t workspace_bytes, void* stream);

/*
 * All selected experts of m tokens in one call, the reference's batched expert
 * block (gpu_expert_batch_start / gpu_expert_batch_add per expert /
 * gpu_expert_batch_finish, engine/runtime/gpu_offload.cu:756-809):
 *   out[m][hidden] = sum_e weights[e] * y_e      (accumulate == 0)
 *   out[m][hidden] += sum_e weights[e] * y_e     (accumulate != 0)
 * with y_e expert e's FFN as gdn_expert_ffn's (weights NULL: all 1).
 * w_gate / w_up / w_down: host arrays of n_experts device pointers,
 * 1 <= n_experts <= GDN_MAX_EXPERTS_PER_CALL; two launches whatever n_experts:
 * one streamed GEMV over all gate and up matrices, then one over all down
 * matrices side by side along k, expert e's inputs its SwiGLU times
 * weights[e] (the weighted sum formed in the GEMV's fp32 sums: equal to the
 * per-expert accumulation up to rounding).  Workspace of
 * gdn_experts_ffn_workspace_size(n_experts, m, hidden, inter) bytes, 256-byte
 * aligned; weights read on the host when the call is made.
 */
#define GDN_MAX_EXPERTS_PER_CALL 8
GDN_API size_t gdn_experts_ffn_workspace_size(int n_experts, int64_t m, int64_t hidden, int64_t inter);
GDN_API int gdn_experts_ffn(int n_experts, const void* const* w_gate, const void* const* w_up,
                  const void* const* w_down, int gate_type, int down_type, int64_t hidden, int64_t inter,
                  const void* x, int x_dtype, int64_t m, const float* weights, float* out, int accumulate,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- the layer */

/* Dimensions, as dn_init_dims derives them (engine/runtime/deltanet_impl.h:32-44):
 * Hv = inner / head_dim, hpg = Hv / Hk, KEY = Hk*d, QKV = 2*KEY + inner. */
typedef struct gdn_dims {
    int32_t hidden;      /* model width (2048 for the 35B-class config) */
    int32_t num_k_heads; /* Hk, ssm.group_count (16) */
    int32_t num_v_heads; /* Hv = ssm.inner_size / ssm.state_size (32) */
    int32_t head_dim;    /* d, ssm.state_size; must be 128 */
} gdn_dims;

/*
 * One layer's weights on the device (the DeltaNet fields of LayerWeights,
 * engine/runtime/transformer.h:63-78).
 *   in_*: the fused input projection, rows in this order:
 *         attn_qkv (QKV rows) | attn_gate = z (inner) | ssm_beta (Hv) | ssm_alpha (Hv);
 *         cols = hidden.  (Rows are independent in a GEMV, so stacking the
 *         reference's four tensors is exact.)
 *   out_*: ssm_out, rows = hidden, cols = inner.
 *   weight_type: GDN_GGML_Q8_0 (planes in in_qs / in_d, out_qs / out_d) or
 *         GDN_GGML_Q4_K (raw superblocks in in_blocks, out_blocks).
 *   conv1d_w [QKV][4] fp32 (ssm_conv1d.weight, tap k=0 oldest);
 *   ssm_a [Hv] (= -exp(A_log)), dt_bias [Hv], head_norm [head_dim] or NULL.
 */
typedef struct gdn_layer {
    gdn_dims dims;
    int32_t weight_type;
    int32_t head_map;
    const int8_t* in_qs;
    const uint16_t* in_d;
    const int8_t* out_qs;
    const uint16_t* out_d;
    const void* in_blocks;
    const void* out_blocks;
    const float* conv1d_w;
    const float* ssm_a;
    const float* dt_bias;
    const float* head_norm;
} gdn_layer;

/* Bytes of scratch gdn_decode_step needs for `batch` sequences. */
GDN_API size_t gdn_decode_workspace_size(const gdn_dims* dims, int64_t batch);

/*
 * One decode token for `batch` independent sequences: deltanet_forward
 * (engine/runtime/deltanet_impl.h:145-377) applied to each sequence b.
 *   x   [batch][hidden] (x_dtype F32 or BF16);  out [batch][hidden] fp32.
 *   S   [batch][Hv][d][d] fp32, row = key index, col = value index (DeltaNetState.S);
 *   conv_buf [batch][4][QKV] fp32 circular window, conv_pos [batch] int32
 *   (DeltaNetState.conv_buf / conv_pos) -- all updated in place.
 *   workspace: >= gdn_decode_workspace_size bytes of device memory, 256-aligned.
 */
GDN_API int gdn_decode_step(const gdn_layer* layer, int64_t batch,
                    const void* x, int x_dtype, float* out,
                    float* S, float* conv_buf, int32_t* conv_pos,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Flags of gdn_decode_step_ex. */
enum {
    /* The five projections as the reference's CPU computes them
     * (GDN_GEMM_REF_EXACT per tensor: Q8_K activations for attn_qkv, attn_gate
     * and ssm_out, fp32 block dots for the 32-row ssm_beta / ssm_alpha); Q8_0
     * layers and fp32 x only.  The rest of the step is the usual fp32 path. */
    GDN_DECODE_REF_PROJECTIONS = 1
};

/* gdn_decode_step with flags (0 = gdn_decode_step).  Same workspace.  No
 * counterpart in the reference: it selects the reference CPU's own projection
 * arithmetic (ref-exact) instead of the fp32-activation GPU route. */
GDN_API int gdn_decode_step_ex(const gdn_layer* layer, int64_t batch,
                               const void* x, int x_dtype, float* out,
                               float* S, float* conv_buf, int32_t* conv_pos,
                               void* workspace, size_t workspace_bytes, int flags, void* stream);

/* Size of the fixed scratch behind gdn_decode_step_noalloc (8 MiB). */
#define GDN_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/*
 * gdn_decode_step without a caller workspace and without any allocation: no
 * counterpart in the reference (its deltanet_forward keeps its scratch on the
 * CPU stack).  Same arguments, results and errors as gdn_decode_step; the
 * scratch is one static device array per device, GDN_NOALLOC_SCRATCH_BYTES
 * long, so batches whose workspace (as gdn_decode_workspace_size, for the
 * call's x_dtype) exceeds it are rejected with GDN_ERR_SHAPE: the 35B Q8_0
 * layer fits up to 63 sequences with fp32 x and up to 46 with bf16 / fp16 x,
 * whose projections run on the tensor cores from 5 sequences (fp32 x from 64)
 * with split-K partials that are reserved only then.
 *   - The first call on each device (with that device current) resolves the
 *     scratch address with cudaGetSymbolAddress; make that first call before
 *     any stream capture.
 *   - Nothing in the scratch has to start at zero: every byte a kernel reads
 *     is written earlier in the same call, so it is never cleared.
 *   - One scratch per device: calls whose GPU work overlaps (different streams
 *     without ordering between them, or several host threads) race on it.
 *     Issue them on one stream, or order the streams with events.
 */
GDN_API int gdn_decode_step_noalloc(const gdn_layer* layer, int64_t batch,
                                    const void* x, int x_dtype, float* out,
                                    float* S, float* conv_buf, int32_t* conv_pos, void* stream);

/* Bytes of scratch gdn_prefill needs for a prompt of T tokens. */
GDN_API size_t gdn_prefill_workspace_size(const gdn_dims* dims, int64_t T);

/*
 * Prefill: T tokens of ONE sequence through the layer, the result of T
 * consecutive deltanet_forward calls (engine/runtime/deltanet_impl.h:145-377;
 * the reference feeds prompts token by token, winmoe_inference.c:2286-2291).
 * Computed in chunks of 64 tokens in the WY form (bf16 tensor-core products,
 * fp32 state and triangular solve); the projections run on the tensor cores
 * (one fp16 weight operand; the beta/alpha gate rows exact).
 *   x [T][hidden] (F32, BF16 or F16);  out [T][hidden] fp32.
 *   S [Hv][d][d], conv_buf [4][QKV], conv_pos [1]: the sequence's state,
 *   read as the state before the prompt and updated to the state after it,
 *   in the layout of gdn_decode_step (ready for decoding).
 *   workspace: >= gdn_prefill_workspace_size bytes, 256-aligned.
 */
GDN_API int gdn_prefill(const gdn_layer* layer, int64_t T, const void* x, int x_dtype, float* out,
                        float* S, float* conv_buf, int32_t* conv_pos,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * gdn_prefill without the output projection, for value heads sharded over
 * GPUs: writes the gated head outputs (deltanet_impl.h:364-371, before the
 * out_proj of :374) as fp16 bits gated[T][num_v_heads * head_dim].  `layer`
 * may be a slice of a full layer (its value heads [h0, h1) with their key
 * groups: in_proj rows, conv weights, ssm_a / dt_bias of those heads); the
 * out_proj planes must still be set.  No single counterpart in the reference,
 * whose layer runs on one device; the slice's rows are computed exactly as in
 * the whole layer.  Same workspace as gdn_prefill.
 */
GDN_API int gdn_prefill_gated(const gdn_layer* layer, int64_t T, const void* x, int x_dtype, uint16_t* gated,
                              float* S, float* conv_buf, int32_t* conv_pos,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * out_proj of gathered head outputs: out[t - t0][hidden] = W_out . g[t] for
 * tokens t in [t0, t1), where g[t] is the concatenation over b of
 * gated[b][t][inner / blocks] (fp16 bits, as gdn_prefill_gated writes them
 * and an all-gather over `blocks` ranks stacks them).  Q8_0 planes out_qs /
 * out_d [hidden][inner] (deltanet_impl.h:374).  T >= 64 runs on the tensor
 * cores exactly as gdn_prefill's out_proj, so a sharded layer reproduces the
 * single-GPU output bit for bit; T < 64 needs blocks == 1.
 */
/*
 * gdn_prefill_gated with each token slice's rows stored where the rank that
 * owns the slice consumes them: with rows = T / ndst, token t's gated row
 * [num_v_heads * head_dim] goes to dst[t / rows] + (t % rows) * ld + col0
 * (fp16 bits; ld and col0 even, every dst 16-byte aligned).  With dst[r] =
 * rank r's [T / G][inner] buffer opened with gdn_ipc_open and col0 = this
 * rank's first head column, the chunked prefill's last kernel scatters the
 * heads straight into the ranks' out_proj operands over NVLink: an
 * all-to-all fused into the producer, each byte crossing once.  T % ndst == 0,
 * ndst <= 8.  No counterpart in the reference (one device).
 */
GDN_API int gdn_prefill_scatter(const gdn_layer* layer, int64_t T, const void* x, int x_dtype,
                                uint16_t* const* dst, int ndst, int64_t ld, int64_t col0,
                                float* S, float* conv_buf, int32_t* conv_pos,
                                void* workspace, size_t workspace_bytes, void* stream);

GDN_API int gdn_out_proj_gathered(const int8_t* out_qs, const uint16_t* out_d, int64_t hidden, int64_t inner,
                                  const uint16_t* gated, int blocks, int64_t T, int64_t t0, int64_t t1,
                                  float* out, void* stream);

/*
 * The same out_proj with the head blocks left where the ranks wrote them:
 * blocks[b] points at rank b's gated[T][inner / blocks] (fp16 bits) -- this
 * GPU's buffer or a peer's opened with gdn_ipc_open -- and the tensor cores
 * read each token slice's K blocks straight from there (plain TMA loads over
 * NVLink, each CTA its own; no copy), in the single-GPU k order.  T >= 64,
 * blocks <= 8.  Replaces the all-gather of the gated heads: each rank reads
 * only the rows of its own token range.  No counterpart in the reference.
 */
GDN_API int gdn_out_proj_blocks(const int8_t* out_qs, const uint16_t* out_d, int64_t hidden, int64_t inner,
                                const uint16_t* const* blocks, int nblocks, int64_t T, int64_t t0, int64_t t1,
                                float* out, void* stream);

/*
 * Device buffers shared between the processes of one node (CUDA IPC), for
 * the head blocks above: gdn_ipc_alloc allocates `bytes` on the current
 * device and writes its 64-byte handle; another process opens the handle with
 * gdn_ipc_open (peer access over NVLink) and releases it with gdn_ipc_close;
 * the owner frees it with gdn_ipc_free after every peer has closed it.
 */
GDN_API int gdn_ipc_alloc(size_t bytes, void** ptr, void* handle64);
GDN_API int gdn_ipc_open(const void* handle64, void** ptr);
GDN_API int gdn_ipc_close(void* ptr);
GDN_API int gdn_ipc_free(void* ptr);

/*
 * Residual add + RMSNorm between stacked layers, per row of `hidden`:
 *   x <- x + add            (winmoe_inference.c:1652; add may be NULL)
 *   y  = (x * scale) * w,   scale = 1 / sqrtf(float(sum x^2 / hidden) + 1e-6)
 *                           (attention.h:29-44, the sum in double; w NULL = ones)
 * x, add fp32 [T][hidden]; y [T][hidden] in y_dtype (F32, BF16 or F16).
 */
GDN_API int gdn_add_rmsnorm(float* x, const float* add, const float* w, void* y, int y_dtype,
                            int64_t T, int64_t hidden, void* stream);

/*
 * gdn_add_rmsnorm over a token slice, y broadcast: row t of the slice is
 * stored at y[b] + (row0 + t) * hidden for every b < ny (ny <= 8) -- every
 * rank's [T][hidden] copy of the next layer's input, peers' copies opened
 * with gdn_ipc_open, written over NVLink by the kernel that computes them
 * (an all-gather fused into the RMSNorm).  No counterpart in the reference.
 */
GDN_API int gdn_add_rmsnorm_bcast(float* x, const float* add, const float* w, void* const* y, int ny,
                                  int y_dtype, int64_t T, int64_t hidden, int64_t row0, void* stream);

/* ------------------------------------------------------ the reference's call */

/* dn_init_dims (engine/runtime/deltanet_impl.h:32-44): the dims every later
 * gdn_layer_forward uses, from the GGUF keys ssm.inner_size, ssm.group_count
 * and ssm.state_size; 0 or less picks the reference's defaults (8192, 16,
 * 128).  head_dim must be 128.  Process-wide, like the reference's statics. */
GDN_API int gdn_dn_init_dims(int ssm_inner_size, int ssm_group_count, int ssm_head_dim);

/* DeltaNetState (deltanet_impl.h:48-60) on the device: S [batch][Hv][d][d]
 * fp32, conv_buf [batch][4][QKV] fp32 (NULL: no conv1d), conv_pos [batch]
 * int32 -- the reference's per-call scratch (tmp_*) is the library's. */
typedef struct gdn_dn_state {
    float* S;
    float* conv_buf;
    int32_t* conv_pos;
} gdn_dn_state;

/*
 * deltanet_forward (engine/runtime/deltanet_impl.h:145-162; the engine's CPU
 * route, winmoe_inference.c:1450-1460) on the GPU, same arguments in the same
 * order plus batch, T and a stream; returns a gdn_status.
 *   output [batch][T][hidden_dim] fp32, x [batch][T][hidden_dim] fp32 and the
 *   state: device memory.  T == 1: one decode token for `batch` sequences
 *   (gdn_decode_step); T > 1: a prompt of T tokens per sequence (gdn_prefill,
 *   sequence after sequence).
 *   w_*: raw GGUF blocks with their GGML type ids -- all Q8_0 (8) or all Q4_K
 *   (12); w_alpha / w_beta may be NULL (those projections are 0, as in the
 *   reference).  conv1d_w [QKV][4], a_log (the GGUF ssm_a = -exp(A_log), as
 *   the engine passes it), dt_bias [Hv], head_norm [128]: fp32, NULL as in
 *   the reference.  All of these may be host or device memory.
 * The first call with a weight set (the pointers above, on this device)
 * prepares it into library-owned device memory (a copy, Q8_0 repacked to
 * planes, the projections fused), kept until gdn_layer_release; later calls
 * with the same pointers reuse it, so the tensors must not change in place.
 * The step runs on one library-owned scratch per device, grown (after a
 * device synchronisation) when a call needs more.  Calls that prepare or grow
 * allocate; make them before any stream capture.  Calls share that scratch:
 * issue them on one stream per device, as the engine's single host thread does.
 */
GDN_API int gdn_layer_forward(float* output, const float* x, gdn_dn_state* state,
                              const void* w_qkv, int w_qkv_type,
                              const void* w_gate, int w_gate_type,
                              const void* w_alpha, int w_alpha_type,
                              const void* w_beta, int w_beta_type,
                              const void* w_out, int w_out_type,
                              const float* conv1d_w, const float* a_log,
                              const float* dt_bias, const float* head_norm,
                              int hidden_dim, int64_t batch, int64_t T, void* stream);
/* Frees the prepared copies of the weight sets whose w_qkv is this pointer
 * (current device).  No counterpart in the reference (its weights are the
 * caller's RAM). */
GDN_API int gdn_layer_release(const void* w_qkv);
/* Frees every prepared weight set and the scratch of the current device. */
GDN_API int gdn_layer_release_all(void);
/* 1 when the reference's expert-cache module is linked beside this library
 * with the renames of gpu_offload_coexist.h (gpu_init then initialises it
 * too), else 0.  No counterpart in the reference. */
GDN_API int gdn_offload_experts_linked(void);

/*
 * Optional phase timing of gdn_decode_step / gdn_prefill, for benchmarks.
 * While enabled (on the calling thread's current device), every call records a
 * CUDA event before and after each of its phases on its stream.
 * gdn_decode_phase_ms waits for the events of the most recent call and
 * writes up to n phase durations in milliseconds:
 *   [0] input projection  [1] conv/L2/gates  [2] state update  [3] out_proj
 * (gdn_prefill records the same four phases; [2] is the chunked recurrence).
 * Returns the number of phases written.  No counterpart in the reference
 * (which times whole tokens with QueryPerformanceCounter,
 * engine/runtime/winmoe_inference.c:1031-1037).
 */
GDN_API int gdn_profile_enable(int on);
GDN_API int gdn_decode_phase_ms(float* ms, int n);

#ifdef __cplusplus
}
#endif
#endif /* WINMOE_GDN_H */
