/*
 * gpu_offload_gdn.h -- the reference engine's DeltaNet and GQA GPU-offload API,
 * exported by winmoe_b200/libwinmoe_gdn.so with the same names, signatures and
 * return convention (0 = ok, -1 = error) as engine/runtime/gpu_offload.h.
 * Each line cites the declaration it replaces.
 *
 * The engine's call sites bind to these unchanged:
 *   gpu_init                      winmoe_inference.c:868
 *   gpu_upload_deltanet_weights   winmoe_inference.c:938-942
 *   gpu_launch_qkv_gate / wait    winmoe_inference.c:1215, 1224
 *   gpu_get_qkv_out / gate_out    winmoe_inference.c:1225-1226
 *   gpu_launch_ssm_out / wait     winmoe_inference.c:1437-1440
 *   gpu_upload_gqa_weights        winmoe_inference.c:956-960
 *   gpu_gqa_projections / output  winmoe_inference.c:1485-1486, 1624
 * Dimension arguments keep the engine's meaning: *_rows = input width,
 * *_cols = output width (winmoe_inference.c:938-942).  After an error,
 * gdn_last_error() (winmoe_gdn.h) says what failed.
 */
#ifndef GPU_OFFLOAD_GDN_H
#define GPU_OFFLOAD_GDN_H

#if defined(__GNUC__)
#define GDN_LEGACY_API __attribute__((visibility("default")))
#else
#define GDN_LEGACY_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

GDN_LEGACY_API int gpu_init(void);                                   /* gpu_offload.h:19 */
GDN_LEGACY_API void gpu_shutdown(void);                              /* gpu_offload.h:20 */
GDN_LEGACY_API int gpu_is_initialized(void);                         /* gpu_offload.h:21 */
GDN_LEGACY_API float gpu_vram_used_mb(void);                         /* gpu_offload.h:22 */

GDN_LEGACY_API int gpu_upload_deltanet_weights(int layer,            /* gpu_offload.h:25-28 */
    const void* qkv_q8, int qkv_rows, int qkv_cols,
    const void* gate_q8, int gate_rows, int gate_cols,
    const void* ssm_out_q8, int ssm_rows, int ssm_cols);

GDN_LEGACY_API int gpu_deltanet_projections(int layer,               /* gpu_offload.h:31-34 */
    const float* normed, int hidden_dim,
    float* qkv_out, int qkv_dim,
    float* gate_out, int gate_dim);

GDN_LEGACY_API int gpu_ssm_out_projection(int layer,                 /* gpu_offload.h:36-38 */
    const float* gated, int gated_dim,
    float* output, int output_dim);

GDN_LEGACY_API int gpu_launch_qkv_gate(int layer, int slot,          /* gpu_offload.h:41-43 */
    const float* normed, int hidden_dim,
    int qkv_dim, int gate_dim);
GDN_LEGACY_API int gpu_wait_qkv_gate(int slot);                      /* gpu_offload.h:44 */

GDN_LEGACY_API int gpu_launch_ssm_out(int layer, int slot,           /* gpu_offload.h:46-47 */
    const float* gated, int gated_dim, int output_dim);
GDN_LEGACY_API int gpu_wait_ssm_out(int slot);                       /* gpu_offload.h:48 */

GDN_LEGACY_API float* gpu_get_qkv_out(int slot);                     /* gpu_offload.h:51 */
GDN_LEGACY_API float* gpu_get_gate_out(int slot);                    /* gpu_offload.h:52 */
GDN_LEGACY_API float* gpu_get_ssm_out_buf(int slot);                 /* gpu_offload.h:53 */

/* Full-attention (GQA) layers: Q+gate, K, V and O projections, synchronous,
 * host buffers in and out.  *_rows = input width, *_cols = output width, as
 * the engine passes them (winmoe_inference.c:956-960, 1485-1486, 1624). */
GDN_LEGACY_API int gpu_upload_gqa_weights(int layer,                 /* gpu_offload.h:56-60 */
    const void* wq_q8, int wq_rows, int wq_cols,
    const void* wk_q8, int wk_rows, int wk_cols,
    const void* wv_q8, int wv_rows, int wv_cols,
    const void* wo_q8, int wo_rows, int wo_cols);
GDN_LEGACY_API int gpu_gqa_projections(int layer,                    /* gpu_offload.h:61-64 */
    const float* normed, int hidden_dim,
    float* q_gate_out, int q_gate_dim,
    float* k_out, int k_dim, float* v_out, int v_dim);
GDN_LEGACY_API int gpu_gqa_output(int layer,                         /* gpu_offload.h:65-67 */
    const float* attn_out, int attn_dim,
    float* output, int hidden_dim);

#ifdef __cplusplus
}
#endif
#endif /* GPU_OFFLOAD_GDN_H */
