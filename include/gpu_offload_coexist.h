/*
 * gpu_offload_coexist.h -- links the reference's expert cache beside
 * libwinmoe_gdn.so.
 *
 * The engine (engine/runtime/winmoe_inference.c) calls two groups of
 * gpu_offload.h functions: the DeltaNet / GQA offload and the lifetime calls
 * (gpu_init, gpu_shutdown, gpu_vram_used_mb: :868, :944, :2335), which this
 * library exports under the same names (gpu_offload_gdn.h), and the expert
 * cache (gpu_set_expert_limit :873, gpu_find_cached_expert :1760 / :1800,
 * gpu_expert_ffn_fused :1803, gpu_cache_expert :1830), which stays the
 * reference's own code (engine/runtime/gpu_offload.cu:535-811), unchanged.
 *
 * Compile that file with this header forced in:
 *
 *   nvcc -O2 -c engine/runtime/gpu_offload.cu -include gpu_offload_coexist.h \
 *        -I <repo>/include -o gpu_offload_experts.o
 *
 * Every function this library also defines is renamed to gdn_ref_*, so the
 * two objects define no gpu_* symbol twice; the expert-cache functions keep
 * their names.  The library's gpu_init / gpu_shutdown / gpu_vram_used_mb call
 * the renamed gdn_ref_offload_init / _shutdown / _vram_used_mb when they are
 * linked (weak references), so the reference module's streams and buffers
 * exist before the engine's first expert call.  gdn_offload_experts_linked()
 * (winmoe_gdn.h) reports whether they were.
 */
#ifndef GPU_OFFLOAD_COEXIST_H
#define GPU_OFFLOAD_COEXIST_H

/* lifetime: called through this library's gpu_init / gpu_shutdown / gpu_vram_used_mb */
#define gpu_init gdn_ref_offload_init
#define gpu_shutdown gdn_ref_offload_shutdown
#define gpu_vram_used_mb gdn_ref_offload_vram_used_mb
#define gpu_is_initialized gdn_ref_offload_is_initialized

/* DeltaNet offload (gpu_offload.h:25-53): served by this library */
#define gpu_upload_deltanet_weights gdn_ref_upload_deltanet_weights
#define gpu_deltanet_projections gdn_ref_deltanet_projections
#define gpu_ssm_out_projection gdn_ref_ssm_out_projection
#define gpu_launch_qkv_gate gdn_ref_launch_qkv_gate
#define gpu_wait_qkv_gate gdn_ref_wait_qkv_gate
#define gpu_launch_ssm_out gdn_ref_launch_ssm_out
#define gpu_wait_ssm_out gdn_ref_wait_ssm_out
#define gpu_get_qkv_out gdn_ref_get_qkv_out
#define gpu_get_gate_out gdn_ref_get_gate_out
#define gpu_get_ssm_out_buf gdn_ref_get_ssm_out_buf

/* GQA projections (gpu_offload.h:56-67): served by this library */
#define gpu_upload_gqa_weights gdn_ref_upload_gqa_weights
#define gpu_gqa_projections gdn_ref_gqa_projections
#define gpu_gqa_output gdn_ref_gqa_output

#endif /* GPU_OFFLOAD_COEXIST_H */
