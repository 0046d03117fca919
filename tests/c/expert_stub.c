/*
 * Stand-in for the reference's expert-cache object where its source tree is
 * absent: the four expert functions the engine calls and the renamed
 * lifetime functions that include/gpu_offload_coexist.h gives the reference's
 * gpu_offload.cu.  An empty cache: nothing is ever found or cached.
 */
#include <stddef.h>

int gdn_ref_offload_init(void) { return 0; }
void gdn_ref_offload_shutdown(void) {}
float gdn_ref_offload_vram_used_mb(void) { return 0.0f; }

void gpu_set_expert_limit(int limit) { (void)limit; }
int gpu_find_cached_expert(int layer, int expert_id) {
    (void)layer;
    (void)expert_id;
    return -1;
}
int gpu_cache_expert(int layer, int expert_id, const void* gate_data, int gate_size, const void* up_data,
                     int up_size, const void* down_data, int down_size) {
    (void)layer; (void)expert_id; (void)gate_data; (void)gate_size;
    (void)up_data; (void)up_size; (void)down_data; (void)down_size;
    return -1;
}
int gpu_expert_ffn_fused(int cache_idx, const float* input, int hidden_dim, int intermediate, float* expert_out) {
    (void)cache_idx; (void)input; (void)hidden_dim; (void)intermediate; (void)expert_out;
    return -1;
}
