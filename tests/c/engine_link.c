/*
 * Links the way the reference engine (engine/runtime/winmoe_inference.c) does
 * against this library: every gpu_* function the engine calls, plus
 * gdn_layer_forward, compiled against the headers in include/ and linked with
 * libwinmoe_gdn.so and the reference's expert cache (its gpu_offload.cu built
 * with include/gpu_offload_coexist.h forced in), or a stand-in for it.
 *
 *   engine_link          prints whether the expert module is linked (no GPU needed)
 *   engine_link --run    also runs every call once on tiny dims (needs a GPU)
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "gpu_offload_gdn.h"
#include "winmoe_gdn.h"

/* The expert-cache prototypes as the engine sees them (gpu_offload.h:70-100). */
int gpu_cache_expert(int layer, int expert_id, const void* gate_data, int gate_size, const void* up_data,
                     int up_size, const void* down_data, int down_size);
int gpu_find_cached_expert(int layer, int expert_id);
int gpu_expert_ffn_fused(int cache_idx, const float* input, int hidden_dim, int intermediate, float* expert_out);
void gpu_set_expert_limit(int limit);

#define CHECK(c)                                                      \
    do {                                                              \
        if (!(c)) {                                                   \
            fprintf(stderr, "FAILED %s:%d: %s (%s)\n", __FILE__, __LINE__, #c, gdn_last_error()); \
            return 1;                                                 \
        }                                                             \
    } while (0)

static uint32_t rng = 12345u;
static uint32_t next_u32(void) {
    rng ^= rng << 13;
    rng ^= rng >> 17;
    rng ^= rng << 5;
    return rng;
}

/* GGUF Q8_0 blocks (fp16 d, 32 int8) with small d, in host memory. */
static void* q8_0_blocks(int rows, int cols) {
    const int nb = cols / 32;
    unsigned char* p = (unsigned char*)malloc((size_t)rows * nb * 34);
    for (int i = 0; i < rows * nb; i++) {
        unsigned char* b = p + (size_t)i * 34;
        const uint16_t d = 0x2000 + (uint16_t)(next_u32() % 0x400); /* fp16 in [2^-7, 2^-6) */
        memcpy(b, &d, 2);
        for (int j = 0; j < 32; j++) b[2 + j] = (unsigned char)(int8_t)((int)(next_u32() % 255) - 127);
    }
    return p;
}

static float* floats(int n, float scale, float offset) {
    float* p = (float*)malloc((size_t)n * sizeof(float));
    for (int i = 0; i < n; i++) p[i] = offset + scale * ((float)(next_u32() % 2001) / 1000.0f - 1.0f);
    return p;
}

/* One pass over the engine's calls in its order (winmoe_inference.c:868-960,
 * 1215-1226, 1437-1440, 1485-1486, 1624, 1760-1830, 2335), then
 * gdn_layer_forward for a decode token and a 70-token prompt. */
static int engine_calls(void) {
    enum { H = 256, INNER = 256, GROUPS = 1, HD = 128, HV = INNER / HD, QKV = 2 * GROUPS * HD + INNER };
    CHECK(gpu_init() == 0);
    gpu_set_expert_limit(4);
    void* w_qkv = q8_0_blocks(QKV, H);
    void* w_gate = q8_0_blocks(INNER, H);
    void* w_out = q8_0_blocks(H, INNER);
    void* w_alpha = q8_0_blocks(HV, H);
    void* w_beta = q8_0_blocks(HV, H);
    CHECK(gpu_upload_deltanet_weights(0, w_qkv, H, QKV, w_gate, H, INNER, w_out, INNER, H) == 0);
    float* normed = floats(H, 1.0f, 0.0f);
    CHECK(gpu_launch_qkv_gate(0, 0, normed, H, QKV, INNER) == 0);
    CHECK(gpu_wait_qkv_gate(0) == 0);
    CHECK(gpu_get_qkv_out(0) != NULL && gpu_get_gate_out(0) != NULL);
    CHECK(isfinite(gpu_get_qkv_out(0)[QKV - 1]) && isfinite(gpu_get_gate_out(0)[INNER - 1]));
    float* gated = floats(INNER, 1.0f, 0.0f);
    CHECK(gpu_launch_ssm_out(0, 0, gated, INNER, H) == 0);
    CHECK(gpu_wait_ssm_out(0) == 0);
    CHECK(gpu_get_ssm_out_buf(0) != NULL && isfinite(gpu_get_ssm_out_buf(0)[H - 1]));
    CHECK(gpu_vram_used_mb() > 0.0f);

    void* wq = q8_0_blocks(2 * INNER, H);
    void* wk = q8_0_blocks(HD, H);
    void* wv = q8_0_blocks(HD, H);
    void* wo = q8_0_blocks(H, INNER);
    CHECK(gpu_upload_gqa_weights(1, wq, H, 2 * INNER, wk, H, HD, wv, H, HD, wo, INNER, H) == 0);
    float* qg = (float*)malloc(2 * INNER * sizeof(float));
    float* ko = (float*)malloc(HD * sizeof(float));
    float* vo = (float*)malloc(HD * sizeof(float));
    float* oo = (float*)malloc(H * sizeof(float));
    CHECK(gpu_gqa_projections(1, normed, H, qg, 2 * INNER, ko, HD, vo, HD) == 0);
    CHECK(gpu_gqa_output(1, gated, INNER, oo, H) == 0);

    /* the expert cache: the reference's own module (or its stand-in) */
    if (gpu_find_cached_expert(0, 3) < 0) {
        /* an expert of intermediate width H, all-zero blocks: gate and up Q4_K
         * [H][H / 256] (144 bytes each), down Q5_K [H][H / 256] (176 bytes each) */
        static unsigned char gu[H * (H / 256) * 144], dn[H * (H / 256) * 176];
        gpu_cache_expert(0, 3, gu, (int)sizeof(gu), gu, (int)sizeof(gu), dn, (int)sizeof(dn));
    }
    const int slot = gpu_find_cached_expert(0, 3);
    if (slot >= 0) {
        float* eo = (float*)malloc(H * sizeof(float));
        gpu_expert_ffn_fused(slot, normed, H, H, eo);
        free(eo);
    }

    /* the reference's layer call on the GPU: host weights, device activations and state */
    CHECK(gdn_dn_init_dims(INNER, GROUPS, HD) == 0);
    float* conv1d_w = floats(QKV * 4, 0.5f, 0.0f);
    float* a_log = floats(HV, 1.0f, -2.0f);
    float* dt_bias = floats(HV, 0.1f, 0.0f);
    float* head_norm = floats(HD, 0.1f, 1.0f);
    const int T = 70;
    float *d_x, *d_out, *d_S, *d_conv;
    int32_t* d_pos;
    CHECK(cudaMalloc((void**)&d_x, (size_t)T * H * 4) == cudaSuccess);
    CHECK(cudaMalloc((void**)&d_out, (size_t)T * H * 4) == cudaSuccess);
    CHECK(cudaMalloc((void**)&d_S, (size_t)HV * HD * HD * 4) == cudaSuccess);
    CHECK(cudaMalloc((void**)&d_conv, (size_t)4 * QKV * 4) == cudaSuccess);
    CHECK(cudaMalloc((void**)&d_pos, 4) == cudaSuccess);
    float* hx = floats(T * H, 1.0f, 0.0f);
    CHECK(cudaMemcpy(d_x, hx, (size_t)T * H * 4, cudaMemcpyHostToDevice) == cudaSuccess);
    CHECK(cudaMemset(d_S, 0, (size_t)HV * HD * HD * 4) == cudaSuccess);
    CHECK(cudaMemset(d_conv, 0, (size_t)4 * QKV * 4) == cudaSuccess);
    CHECK(cudaMemset(d_pos, 0, 4) == cudaSuccess);
    gdn_dn_state st = {d_S, d_conv, d_pos};
    CHECK(gdn_layer_forward(d_out, d_x, &st, w_qkv, GDN_GGML_Q8_0, w_gate, GDN_GGML_Q8_0, w_alpha, GDN_GGML_Q8_0,
                            w_beta, GDN_GGML_Q8_0, w_out, GDN_GGML_Q8_0, conv1d_w, a_log, dt_bias, head_norm, H, 1,
                            T, NULL) == GDN_OK);
    CHECK(gdn_layer_forward(d_out, d_x, &st, w_qkv, GDN_GGML_Q8_0, w_gate, GDN_GGML_Q8_0, w_alpha, GDN_GGML_Q8_0,
                            w_beta, GDN_GGML_Q8_0, w_out, GDN_GGML_Q8_0, conv1d_w, a_log, dt_bias, head_norm, H, 1,
                            1, NULL) == GDN_OK);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    float out[H];
    int32_t pos = 0;
    CHECK(cudaMemcpy(out, d_out, sizeof(out), cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(cudaMemcpy(&pos, d_pos, 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    for (int i = 0; i < H; i++) CHECK(isfinite(out[i]));
    CHECK(pos == T + 1);
    CHECK(gdn_check_device_error(NULL) == GDN_OK);
    CHECK(gdn_layer_release(w_qkv) == GDN_OK);
    CHECK(gdn_layer_release_all() == GDN_OK);
    gpu_shutdown();
    printf("engine calls ok\n");
    return 0;
}

int main(int argc, char** argv) {
    printf("experts_linked=%d abi=%d\n", gdn_offload_experts_linked(), gdn_abi_version());
    if (argc > 1 && strcmp(argv[1], "--run") == 0) return engine_calls();
    return 0;
}
