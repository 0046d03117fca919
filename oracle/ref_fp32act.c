/*
 * TEST INFRASTRUCTURE ONLY -- never linked into, loaded by, or called from the
 * product path (winmoe_b200/).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load the library built
 * from this file, and there only as the checker or the timed CPU baseline.
 *
 * Oracle mode "ref-fp32act": the reference's deltanet_forward
 * (engine/runtime/deltanet_impl.h:145-377), compiled IN PLACE from the reference
 * tree, with the projection dispatch replaced by fp32-activation GEMVs.  That is
 * the arithmetic of the reference's own GPU route:
 *   - Q8_0: every row is a sum of q8_dot_block (engine/runtime/q8_dequant.h:21-32)
 *     over its 32-blocks, the per-row semantics of q8_matvec_kernel
 *     (engine/runtime/gpu_offload.cu:152-199) -- no Q8_K activation quantisation;
 *   - Q4_K: the float dequant w = (d*sc)*q - (dmin*m) of q4k_matvec_kernel
 *     (engine/runtime/gpu_offload.cu:237-250) against fp32 activations;
 *   - Q5_K: the same with the fifth bit from qh, q5k_matvec_kernel
 *     (engine/runtime/gpu_offload.cu:296-317).
 * Everything else in the layer (conv1d, gates, L2-norm, recurrence, RMSNorm,
 * SiLU gate) is the reference's code, unmodified.
 *
 * transformer.h is deliberately not included: this file defines the static
 * quant_matvec that deltanet_impl.h calls.
 */
#define _GNU_SOURCE
#include <alloca.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define _malloca(n) alloca(n)
#define _freea(p) ((void)(p))
#define _isnan(x) isnan(x)

#include "iq2xxs_grid_def.h"
#include "iq2_dequant.h"
#include "q8k_quant.h"
#include "q4k_dequant.h"
#include "q5k_dequant.h"
#include "q8_dequant.h"

#define EXPORT __attribute__((visibility("default")))

/* One Q4_K row with fp32 activations, following gpu_offload.cu:222-250 (per
 * 256-superblock: for chunk c and byte j, w_lo*x[64c+j] + w_hi*x[64c+32+j]). */
static float q4k_row_fp32act(const block_q4_K* row, const float* x, int nblk) {
    float total = 0.0f;
    for (int b = 0; b < nblk; b++) {
        const block_q4_K* blk = &row[b];
        float d = fp16_to_fp32(blk->d), dmin = fp16_to_fp32(blk->dmin);
        uint8_t sc[8], mn[8];
        decode_q4k_scales(blk->scales, sc, mn);
        float bs = 0.0f;
        for (int c = 0; c < 4; c++) {
            float sc_lo = d * (float)sc[2 * c], mn_lo = dmin * (float)mn[2 * c];
            float sc_hi = d * (float)sc[2 * c + 1], mn_hi = dmin * (float)mn[2 * c + 1];
            for (int j = 0; j < 32; j++) {
                uint8_t p = blk->qs[32 * c + j];
                float w_lo = sc_lo * (float)(p & 0x0F) - mn_lo;
                float w_hi = sc_hi * (float)(p >> 4) - mn_hi;
                bs += w_lo * x[b * 256 + 64 * c + j] + w_hi * x[b * 256 + 64 * c + 32 + j];
            }
        }
        total += bs;
    }
    return total;
}

/* One Q5_K row with fp32 activations, following gpu_offload.cu:296-317. */
static float q5k_row_fp32act(const block_q5_K* row, const float* x, int nblk) {
    float total = 0.0f;
    for (int b = 0; b < nblk; b++) {
        const block_q5_K* blk = &row[b];
        float d = fp16_to_fp32(blk->d), dmin = fp16_to_fp32(blk->dmin);
        uint8_t sc[8], mn[8];
        decode_q4k_scales(blk->scales, sc, mn);
        float bs = 0.0f;
        for (int c = 0; c < 4; c++) {
            float sc_lo = d * (float)sc[2 * c], mn_lo = dmin * (float)mn[2 * c];
            float sc_hi = d * (float)sc[2 * c + 1], mn_hi = dmin * (float)mn[2 * c + 1];
            for (int j = 0; j < 32; j++) {
                uint8_t p = blk->qs[32 * c + j];
                int q_lo = (p & 0x0F) | (((blk->qh[j] >> (2 * c)) & 1) << 4);
                int q_hi = (p >> 4) | (((blk->qh[j] >> (2 * c + 1)) & 1) << 4);
                float w_lo = sc_lo * (float)q_lo - mn_lo;
                float w_hi = sc_hi * (float)q_hi - mn_hi;
                bs += w_lo * x[b * 256 + 64 * c + j] + w_hi * x[b * 256 + 64 * c + 32 + j];
            }
        }
        total += bs;
    }
    return total;
}

static void quant_matvec(float* out, const void* W, const float* x,
                         int out_dim, int in_dim, int type) {
    if (type == 8) {
        const block_q8_0* blocks = (const block_q8_0*)W;
        int bpr = in_dim / 32;
        for (int r = 0; r < out_dim; r++) {
            float sum = 0.0f;
            for (int b = 0; b < bpr; b++) sum += q8_dot_block(&blocks[(size_t)r * bpr + b], &x[b * 32]);
            out[r] = sum;
        }
    } else if (type == 12) {
        const block_q4_K* blocks = (const block_q4_K*)W;
        int bpr = in_dim / 256;
        for (int r = 0; r < out_dim; r++) out[r] = q4k_row_fp32act(&blocks[(size_t)r * bpr], x, bpr);
    } else if (type == 13) {
        const block_q5_K* blocks = (const block_q5_K*)W;
        int bpr = in_dim / 256;
        for (int r = 0; r < out_dim; r++) out[r] = q5k_row_fp32act(&blocks[(size_t)r * bpr], x, bpr);
    } else {
        const float* wf = (const float*)W;
        for (int r = 0; r < out_dim; r++) {
            float s = 0.0f;
            for (int c = 0; c < in_dim; c++) s += wf[(size_t)r * in_dim + c] * x[c];
            out[r] = s;
        }
    }
}

#include "deltanet_impl.h"

EXPORT int reff_init_dims(int inner, int groups, int head_dim) {
    dn_init_dims(inner, groups, head_dim);
    return DN_QKV_DIM;
}

/* One token of deltanet_forward for one sequence; see ref_exact.c for the buffers. */
EXPORT void reff_deltanet_forward(
    float* out, const float* x, float* S, float* conv_buf, int* conv_pos,
    const void* w_qkv, int w_qkv_type, const void* w_gate, int w_gate_type,
    const void* w_alpha, int w_alpha_type, const void* w_beta, int w_beta_type,
    const void* w_out, int w_out_type, const float* conv1d_w,
    const float* ssm_a, const float* dt_bias, const float* head_norm, int hidden) {
    DeltaNetState st;
    st.S = S;
    st.conv_buf = conv_buf;
    st.conv_pos = *conv_pos;
    st.tmp_qkv = (float*)malloc(sizeof(float) * DN_QKV_DIM);
    st.tmp_z = (float*)malloc(sizeof(float) * DN_GATE_DIM);
    st.tmp_alpha = (float*)malloc(sizeof(float) * DN_NUM_GATES);
    st.tmp_beta = (float*)malloc(sizeof(float) * DN_NUM_GATES);
    st.tmp_head_out = (float*)calloc(DN_INNER, sizeof(float));
    st.tmp_normed = (float*)malloc(sizeof(float) * DN_INNER);
    st.tmp_gated = (float*)malloc(sizeof(float) * DN_INNER);
    deltanet_forward(out, x, &st, w_qkv, w_qkv_type, w_gate, w_gate_type,
                     w_alpha, w_alpha_type, w_beta, w_beta_type, w_out, w_out_type,
                     conv1d_w, ssm_a, dt_bias, head_norm, hidden);
    *conv_pos = st.conv_pos;
    free(st.tmp_qkv); free(st.tmp_z); free(st.tmp_alpha); free(st.tmp_beta);
    free(st.tmp_head_out); free(st.tmp_normed); free(st.tmp_gated);
}

/* The fp32-activation projection used above, exported for GEMV parity tests. */
EXPORT void reff_quant_matvec(float* out, const void* W, const float* x,
                              int out_dim, int in_dim, int type) {
    quant_matvec(out, W, x, out_dim, in_dim, type);
}
