/*
 * TEST INFRASTRUCTURE ONLY -- never linked into, loaded by, or called from the
 * product path (winmoe_b200/).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load the library built
 * from this file, and there only as the checker or the timed CPU baseline.
 *
 * Oracle mode "ref-exact": the reference engine's own CPU Gated DeltaNet path,
 * compiled IN PLACE from the reference tree (REF_DIR/engine/runtime, passed with
 * -I by oracle/Makefile; no reference source is copied into this repository).
 *
 * The include order follows engine/runtime/winmoe_inference.c:24-30,119-122, so
 * quant_matvec is the unmodified dispatch of engine/runtime/transformer.h:157-194:
 * Q8_0 projections with out_dim >= 128 quantise the activation to Q8_K (int8)
 * first (engine/runtime/q8_dequant.h:77-80).
 *
 * The only additions are the MSVC spellings the headers use, mapped to their
 * POSIX equivalents, and the C-ABI wrappers below (prefix refx_).
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
#define _fseeki64 fseeko
#define _ftelli64 ftello

/* engine/runtime/q6k_dequant.h:143 declares this extern; the engine's main sets it. */
int g_q6k_use_scalar = 0;

#include "iq2xxs_grid_def.h"
#include "iq2_dequant.h"
#include "q8k_quant.h"
#include "q4k_dequant.h"
#include "q5k_dequant.h"
#include "q6k_dequant.h"
#include "q8_dequant.h"
#include "gguf_parser.h"
#include "transformer.h"
#include "deltanet_impl.h"

#define EXPORT __attribute__((visibility("default")))

/* dn_init_dims (engine/runtime/deltanet_impl.h:32-44).  Returns the QKV width. */
EXPORT int refx_init_dims(int inner, int groups, int head_dim) {
    dn_init_dims(inner, groups, head_dim);
    return DN_QKV_DIM;
}

/*
 * One token of deltanet_forward (engine/runtime/deltanet_impl.h:145-377) for one
 * sequence.  S [Hv][d][d] and conv_buf [4][QKV] are the caller's buffers and are
 * updated in place, as DeltaNetState (deltanet_impl.h:48-60) would be;
 * *conv_pos is the circular-window position (deltanet_impl.h:220-222).
 */
EXPORT void refx_deltanet_forward(
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

/* quant_matvec (engine/runtime/transformer.h:157-194), unmodified dispatch. */
EXPORT void refx_quant_matvec(float* out, const void* W, const float* x,
                              int out_dim, int in_dim, int type) {
    quant_matvec(out, W, x, out_dim, in_dim, type);
}

/* q8_dequant_row (engine/runtime/q8_dequant.h:116-126). */
EXPORT void refx_q8_dequant_row(float* out, const void* data, int n) {
    q8_dequant_row(out, data, n);
}

/* quantize_row_q8_K (engine/runtime/q8k_quant.h:99-104); out holds n/256 blocks of 292 bytes. */
EXPORT int refx_q8k_block_bytes(void) { return (int)sizeof(block_q8_K); }
EXPORT void refx_quantize_row_q8_K(void* out, const float* x, int n) {
    quantize_row_q8_K((block_q8_K*)out, x, n);
}

/* decode_q4k_scales (engine/runtime/q4k_dequant.h:43-60). */
EXPORT void refx_decode_q4k_scales(const uint8_t* q, uint8_t* scales, uint8_t* mins) {
    decode_q4k_scales(q, scales, mins);
}

/* q4k_matvec (engine/runtime/q4k_dequant.h:174-210): Q8_K activations, integer dot. */
EXPORT void refx_q4k_matvec(float* out, const void* W, const float* x, int out_dim, int in_dim) {
    q4k_matvec(out, W, x, out_dim, in_dim);
}

/* q4k_dot_block (engine/runtime/q4k_dequant.h:69-105): the float fallback with its own nibble order. */
EXPORT float refx_q4k_dot_block(const void* block, const float* y) {
    return q4k_dot_block((const block_q4_K*)block, y);
}

/* fp16_to_fp32 (engine/runtime/iq2_dequant.h:22-40). */
EXPORT float refx_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }

/* rmsnorm (engine/runtime/attention.h:29-44): the pre-layer norm. */
EXPORT void refx_rmsnorm(float* out, const float* x, const float* w, int dim) {
    rmsnorm(out, x, w, dim);
}

/* parse_gguf / find_tensor (engine/runtime/gguf_parser.h:149-250, 350-358) on a
 * file: the reference's own reading of a GGUF, to check files written and read
 * by winmoe_b200.gguf.  meta: n_tensors, hidden, ssm inner, groups, state size,
 * conv kernel, layers, data_start.  info: type, n_dims, dims[4], offset. */
EXPORT int refx_gguf_probe(const char* path, long long* meta) {
    GGUFModel* m = (GGUFModel*)calloc(1, sizeof(GGUFModel));
    if (!m) return -2;
    int rc = parse_gguf(path, m);
    if (rc == 0) {
        meta[0] = (long long)m->n_tensors;
        meta[1] = m->hidden_dim;
        meta[2] = m->ssm_inner_size;
        meta[3] = m->ssm_group_count;
        meta[4] = m->ssm_state_size;
        meta[5] = m->ssm_conv_kernel;
        meta[6] = m->num_layers;
        meta[7] = (long long)m->data_start;
    }
    free(m);
    return rc;
}

EXPORT int refx_gguf_tensor(const char* path, const char* name, long long* info) {
    GGUFModel* m = (GGUFModel*)calloc(1, sizeof(GGUFModel));
    if (!m) return -2;
    int rc = parse_gguf(path, m);
    if (rc == 0) {
        TensorInfo* t = find_tensor(m, name);
        if (!t) {
            rc = -3;
        } else {
            info[0] = t->type;
            info[1] = t->n_dims;
            for (int d = 0; d < 4; d++) info[2 + d] = (long long)t->dims[d];
            info[6] = (long long)t->offset;
        }
    }
    free(m);
    return rc;
}
