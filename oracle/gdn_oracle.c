/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle.  Never linked into, loaded by, or
 * called from the product path (winmoe_b200/).  Only tests/,
 * __graft_entry__.smoke() and the cpu_baseline / --impl reference legs of
 * bench.py may load it, and there only as the checker or the timed baseline.
 *
 * A plain-C restatement (no intrinsics, no OpenMP) of the reference's CPU
 * Gated DeltaNet path and its GGUF quant kernels.  Each function names the
 * reference file:line it restates.  Where the reference reduces in a fixed
 * SIMD order, the same order is written out as scalar code, so this file and
 * the in-place reference build (oracle/_ref) agree bit for bit when both are
 * compiled with -ffp-contract=off.  That agreement is what pins this oracle:
 * tests/test_oracle_pin.py checks it live against oracle/_ref, and
 * tests/test_oracle_golden.py against fixtures that oracle/_ref produced.
 *
 * Activation modes for the projections (argument act_mode):
 *   0  "exact"  -- the reference CPU dispatch: a Q8_0 GEMV with out_dim >= 128
 *                  and in_dim >= 256 quantises x to Q8_K int8 first
 *                  (engine/runtime/q8_dequant.h:75-80); Q4_K always does.
 *   1  "fp32"   -- fp32 activations, the arithmetic of the reference GPU
 *                  kernels (engine/runtime/gpu_offload.cu:152-199, 206-268).
 * Head map (argument head_map):
 *   0  grouped     g = h / (Hv/Hk)   (engine/runtime/deltanet_impl.h:280)
 *   1  interleaved g = h % Hk        (engine/runtime/winmoe_inference.c:1330)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

#define QK8_0 32
#define Q8_0_BYTES 34
#define QK_K 256
#define Q4_K_BYTES 144
#define Q5_K_BYTES 176
#define Q8_K_BYTES 292 /* float d; int8 qs[256]; int16 bsums[16] */
#define CONV_W 4

/* ---------------------------------------------------------------- fp16 */

/* fp16_to_fp32: engine/runtime/iq2_dequant.h:22-40 (exact, subnormals included). */
EXPORT float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    float v;
    if (ex == 0) {
        if (man == 0) return sign ? -0.0f : 0.0f;
        v = ldexpf((float)man, -24);
        return sign ? -v : v;
    }
    if (ex == 0x1f) {
        if (man == 0) return sign ? -INFINITY : INFINITY;
        return NAN;
    }
    v = ldexpf((float)(man + 1024), (int)ex - 25);
    return sign ? -v : v;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ---------------------------------------------------------------- Q8_0 */

/* q8_dequant_row: engine/runtime/q8_dequant.h:116-126.  w = d * q, one rounding. */
EXPORT void orc_q8_0_dequant(float* out, const uint8_t* blocks, long n) {
    for (long b = 0; b < n / QK8_0; b++) {
        const uint8_t* blk = blocks + b * Q8_0_BYTES;
        float d = orc_fp16_to_fp32(rd16(blk));
        for (int j = 0; j < QK8_0; j++) out[b * QK8_0 + j] = d * (float)(int8_t)blk[2 + j];
    }
}

/* Horizontal sum of 16 lanes in the order of GCC's _mm512_reduce_add_ps. */
static float hsum16(const float* a) {
    float t3[8], t6[4];
    for (int i = 0; i < 8; i++) t3[i] = a[8 + i] + a[i];
    for (int i = 0; i < 4; i++) t6[i] = t3[4 + i] + t3[i];
    float t80 = t6[0] + t6[2], t81 = t6[1] + t6[3];
    return t80 + t81;
}

/* q8_dot_block: engine/runtime/q8_dequant.h:21-32 (two 16-lane FMAs, then reduce, then *d). */
static float q8_0_dot_fp32(const uint8_t* blk, const float* y) {
    float d = orc_fp16_to_fp32(rd16(blk));
    const int8_t* q = (const int8_t*)(blk + 2);
    float acc[16];
    for (int i = 0; i < 16; i++) acc[i] = fmaf((float)q[i], y[i], 0.0f);
    for (int i = 0; i < 16; i++) acc[i] = fmaf((float)q[16 + i], y[16 + i], acc[i]);
    return d * hsum16(acc);
}

/* quantize_block_q8_K: engine/runtime/q8k_quant.h:32-93.  Writes d, qs, bsums. */
static void quantize_block_q8_K(uint8_t* outb, const float* x) {
    float amax = 0.0f;
    for (int i = 0; i < QK_K; i++) {
        float a = fabsf(x[i]);
        amax = (a > amax) ? a : amax;
    }
    float* d_out = (float*)outb;
    int8_t* qs = (int8_t*)(outb + 4);
    int16_t* bs = (int16_t*)(outb + 4 + QK_K);
    if (amax < 1e-10f) {
        *d_out = 0.0f;
        memset(qs, 0, QK_K);
        memset(bs, 0, 32);
        return;
    }
    float d = amax / 127.0f;
    float id = 1.0f / d;
    *d_out = d;
    for (int i = 0; i < QK_K; i++) {
        long v = lrintf(x[i] * id); /* cvtps_epi32: round to nearest even */
        if (v < -127) v = -127;
        if (v > 127) v = 127;
        qs[i] = (int8_t)v;
    }
    for (int i = 0; i < 16; i++) {
        int16_t s = 0;
        for (int j = 0; j < 16; j++) s = (int16_t)(s + qs[i * 16 + j]);
        bs[i] = s;
    }
}

/* quantize_row_q8_K: engine/runtime/q8k_quant.h:99-104. */
EXPORT void orc_quantize_row_q8_K(uint8_t* out, const float* x, long n) {
    for (long b = 0; b < n / QK_K; b++) quantize_block_q8_K(out + b * Q8_K_BYTES, x + b * QK_K);
}

/* q8_dot_q8k: engine/runtime/q8_dequant.h:35-61.  The integer dot is exact and
 * every partial fits 24 bits, so the float horizontal sum is exact too. */
static float q8_0_dot_q8k(const uint8_t* blk, float a_d, const int8_t* a_q) {
    float d = orc_fp16_to_fp32(rd16(blk)) * a_d;
    const int8_t* q = (const int8_t*)(blk + 2);
    int32_t s = 0;
    for (int j = 0; j < QK8_0; j++) s += (int32_t)q[j] * (int32_t)a_q[j];
    return d * (float)s;
}

/* q8_matvec: engine/runtime/q8_dequant.h:63-113 (act_mode 0) or the per-row
 * fp32 dot of the GPU kernel (act_mode 1). */
EXPORT void orc_q8_0_matvec(float* out, const uint8_t* W, const float* x,
                            int out_dim, int in_dim, int act_mode) {
    int bpr = in_dim / QK8_0;
    int nk = in_dim / QK_K;
    uint8_t* xq = NULL;
    if (act_mode == 0 && nk > 0 && out_dim >= 128) {
        xq = (uint8_t*)malloc((size_t)nk * Q8_K_BYTES);
        orc_quantize_row_q8_K(xq, x, (long)nk * QK_K);
    }
    for (int r = 0; r < out_dim; r++) {
        const uint8_t* row = W + (size_t)r * bpr * Q8_0_BYTES;
        float sum = 0.0f;
        if (xq) {
            for (int qb = 0; qb < nk; qb++) {
                const uint8_t* kb = xq + (size_t)qb * Q8_K_BYTES;
                float ad = *(const float*)kb;
                for (int sb = 0; sb < 8; sb++) {
                    int bidx = qb * 8 + sb;
                    if (bidx < bpr)
                        sum += q8_0_dot_q8k(row + (size_t)bidx * Q8_0_BYTES, ad,
                                            (const int8_t*)(kb + 4 + sb * 32));
                }
            }
        } else {
            for (int b = 0; b < bpr; b++) sum += q8_0_dot_fp32(row + (size_t)b * Q8_0_BYTES, x + b * QK8_0);
        }
        out[r] = sum;
    }
    free(xq);
}

/* ---------------------------------------------------------------- Q4_K */

/* decode_q4k_scales: engine/runtime/q4k_dequant.h:43-60 (= gpu_get_scale_min,
 * engine/runtime/gpu_offload.cu:90-98). */
EXPORT void orc_q4_k_scales(const uint8_t* q, uint8_t* sc, uint8_t* mn) {
    for (int j = 0; j < 4; j++) {
        sc[j] = q[j] & 63;
        mn[j] = q[j + 4] & 63;
    }
    for (int j = 4; j < 8; j++) {
        sc[j] = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        mn[j] = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Q4_K float dequant in the GGML nibble layout, fp32 expression of
 * engine/runtime/gpu_offload.cu:237-250: chunk c, byte j -> low nibble is weight
 * 64c+j with (sc,m)[2c], high nibble is weight 64c+32+j with (sc,m)[2c+1];
 * w = (d*sc)*q - (dmin*m), each operation rounded once (no contraction). */
EXPORT void orc_q4_k_dequant(float* out, const uint8_t* blocks, long n) {
    for (long b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = blocks + b * Q4_K_BYTES;
        float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
        uint8_t sc[8], mn[8];
        orc_q4_k_scales(blk + 4, sc, mn);
        const uint8_t* qs = blk + 16;
        for (int c = 0; c < 4; c++) {
            float sl = d * (float)sc[2 * c], ml = dmin * (float)mn[2 * c];
            float sh = d * (float)sc[2 * c + 1], mh = dmin * (float)mn[2 * c + 1];
            for (int j = 0; j < 32; j++) {
                uint8_t p = qs[32 * c + j];
                float pl = sl * (float)(p & 0x0F), ph = sh * (float)(p >> 4);
                out[b * QK_K + 64 * c + j] = pl - ml;
                out[b * QK_K + 64 * c + 32 + j] = ph - mh;
            }
        }
    }
}

/* q4k_dot_q8k: engine/runtime/q4k_dequant.h:112-168.  Integer lane l of the
 * 8-lane accumulator holds bytes 4l..4l+3 of every 32-byte chunk (maddubs then
 * madd pair adjacent lanes); each lane is scaled by d, then reduced in the
 * order add(lo128, hi128), hadd, hadd. */
static float q4_k_dot_q8k(const uint8_t* blk, const uint8_t* kb) {
    float ad = *(const float*)kb;
    const int8_t* q8 = (const int8_t*)(kb + 4);
    const int16_t* bs = (const int16_t*)(kb + 4 + QK_K);
    float d = orc_fp16_to_fp32(rd16(blk)) * ad;
    float dmin = orc_fp16_to_fp32(rd16(blk + 2)) * ad;
    uint8_t sc[8], mn[8];
    orc_q4_k_scales(blk + 4, sc, mn);
    int32_t min_sum = 0;
    for (int s = 0; s < 8; s++) min_sum += (int32_t)mn[s] * (bs[2 * s] + bs[2 * s + 1]);
    const uint8_t* qs = blk + 16;
    int32_t lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < 4; c++) {
        for (int b = 0; b < 32; b++) {
            int l = b / 4;
            uint8_t p = qs[32 * c + b];
            lane[l] += (int32_t)sc[2 * c] * (int32_t)(p & 0x0F) * (int32_t)q8[64 * c + b];
            lane[l] += (int32_t)sc[2 * c + 1] * (int32_t)(p >> 4) * (int32_t)q8[64 * c + 32 + b];
        }
    }
    float v[8];
    for (int l = 0; l < 8; l++) v[l] = d * (float)lane[l];
    float s4[4];
    for (int i = 0; i < 4; i++) s4[i] = v[i] + v[4 + i];
    float h0 = s4[0] + s4[1], h1 = s4[2] + s4[3];
    float result = h0 + h1;
    return result - dmin * (float)min_sum;
}

/* Q4_K GEMV.  act_mode 0: q4k_matvec (engine/runtime/q4k_dequant.h:174-210),
 * Q8_K activations.  act_mode 1: fp32 activations, per-superblock sum of
 * w_lo*x + w_hi*x in the loop order of engine/runtime/gpu_offload.cu:222-250. */
EXPORT void orc_q4_k_matvec(float* out, const uint8_t* W, const float* x,
                            int out_dim, int in_dim, int act_mode) {
    int bpr = in_dim / QK_K;
    uint8_t* xq = NULL;
    if (act_mode == 0) {
        xq = (uint8_t*)malloc((size_t)bpr * Q8_K_BYTES);
        orc_quantize_row_q8_K(xq, x, (long)bpr * QK_K);
    }
    for (int r = 0; r < out_dim; r++) {
        const uint8_t* row = W + (size_t)r * bpr * Q4_K_BYTES;
        float sum = 0.0f;
        for (int b = 0; b < bpr; b++) {
            const uint8_t* blk = row + (size_t)b * Q4_K_BYTES;
            if (xq) {
                sum += q4_k_dot_q8k(blk, xq + (size_t)b * Q8_K_BYTES);
                continue;
            }
            float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
            uint8_t sc[8], mn[8];
            orc_q4_k_scales(blk + 4, sc, mn);
            float bsum = 0.0f;
            for (int c = 0; c < 4; c++) {
                float sl = d * (float)sc[2 * c], ml = dmin * (float)mn[2 * c];
                float sh = d * (float)sc[2 * c + 1], mh = dmin * (float)mn[2 * c + 1];
                for (int j = 0; j < 32; j++) {
                    uint8_t p = blk[16 + 32 * c + j];
                    float wl = sl * (float)(p & 0x0F) - ml;
                    float wh = sh * (float)(p >> 4) - mh;
                    bsum += wl * x[b * QK_K + 64 * c + j] + wh * x[b * QK_K + 64 * c + 32 + j];
                }
            }
            sum += bsum;
        }
        out[r] = sum;
    }
    free(xq);
}

/* ---------------------------------------------------------------- Q5_K */

/* The 5-bit value of weight 64c + j (low: half 0) or 64c + 32 + j (half 1) of a
 * Q5_K superblock in the GGML layout of engine/runtime/gpu_offload.cu:302-309
 * (and q5k_dot_q8k, q5k_dequant.h:103-128): the nibble of qs[32c + j] with bit
 * 2c + half of qh[j] as its fifth bit. */
static inline int q5_k_value(const uint8_t* blk, int c, int j, int half) {
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48;
    int nib = half ? (qs[32 * c + j] >> 4) : (qs[32 * c + j] & 0x0F);
    return nib | (((qh[j] >> (2 * c + half)) & 1) << 4);
}

/* Q5_K float dequant, fp32 expression of engine/runtime/gpu_offload.cu:302-309:
 * w = (d*sc)*q - (dmin*m), each operation rounded once. */
EXPORT void orc_q5_k_dequant(float* out, const uint8_t* blocks, long n) {
    for (long b = 0; b < n / QK_K; b++) {
        const uint8_t* blk = blocks + b * Q5_K_BYTES;
        float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
        uint8_t sc[8], mn[8];
        orc_q4_k_scales(blk + 4, sc, mn);
        for (int c = 0; c < 4; c++) {
            float sl = d * (float)sc[2 * c], ml = dmin * (float)mn[2 * c];
            float sh = d * (float)sc[2 * c + 1], mh = dmin * (float)mn[2 * c + 1];
            for (int j = 0; j < 32; j++) {
                float pl = sl * (float)q5_k_value(blk, c, j, 0), ph = sh * (float)q5_k_value(blk, c, j, 1);
                out[b * QK_K + 64 * c + j] = pl - ml;
                out[b * QK_K + 64 * c + 32 + j] = ph - mh;
            }
        }
    }
}

/* q5k_dot_q8k: engine/runtime/q5k_dequant.h:80-157, the same integer lanes as
 * Q4_K (lane l holds bytes 4l..4l+3 of every 32-byte chunk), then d times each
 * lane, reduced as add(lo128, hi128), hadd, hadd. */
static float q5_k_dot_q8k(const uint8_t* blk, const uint8_t* kb) {
    float ad = *(const float*)kb;
    const int8_t* q8 = (const int8_t*)(kb + 4);
    const int16_t* bs = (const int16_t*)(kb + 4 + QK_K);
    float d = orc_fp16_to_fp32(rd16(blk)) * ad;
    float dmin = orc_fp16_to_fp32(rd16(blk + 2)) * ad;
    uint8_t sc[8], mn[8];
    orc_q4_k_scales(blk + 4, sc, mn);
    int32_t min_sum = 0;
    for (int s = 0; s < 8; s++) min_sum += (int32_t)mn[s] * (bs[2 * s] + bs[2 * s + 1]);
    int32_t lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = 0; c < 4; c++) {
        for (int b = 0; b < 32; b++) {
            int l = b / 4;
            lane[l] += (int32_t)sc[2 * c] * (int32_t)q5_k_value(blk, c, b, 0) * (int32_t)q8[64 * c + b];
            lane[l] += (int32_t)sc[2 * c + 1] * (int32_t)q5_k_value(blk, c, b, 1) * (int32_t)q8[64 * c + 32 + b];
        }
    }
    float v[8];
    for (int l = 0; l < 8; l++) v[l] = d * (float)lane[l];
    float s4[4];
    for (int i = 0; i < 4; i++) s4[i] = v[i] + v[4 + i];
    float h0 = s4[0] + s4[1], h1 = s4[2] + s4[3];
    float result = h0 + h1;
    return result - dmin * (float)min_sum;
}

/* Q5_K GEMV.  act_mode 0: q5k_matvec (engine/runtime/q5k_dequant.h:160-195),
 * Q8_K activations.  act_mode 1: fp32 activations, per-superblock sum of
 * w_lo*x + w_hi*x in the loop order of engine/runtime/gpu_offload.cu:296-317. */
EXPORT void orc_q5_k_matvec(float* out, const uint8_t* W, const float* x,
                            int out_dim, int in_dim, int act_mode) {
    int bpr = in_dim / QK_K;
    uint8_t* xq = NULL;
    if (act_mode == 0) {
        xq = (uint8_t*)malloc((size_t)bpr * Q8_K_BYTES);
        orc_quantize_row_q8_K(xq, x, (long)bpr * QK_K);
    }
    for (int r = 0; r < out_dim; r++) {
        const uint8_t* row = W + (size_t)r * bpr * Q5_K_BYTES;
        float sum = 0.0f;
        for (int b = 0; b < bpr; b++) {
            const uint8_t* blk = row + (size_t)b * Q5_K_BYTES;
            if (xq) {
                sum += q5_k_dot_q8k(blk, xq + (size_t)b * Q8_K_BYTES);
                continue;
            }
            float d = orc_fp16_to_fp32(rd16(blk)), dmin = orc_fp16_to_fp32(rd16(blk + 2));
            uint8_t sc[8], mn[8];
            orc_q4_k_scales(blk + 4, sc, mn);
            float bsum = 0.0f;
            for (int c = 0; c < 4; c++) {
                float sl = d * (float)sc[2 * c], ml = dmin * (float)mn[2 * c];
                float sh = d * (float)sc[2 * c + 1], mh = dmin * (float)mn[2 * c + 1];
                for (int j = 0; j < 32; j++) {
                    float wl = sl * (float)q5_k_value(blk, c, j, 0) - ml;
                    float wh = sh * (float)q5_k_value(blk, c, j, 1) - mh;
                    bsum += wl * x[b * QK_K + 64 * c + j] + wh * x[b * QK_K + 64 * c + 32 + j];
                }
            }
            sum += bsum;
        }
        out[r] = sum;
    }
    free(xq);
}

/* ------------------------------------------------------------ projection */

/* quant_matvec dispatch: engine/runtime/transformer.h:157-194, types 8 (Q8_0),
 * 12 (Q4_K) and 13 (Q5_K); any other type is read as fp32 rows. */
EXPORT void orc_quant_matvec(float* out, const void* W, const float* x,
                             int out_dim, int in_dim, int type, int act_mode) {
    if (type == 8) {
        orc_q8_0_matvec(out, (const uint8_t*)W, x, out_dim, in_dim, act_mode);
    } else if (type == 12) {
        orc_q4_k_matvec(out, (const uint8_t*)W, x, out_dim, in_dim, act_mode);
    } else if (type == 13) {
        orc_q5_k_matvec(out, (const uint8_t*)W, x, out_dim, in_dim, act_mode);
    } else {
        const float* wf = (const float*)W;
        for (int r = 0; r < out_dim; r++) {
            float s = 0.0f;
            for (int c = 0; c < in_dim; c++) s += wf[(size_t)r * in_dim + c] * x[c];
            out[r] = s;
        }
    }
}

/* One expert's FFN for one token, the fused GPU route of
 * engine/runtime/gpu_offload.cu:718-751 (gpu_expert_ffn_fused): gate and up
 * projections (hidden -> inter), SwiGLU act = (g * sigmoid(g)) * up with
 * sigmoid = 1 / (1 + expf(-g)) (swiglu_kernel, gpu_offload.cu:460-466), then the
 * down projection (inter -> hidden).  `weight` scales the result into out
 * (accumulate != 0: out += weight * y, gpu_offload.cu:469-471 and 785-789;
 * else out = y). */
EXPORT void orc_expert_ffn(float* out, const float* x, const void* w_gate, const void* w_up, const void* w_down,
                           int gate_type, int down_type, int hidden, int inter, float weight, int accumulate,
                           int act_mode) {
    float* g = (float*)malloc((size_t)inter * sizeof(float));
    float* u = (float*)malloc((size_t)inter * sizeof(float));
    float* y = (float*)malloc((size_t)hidden * sizeof(float));
    orc_quant_matvec(g, w_gate, x, inter, hidden, gate_type, act_mode);
    orc_quant_matvec(u, w_up, x, inter, hidden, gate_type, act_mode);
    for (int i = 0; i < inter; i++) {
        float sig = 1.0f / (1.0f + expf(-g[i]));
        g[i] = (g[i] * sig) * u[i];
    }
    orc_quant_matvec(y, w_down, g, hidden, inter, down_type, act_mode);
    for (int i = 0; i < hidden; i++) out[i] = accumulate ? out[i] + weight * y[i] : y[i];
    free(g);
    free(u);
    free(y);
}

/* ------------------------------------------------------------ GDN helpers */

/* softplus_stable / sigmoid_stable: engine/runtime/deltanet_impl.h:103-115. */
static float softplus_stable(float x) { return log1pf(expf(-fabsf(x))) + fmaxf(x, 0.0f); }
static float sigmoid_stable(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    float z = expf(x);
    return z / (1.0f + z);
}

/* dn_l2norm: engine/runtime/deltanet_impl.h:85-91 (double sum, no 1/sqrt(d)). */
static void l2norm(float* x, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    float inv = 1.0f / (sqrtf((float)ss) + 1e-6f);
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* rmsnorm: engine/runtime/attention.h:29-44 (the pre-layer norm of the stack).
 * The reference scales x*scale then *w in 8-wide vectors; scalar order is the same. */
EXPORT void orc_rmsnorm(float* out, const float* x, const float* w, int dim) {
    double ss = 0.0;
    for (int i = 0; i < dim; i++) ss += (double)x[i] * (double)x[i];
    float scale = 1.0f / sqrtf((float)(ss / dim) + 1e-6f);
    for (int i = 0; i < dim; i++) out[i] = (x[i] * scale) * w[i];
}

/* Dimensions, derived as dn_init_dims does (engine/runtime/deltanet_impl.h:32-44). */
typedef struct {
    int hidden, hd, hk, hv, hpg, key, inner, qkv;
} dims_t;

static dims_t make_dims(int hidden, int inner, int groups, int head_dim) {
    dims_t d;
    d.hidden = hidden;
    d.hd = head_dim > 0 ? head_dim : 128;
    d.hk = groups > 0 ? groups : 16;
    d.inner = inner > 0 ? inner : 8192;
    d.hv = d.inner / d.hd;
    d.hpg = d.hv / d.hk;
    d.key = d.hk * d.hd;
    d.qkv = 2 * d.key + d.inner;
    return d;
}

/*
 * The layer between the projections and out_proj, for one token of one
 * sequence: deltanet_impl.h:218-371.
 *   qkv [QKV] raw projection (overwritten with conv+SiLU, then L2-normed q/k);
 *   z [INNER]; alpha_raw, beta_raw [Hv]; S [Hv][d][d] (row = k index,
 *   col = v index); conv_buf [4][QKV] with *conv_pos.
 *   gated [INNER] receives normed * silu(z), the input of out_proj.
 *   decay_out / beta_out [Hv] (optional) receive the per-head gates;
 *   head_out [INNER] (optional) the pre-norm head outputs.
 */
EXPORT void orc_gdn_core(int hidden, int inner, int groups, int head_dim, int head_map,
                         float* qkv, const float* z, const float* alpha_raw, const float* beta_raw,
                         float* S, float* conv_buf, int* conv_pos,
                         const float* conv1d_w, const float* ssm_a, const float* dt_bias,
                         const float* head_norm, float* gated,
                         float* decay_out, float* beta_out, float* head_out) {
    dims_t D = make_dims(hidden, inner, groups, head_dim);
    int hd = D.hd;
    /* conv1d + SiLU: deltanet_impl.h:218-236 (k=0 oldest ... k=3 newest). */
    if (conv_buf && conv1d_w) {
        int slot = *conv_pos % CONV_W;
        memcpy(conv_buf + (size_t)slot * D.qkv, qkv, sizeof(float) * D.qkv);
        *conv_pos += 1;
        for (int i = 0; i < D.qkv; i++) {
            float sum = 0.0f;
            for (int k = 0; k < CONV_W; k++) {
                int hs = ((*conv_pos - CONV_W + k) % CONV_W + CONV_W) % CONV_W;
                sum += conv1d_w[(size_t)i * CONV_W + k] * conv_buf[(size_t)hs * D.qkv + i];
            }
            float sig = 1.0f / (1.0f + expf(-sum));
            qkv[i] = sum * sig;
        }
    }
    float* Q = qkv;
    float* K = qkv + D.key;
    float* V = qkv + 2 * D.key;
    /* gates: deltanet_impl.h:247-261. */
    float* decay = (float*)malloc(sizeof(float) * D.hv);
    float* beta = (float*)malloc(sizeof(float) * D.hv);
    for (int h = 0; h < D.hv; h++) {
        float a = (ssm_a && dt_bias) ? expf(ssm_a[h] * softplus_stable(alpha_raw[h] + dt_bias[h])) : 0.99f;
        if (a > 1.0f) a = 1.0f;
        if (a < 0.0f) a = 0.0f;
        if (isnan(a)) a = 0.99f;
        decay[h] = a;
        beta[h] = sigmoid_stable(beta_raw[h]);
        if (decay_out) decay_out[h] = a;
        if (beta_out) beta_out[h] = beta[h];
    }
    /* L2 norm of q and k per key head: deltanet_impl.h:264-267. */
    for (int g = 0; g < D.hk; g++) {
        l2norm(Q + g * hd, hd);
        l2norm(K + g * hd, hd);
    }
    /* recurrence: deltanet_impl.h:279-348. */
    float* ho = (float*)calloc((size_t)D.inner, sizeof(float));
    float scale = 1.0f / sqrtf((float)hd);
    float* ret = (float*)malloc(sizeof(float) * hd);
    float* delta = (float*)malloc(sizeof(float) * hd);
    float* acc = (float*)malloc(sizeof(float) * hd);
    for (int h = 0; h < D.hv; h++) {
        int g = head_map ? (h % D.hk) : (h / D.hpg);
        float* Sh = S + (size_t)h * hd * hd;
        const float* k = K + g * hd;
        const float* v = V + h * hd;
        const float* q = Q + g * hd;
        float dg = decay[h], b = beta[h];
        for (int c = 0; c < hd; c++) ret[c] = 0.0f;
        for (int r = 0; r < hd; r++) {
            float* row = Sh + (size_t)r * hd;
            for (int c = 0; c < hd; c++) {
                row[c] = row[c] * dg;
                ret[c] = fmaf(k[r], row[c], ret[c]);
            }
        }
        for (int c = 0; c < hd; c++) delta[c] = b * (v[c] - ret[c]);
        for (int r = 0; r < hd; r++) {
            float* row = Sh + (size_t)r * hd;
            for (int c = 0; c < hd; c++) row[c] = fmaf(k[r], delta[c], row[c]);
        }
        for (int c = 0; c < hd; c++) acc[c] = 0.0f;
        for (int r = 0; r < hd; r++) {
            const float* row = Sh + (size_t)r * hd;
            for (int c = 0; c < hd; c++) acc[c] = fmaf(q[r], row[c], acc[c]);
        }
        for (int c = 0; c < hd; c++) ho[h * hd + c] = acc[c] * scale;
    }
    if (head_out) memcpy(head_out, ho, sizeof(float) * D.inner);
    /* per-head RMSNorm (deltanet_impl.h:350-361) and SiLU(z) gate (364-371). */
    for (int h = 0; h < D.hv; h++) {
        const float* o = ho + h * hd;
        double ss = 0.0;
        for (int i = 0; i < hd; i++) ss += (double)o[i] * (double)o[i];
        float inv = 1.0f / sqrtf((float)(ss / hd) + 1e-6f);
        for (int i = 0; i < hd; i++) {
            float nv = head_norm ? (o[i] * inv) * head_norm[i] : o[i] * inv;
            float zv = z[h * hd + i];
            if (zv > 88.0f) zv = 88.0f;
            if (zv < -88.0f) zv = -88.0f;
            gated[h * hd + i] = nv * (zv / (1.0f + expf(-zv)));
        }
    }
    free(ret); free(delta); free(acc); free(ho); free(decay); free(beta);
}

/*
 * One token of deltanet_forward (engine/runtime/deltanet_impl.h:145-377) for one
 * sequence: projections (189-196), orc_gdn_core, out_proj (374).
 * Weight types are GGML ids (8 = Q8_0, 12 = Q4_K); w_alpha / w_beta may be NULL
 * (then the raw gates are zero, deltanet_impl.h:192-196).
 */
EXPORT void orc_deltanet_forward(int hidden, int inner, int groups, int head_dim,
                                 int act_mode, int head_map,
                                 float* out, const float* x, float* S, float* conv_buf, int* conv_pos,
                                 const void* w_qkv, int t_qkv, const void* w_gate, int t_gate,
                                 const void* w_alpha, int t_alpha, const void* w_beta, int t_beta,
                                 const void* w_out, int t_out, const float* conv1d_w,
                                 const float* ssm_a, const float* dt_bias, const float* head_norm) {
    dims_t D = make_dims(hidden, inner, groups, head_dim);
    float* qkv = (float*)malloc(sizeof(float) * D.qkv);
    float* z = (float*)malloc(sizeof(float) * D.inner);
    float* ar = (float*)calloc((size_t)D.hv, sizeof(float));
    float* br = (float*)calloc((size_t)D.hv, sizeof(float));
    float* gated = (float*)malloc(sizeof(float) * D.inner);
    orc_quant_matvec(qkv, w_qkv, x, D.qkv, hidden, t_qkv, act_mode);
    orc_quant_matvec(z, w_gate, x, D.inner, hidden, t_gate, act_mode);
    if (w_alpha) orc_quant_matvec(ar, w_alpha, x, D.hv, hidden, t_alpha, act_mode);
    if (w_beta) orc_quant_matvec(br, w_beta, x, D.hv, hidden, t_beta, act_mode);
    orc_gdn_core(hidden, inner, groups, head_dim, head_map, qkv, z, ar, br, S, conv_buf, conv_pos,
                 conv1d_w, ssm_a, dt_bias, head_norm, gated, NULL, NULL, NULL);
    orc_quant_matvec(out, w_out, gated, hidden, D.inner, t_out, act_mode);
    free(qkv); free(z); free(ar); free(br); free(gated);
}
