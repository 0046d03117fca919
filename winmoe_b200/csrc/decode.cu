// Decode step of the Gated DeltaNet layer for a batch of independent sequences.
//
//   proj  = in_proj(x)                   [B][QKV | inner | Hv (beta) | Hv (alpha)]
//   prep  : conv1d window + SiLU, L2-norm of q/k heads, decay/beta gates
//   state : S <- decay*S; r = S^T k; delta = beta (v - r); S += k delta^T;
//           o = S^T q / sqrt(d); per-head RMSNorm * w; * SiLU(z)  -> gated
//   out   = out_proj(gated)
//
// Reference: deltanet_forward, engine/runtime/deltanet_impl.h:145-377
// (conv 218-236, gates 247-261, L2 264-267, recurrence 279-348, norm 350-361,
// gate 364-371, out_proj 374).
//
// The state kernel is the HBM-bound part: every (sequence, value head) owns a
// 128x128 fp32 state (64 KiB) that is read once and written once per token.
#include "gdn_common.cuh"
#include "quant.cuh"
#include "decode.cuh"

namespace gdn {

constexpr int HD = 128;  // head_dim (the reference's AVX loops assume 128 too)

// --------------------------------------------------------------- prep kernel
//
// grid (QKV/128, B), block 128: block x covers channels [128x, 128x+128) of the
// qkv vector -- one q head, one k head or one v head.  Channel c of sequence b:
//   window slot p%4 <- raw projection; out = sum_k w[c][k] * window[(p+1-4+k)%4]
//   (k = 0 oldest, k = 3 the value just stored), then SiLU.
// q/k heads are then L2-normalised with a double-precision sum of squares.
// The block of value head h also computes the gates of head h.
__global__ void __launch_bounds__(128) gdn_prep_kernel(const float* __restrict__ proj, int64_t proj_stride,
                                                       float* __restrict__ act, float* __restrict__ gates,
                                                       float* __restrict__ conv_buf, const int32_t* __restrict__ conv_pos,
                                                       const float* __restrict__ conv_w, const float* __restrict__ ssm_a,
                                                       const float* __restrict__ dt_bias, int qkv, int key_dim,
                                                       int hv) {
    const int b = blockIdx.y;
    const int ch = blockIdx.x * HD + threadIdx.x;
    const float* pr = proj + (int64_t)b * proj_stride;
    float xv = pr[ch];
    if (conv_w != nullptr && conv_buf != nullptr) {
        const int p = conv_pos[b];
        float* win = conv_buf + (int64_t)b * 4 * qkv;
        win[(int64_t)(p & 3) * qkv + ch] = xv;
        const float4 w = reinterpret_cast<const float4*>(conv_w)[ch];
        const float wk[4] = {w.x, w.y, w.z, w.w};
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int slot = (p - 3 + k) & 3;  // (p+1-4+k) mod 4
            const float hv_ = (k == 3) ? xv : win[(int64_t)slot * qkv + ch];
            sum = __fadd_rn(sum, __fmul_rn(wk[k], hv_));
        }
        const float sig = 1.0f / (1.0f + expf(-sum));
        xv = __fmul_rn(sum, sig);
    }
    if (ch < 2 * key_dim) {
        // L2 norm over the 128 channels of this q or k head (deltanet_impl.h:85-91).
        __shared__ double red[4];
        double ss = (double)xv * (double)xv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        ss = red[0] + red[1] + red[2] + red[3];
        const float inv = 1.0f / (sqrtf((float)ss) + 1e-6f);
        xv = __fmul_rn(xv, inv);
    } else if (threadIdx.x == 0) {
        const int h = (ch - 2 * key_dim) / HD;
        if (h < hv) {
            const float beta_raw = pr[qkv + hv * HD + h];
            const float alpha_raw = pr[qkv + hv * HD + hv + h];
            float a = 0.99f;
            if (ssm_a != nullptr && dt_bias != nullptr) {
                const float x = alpha_raw + dt_bias[h];
                const float sp = log1pf(expf(-fabsf(x))) + fmaxf(x, 0.0f);
                a = expf(ssm_a[h] * sp);
            }
            a = (a > 1.0f) ? 1.0f : a;
            a = (a < 0.0f) ? 0.0f : a;
            if (isnan(a)) a = 0.99f;
            float bt;
            if (beta_raw >= 0.0f) {
                bt = 1.0f / (1.0f + expf(-beta_raw));
            } else {
                const float z = expf(beta_raw);
                bt = z / (1.0f + z);
            }
            gates[(int64_t)b * 2 * hv + h] = a;
            gates[(int64_t)b * 2 * hv + hv + h] = bt;
        }
    }
    act[(int64_t)b * qkv + ch] = xv;
}

// -------------------------------------------------------------- state kernel
//
// grid (Hv, B), block 256 = 8 warps.  Warp w owns state rows [16w, 16w+16),
// lane l owns columns [4l, 4l+4): 16 float4 registers per thread, so each warp
// load/store instruction moves one full 512-byte state row.
__global__ void __launch_bounds__(256, 2) gdn_state_kernel(
    const float* __restrict__ act, const float* __restrict__ gates, const float* __restrict__ proj,
    int64_t proj_stride, float* __restrict__ S, const float* __restrict__ head_norm, float* __restrict__ gated,
    __half* __restrict__ gated_h, int32_t* __restrict__ conv_pos, int bump_conv, int qkv, int key_dim, int hv,
    int hk, int head_map) {
    const int h = blockIdx.x, b = blockIdx.y;
    const int t = threadIdx.x, w = t >> 5, l = t & 31;
    const int hpg = hv / hk;
    const int g = head_map ? (h % hk) : (h / hpg);

    __shared__ float sq[HD], sk[HD], sv[HD], sdelta[HD];
    __shared__ float red[8][HD];
    __shared__ double dred[4];

    float* Sh = S + ((int64_t)b * hv + h) * HD * HD;
    const float4* Sv = reinterpret_cast<const float4*>(Sh);
    float4 s[16];
#pragma unroll
    for (int i = 0; i < 16; i++) s[i] = Sv[(16 * w + i) * (HD / 4) + l];

    const float* a = act + (int64_t)b * qkv;
    if (t < HD) {
        sq[t] = a[g * HD + t];
        sk[t] = a[key_dim + g * HD + t];
        sv[t] = a[2 * key_dim + h * HD + t];
    }
    const float dg = gates[(int64_t)b * 2 * hv + h];
    const float bt = gates[(int64_t)b * 2 * hv + hv + h];
    __syncthreads();

    // decay + retrieve (deltanet_impl.h:298-307)
    float4 rp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float kr = sk[16 * w + i];
        s[i].x = __fmul_rn(s[i].x, dg);
        s[i].y = __fmul_rn(s[i].y, dg);
        s[i].z = __fmul_rn(s[i].z, dg);
        s[i].w = __fmul_rn(s[i].w, dg);
        rp.x = fmaf(kr, s[i].x, rp.x);
        rp.y = fmaf(kr, s[i].y, rp.y);
        rp.z = fmaf(kr, s[i].z, rp.z);
        rp.w = fmaf(kr, s[i].w, rp.w);
    }
    reinterpret_cast<float4*>(red[w])[l] = rp;
    __syncthreads();
    if (t < HD) {
        float r = 0.0f;
#pragma unroll
        for (int ww = 0; ww < 8; ww++) r += red[ww][t];
        sdelta[t] = __fmul_rn(bt, __fsub_rn(sv[t], r));  // deltanet_impl.h:311-317
    }
    __syncthreads();

    // update + output read (deltanet_impl.h:320-347)
    const float4 dl = reinterpret_cast<const float4*>(sdelta)[l];
    float4 op = make_float4(0.f, 0.f, 0.f, 0.f);
    float4* So = reinterpret_cast<float4*>(Sh);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        const float kr = sk[16 * w + i];
        const float qr = sq[16 * w + i];
        s[i].x = fmaf(kr, dl.x, s[i].x);
        s[i].y = fmaf(kr, dl.y, s[i].y);
        s[i].z = fmaf(kr, dl.z, s[i].z);
        s[i].w = fmaf(kr, dl.w, s[i].w);
        op.x = fmaf(qr, s[i].x, op.x);
        op.y = fmaf(qr, s[i].y, op.y);
        op.z = fmaf(qr, s[i].z, op.z);
        op.w = fmaf(qr, s[i].w, op.w);
        So[(16 * w + i) * (HD / 4) + l] = s[i];
    }
    __syncthreads();  // every warp is done with red[] from the retrieve pass
    reinterpret_cast<float4*>(red[w])[l] = op;
    __syncthreads();

    // output, per-head RMSNorm (deltanet_impl.h:350-361) and SiLU(z) gate (364-371)
    float o = 0.0f;
    if (t < HD) {
        for (int ww = 0; ww < 8; ww++) o += red[ww][t];
        o = __fmul_rn(o, 0.08838834764831845f);  // 1/sqrt(128), as 1.0f/sqrtf(128.0f)
        double ss = (double)o * (double)o;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (l == 0) dred[w] = ss;
    }
    __syncthreads();
    if (t < HD) {
        const double ss = dred[0] + dred[1] + dred[2] + dred[3];
        const float inv = 1.0f / sqrtf((float)(ss / HD) + 1e-6f);
        float nv = __fmul_rn(o, inv);
        if (head_norm != nullptr) nv = __fmul_rn(nv, head_norm[t]);
        float zv = proj[(int64_t)b * proj_stride + qkv + h * HD + t];
        zv = fminf(fmaxf(zv, -88.0f), 88.0f);
        const float gv = __fmul_rn(nv, zv / (1.0f + expf(-zv)));
        const int64_t idx = (int64_t)b * hv * HD + h * HD + t;
        if (gated != nullptr) gated[idx] = gv;
        if (gated_h != nullptr) gated_h[idx] = __float2half_rn(gv);
    }
    if (bump_conv && h == 0 && t == 0) conv_pos[b] += 1;
}

// ---------------------------------------------------------------- the step

size_t decode_workspace_bytes(const gdn_dims& d, int64_t batch) {
    const int64_t hv = d.num_v_heads, key = (int64_t)d.num_k_heads * d.head_dim, inner = hv * d.head_dim;
    const int64_t qkv = 2 * key + inner, np = qkv + inner + 2 * hv;
    size_t bytes = 0;
    bytes += round_up((size_t)batch * np * 4, 256);     // proj
    bytes += round_up((size_t)batch * qkv * 4, 256);    // act
    bytes += round_up((size_t)batch * 2 * hv * 4, 256); // gates
    bytes += round_up((size_t)batch * inner * 4, 256);  // gated fp32
    bytes += round_up((size_t)batch * inner * 2, 256);  // gated fp16 (tensor-core out_proj)
    bytes += round_up((size_t)batch * d.hidden * 2, 256); // x fp16 (tensor-core in_proj)
    return bytes;
}

int validate_layer(const gdn_layer* L) {
    if (L == nullptr) return fail(GDN_ERR_ARG, "layer is NULL");
    const gdn_dims& d = L->dims;
    if (d.head_dim != HD) return fail(GDN_ERR_SHAPE, "head_dim must be 128 (got %d)", d.head_dim);
    if (d.num_k_heads <= 0 || d.num_v_heads <= 0 || d.num_v_heads % d.num_k_heads != 0)
        return fail(GDN_ERR_SHAPE, "num_v_heads (%d) must be a positive multiple of num_k_heads (%d)",
                    d.num_v_heads, d.num_k_heads);
    if (d.hidden <= 0 || d.hidden % 256 != 0) return fail(GDN_ERR_SHAPE, "hidden must be a positive multiple of 256 (got %d)", d.hidden);
    if (L->head_map != GDN_HEAD_MAP_GROUPED && L->head_map != GDN_HEAD_MAP_INTERLEAVED)
        return fail(GDN_ERR_ARG, "head_map must be 0 or 1 (got %d)", L->head_map);
    if (L->weight_type == GDN_GGML_Q8_0) {
        if (!L->in_qs || !L->in_d || !L->out_qs || !L->out_d) return fail(GDN_ERR_ARG, "Q8_0 weight planes are NULL");
        if (!aligned(L->in_qs, 16) || !aligned(L->out_qs, 16)) return fail(GDN_ERR_ARG, "Q8_0 qs planes must be 16-byte aligned");
    } else if (L->weight_type == GDN_GGML_Q4_K) {
        if (!L->in_blocks || !L->out_blocks) return fail(GDN_ERR_ARG, "Q4_K weight blocks are NULL");
        if (!aligned(L->in_blocks, 16) || !aligned(L->out_blocks, 16)) return fail(GDN_ERR_ARG, "Q4_K blocks must be 16-byte aligned");
    } else {
        return fail(GDN_ERR_TYPE, "weight_type %d is not supported (8 = Q8_0, 12 = Q4_K)", L->weight_type);
    }
    if (L->conv1d_w && !aligned(L->conv1d_w, 16)) return fail(GDN_ERR_ARG, "conv1d_w must be 16-byte aligned");
    return GDN_OK;
}

// ----------------------------------------------------------- phase timing

namespace {
constexpr int kPhases = 4;
struct PhaseEvents {
    bool on = false;
    bool created = false;
    cudaEvent_t ev[kPhases + 1];
};
PhaseEvents g_phase[64];

PhaseEvents* phase_events() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    return g_phase[dev].on ? &g_phase[dev] : nullptr;
}

inline int mark(PhaseEvents* pe, int i, cudaStream_t s) {
    if (pe) GDN_CUDA(cudaEventRecord(pe->ev[i], s));
    return GDN_OK;
}
}  // namespace

int profile_enable(int on) {
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(GDN_ERR_ARG, "device %d out of range", dev);
    PhaseEvents& pe = g_phase[dev];
    if (on && !pe.created) {
        for (int i = 0; i <= kPhases; i++) GDN_CUDA(cudaEventCreate(&pe.ev[i]));
        pe.created = true;
    }
    pe.on = on != 0;
    return GDN_OK;
}

int phase_ms(float* ms, int n) {
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || !g_phase[dev].created) return fail(GDN_ERR_STATE, "profiling was never enabled");
    PhaseEvents& pe = g_phase[dev];
    GDN_CUDA(cudaEventSynchronize(pe.ev[kPhases]));
    int w = 0;
    for (int i = 0; i < kPhases && i < n; i++, w++) GDN_CUDA(cudaEventElapsedTime(&ms[i], pe.ev[i], pe.ev[i + 1]));
    return w;
}

// Tensor-core projections pay off once a batch fills an M=128 tile reasonably.
constexpr int64_t kTcMinBatch = 64;

static int project(const gdn_layer* L, bool in, const void* x, int x_dtype, __half* x_h, int64_t m, float* y,
                   cudaStream_t s) {
    const gdn_dims& d = L->dims;
    const int64_t inner = (int64_t)d.num_v_heads * d.head_dim;
    const int64_t qkv = 2 * (int64_t)d.num_k_heads * d.head_dim + inner;
    const int64_t n = in ? qkv + inner + 2 * d.num_v_heads : d.hidden;
    const int64_t k = in ? d.hidden : inner;
    if (L->weight_type == GDN_GGML_Q4_K)
        return launch_q4_k_gemv(in ? L->in_blocks : L->out_blocks, n, k, x, x_dtype, m, y, s);
    const int8_t* qs = in ? L->in_qs : L->out_qs;
    const uint16_t* dd = in ? L->in_d : L->out_d;
    if (m >= kTcMinBatch && k % 64 == 0) {
        const __half* a = static_cast<const __half*>(x);
        if (x_dtype != GDN_DTYPE_F16) {
            int st = launch_to_f16(x, x_dtype, x_h, m * k, s);
            if (st) return st;
            a = x_h;
        }
        return launch_q8_0_gemm_tc(qs, dd, n, k, a, m, y, s);
    }
    return launch_q8_0_gemv(qs, dd, n, k, x, x_dtype, m, y, s);
}

int decode_step(const gdn_layer* L, int64_t B, const void* x, int x_dtype, float* out, float* S, float* conv_buf,
                int32_t* conv_pos, void* ws, size_t ws_bytes, cudaStream_t s) {
    int st = validate_layer(L);
    if (st) return st;
    if (B <= 0 || B > 65535) return fail(GDN_ERR_SHAPE, "batch must be in [1, 65535] (got %lld)", (long long)B);
    if (!x || !out || !S || !conv_pos) return fail(GDN_ERR_ARG, "x, out, S and conv_pos must be non-NULL");
    if (x_dtype != GDN_DTYPE_F32 && x_dtype != GDN_DTYPE_BF16 && x_dtype != GDN_DTYPE_F16)
        return fail(GDN_ERR_TYPE, "x_dtype %d is not supported", x_dtype);
    if (!aligned(S, 16)) return fail(GDN_ERR_ARG, "S must be 16-byte aligned");
    const gdn_dims& d = L->dims;
    const size_t need = decode_workspace_bytes(d, B);
    if (ws == nullptr || ws_bytes < need || !aligned(ws, 256))
        return fail(GDN_ERR_ARG, "workspace must be 256-aligned and hold %zu bytes (got %zu)", need, ws_bytes);
    const int hv = d.num_v_heads, hk = d.num_k_heads;
    const int key = hk * HD, inner = hv * HD, qkv = 2 * key + inner;
    const int64_t np = (int64_t)qkv + inner + 2 * hv;

    char* p = static_cast<char*>(ws);
    float* proj = reinterpret_cast<float*>(p); p += round_up((size_t)B * np * 4, 256);
    float* act = reinterpret_cast<float*>(p); p += round_up((size_t)B * qkv * 4, 256);
    float* gates = reinterpret_cast<float*>(p); p += round_up((size_t)B * 2 * hv * 4, 256);
    float* gated = reinterpret_cast<float*>(p); p += round_up((size_t)B * inner * 4, 256);
    __half* gated_h = reinterpret_cast<__half*>(p); p += round_up((size_t)B * inner * 2, 256);
    __half* x_h = reinterpret_cast<__half*>(p);

    const bool tc_out = (L->weight_type == GDN_GGML_Q8_0) && B >= kTcMinBatch;
    PhaseEvents* pe = phase_events();

    if ((st = mark(pe, 0, s))) return st;
    st = project(L, true, x, x_dtype, x_h, B, proj, s);
    if (st) return st;
    if ((st = mark(pe, 1, s))) return st;
    const bool conv = (L->conv1d_w != nullptr && conv_buf != nullptr);
    gdn_prep_kernel<<<dim3(qkv / HD, (unsigned)B), HD, 0, s>>>(proj, np, act, gates, conv ? conv_buf : nullptr, conv_pos,
                                                               conv ? L->conv1d_w : nullptr, L->ssm_a, L->dt_bias, qkv,
                                                               key, hv);
    GDN_LAUNCH_CHECK("gdn_prep_kernel");
    if ((st = mark(pe, 2, s))) return st;
    gdn_state_kernel<<<dim3(hv, (unsigned)B), 256, 0, s>>>(act, gates, proj, np, S, L->head_norm,
                                                          tc_out ? nullptr : gated, tc_out ? gated_h : nullptr,
                                                          conv_pos, conv ? 1 : 0, qkv, key, hv, hk, L->head_map);
    GDN_LAUNCH_CHECK("gdn_state_kernel");
    if ((st = mark(pe, 3, s))) return st;
    st = tc_out ? project(L, false, gated_h, GDN_DTYPE_F16, nullptr, B, out, s)
                : project(L, false, gated, GDN_DTYPE_F32, nullptr, B, out, s);
    if (st) return st;
    return mark(pe, 4, s);
}

}  // namespace gdn
