// gdn_layer_forward: the reference's layer call with its own argument list.
//
// The reference engine's CPU route calls
//   deltanet_forward(output, x, state, w_qkv, t, w_gate, t, w_alpha, t,
//                    w_beta, t, w_out, t, conv1d_w, a_log, dt_bias, head_norm, hidden)
// (engine/runtime/deltanet_impl.h:145-162, call site winmoe_inference.c:1450-1460)
// with raw GGUF blocks plus GGML type ids, dims set once by dn_init_dims
// (deltanet_impl.h:32-44), and a DeltaNetState it mutates in place.  This
// file keeps that call and adds batch, T and a stream: the weight set is
// prepared once (uploaded if it lives in host memory, the Q8_0 blocks
// repacked to planes, the five projections fused into the layer's in_proj)
// into module-owned device memory, as gpu_upload_deltanet_weights does for
// the offload API (engine/runtime/gpu_offload.cu:1041-1070); later calls with
// the same pointers reuse it.  The step itself is gdn_decode_step (T == 1) or
// gdn_prefill (T > 1, sequence by sequence) on a module-owned scratch.
#include <string.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <vector>

#include "gdn_common.cuh"
#include "quant.cuh"
#include "decode.cuh"
#include "prefill.cuh"

namespace gdn {
namespace {

constexpr int kMaxDevices = 64;

// dn_init_dims state (the reference keeps these as file statics; its defaults
// are the large model's: inner 8192, 16 key groups, head_dim 128).
struct DnDims {
    int inner = 8192, groups = 16, head_dim = 128;
} g_dims;

// One prepared weight set: its source pointers and types (the cache key) and
// the device copies in the layout of gdn_layer.
struct Prepared {
    int dev = -1;
    const void* src[5] = {};  // w_qkv, w_gate, w_alpha, w_beta, w_out
    int type[5] = {};
    const float* psrc[4] = {};  // conv1d_w, a_log, dt_bias, head_norm
    gdn_dims dims{};
    gdn_layer layer{};
    void* mem = nullptr;
    size_t bytes = 0;
};

struct Scratch {
    void* p = nullptr;
    size_t bytes = 0;
};

std::mutex g_mu;
std::vector<std::unique_ptr<Prepared>> g_prepared;  // entries never move: callers keep &layer
Scratch g_scratch[kMaxDevices];

// Device memory stays where it is; host memory (the engine's RAM copies of the
// GGUF tensors) is copied to `dst`.  Either way the bytes end up at `dst`.
int to_device(void* dst, const void* src, size_t bytes, cudaStream_t s) {
    GDN_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s));
    return GDN_OK;
}

bool is_device_ptr(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

size_t take(size_t& off, size_t bytes) {
    const size_t r = off;
    off += round_up(bytes, 256);
    return r;
}

int prepare(Prepared& P, cudaStream_t s) {
    const gdn_dims& d = P.dims;
    const int64_t H = d.hidden, hv = d.num_v_heads, key = (int64_t)d.num_k_heads * d.head_dim;
    const int64_t inner = hv * d.head_dim, qkv = 2 * key + inner, np = qkv + inner + 2 * hv;
    // rows of each source tensor inside the fused in_proj: qkv | gate (z) | beta | alpha
    const int64_t rows[4] = {qkv, inner, hv, hv};
    const int64_t row0[4] = {0, qkv, qkv + inner + hv, qkv + inner};  // src order: qkv, gate, alpha, beta
    const bool q8 = P.type[0] == GDN_GGML_Q8_0;
    const int64_t in_row_bytes = q8 ? H / 32 * 34 : H / 256 * 144;
    const int64_t out_row_bytes = q8 ? inner / 32 * 34 : inner / 256 * 144;

    size_t off = 0;
    size_t o_in_qs = 0, o_in_d = 0, o_out_qs = 0, o_out_d = 0, o_in_blk = 0, o_out_blk = 0;
    if (q8) {
        o_in_qs = take(off, (size_t)np * H);
        o_in_d = take(off, (size_t)np * (H / 32) * 2);
        o_out_qs = take(off, (size_t)H * inner);
        o_out_d = take(off, (size_t)H * (inner / 32) * 2);
    } else {
        o_in_blk = take(off, (size_t)np * in_row_bytes);
        o_out_blk = take(off, (size_t)H * out_row_bytes);
    }
    const size_t o_conv = take(off, (size_t)qkv * 4 * 4);
    const size_t o_a = take(off, (size_t)hv * 4), o_dt = take(off, (size_t)hv * 4), o_hn = take(off, (size_t)d.head_dim * 4);
    // Q8_0 blocks of host-memory tensors are staged here before the repack
    const size_t o_stage = take(off, q8 ? (size_t)std::max(qkv * in_row_bytes, H * out_row_bytes) : 0);
    GDN_CUDA(cudaMalloc(&P.mem, off));
    P.bytes = off;
    char* base = static_cast<char*>(P.mem);

    gdn_layer& L = P.layer;
    L = gdn_layer{};
    L.dims = d;
    L.weight_type = q8 ? GDN_GGML_Q8_0 : GDN_GGML_Q4_K;
    L.head_map = GDN_HEAD_MAP_GROUPED;  // deltanet_impl.h:280
    int st;
    if (q8) {
        int8_t* in_qs = reinterpret_cast<int8_t*>(base + o_in_qs);
        uint16_t* in_d = reinterpret_cast<uint16_t*>(base + o_in_d);
        for (int i = 0; i < 4; i++) {
            int8_t* qs = in_qs + row0[i] * H;
            uint16_t* dd = in_d + row0[i] * (H / 32);
            if (P.src[i] == nullptr) {  // the reference's memset: those raw projections are 0
                GDN_CUDA(cudaMemsetAsync(qs, 0, (size_t)rows[i] * H, s));
                GDN_CUDA(cudaMemsetAsync(dd, 0, (size_t)rows[i] * (H / 32) * 2, s));
                continue;
            }
            const void* blocks = P.src[i];
            if (!is_device_ptr(blocks)) {
                if ((st = to_device(base + o_stage, blocks, (size_t)rows[i] * in_row_bytes, s))) return st;
                blocks = base + o_stage;
            }
            if ((st = launch_q8_0_repack(blocks, qs, dd, rows[i], H, s))) return st;
        }
        const void* ob = P.src[4];
        if (!is_device_ptr(ob)) {
            if ((st = to_device(base + o_stage, ob, (size_t)H * out_row_bytes, s))) return st;
            ob = base + o_stage;
        }
        L.out_qs = reinterpret_cast<int8_t*>(base + o_out_qs);
        L.out_d = reinterpret_cast<uint16_t*>(base + o_out_d);
        if ((st = launch_q8_0_repack(ob, const_cast<int8_t*>(L.out_qs), const_cast<uint16_t*>(L.out_d), H, inner, s)))
            return st;
        L.in_qs = in_qs;
        L.in_d = in_d;
    } else {
        char* in_blk = base + o_in_blk;
        for (int i = 0; i < 4; i++) {
            char* dst = in_blk + row0[i] * in_row_bytes;
            if (P.src[i] == nullptr) {
                GDN_CUDA(cudaMemsetAsync(dst, 0, (size_t)rows[i] * in_row_bytes, s));
            } else if ((st = to_device(dst, P.src[i], (size_t)rows[i] * in_row_bytes, s))) {
                return st;
            }
        }
        if ((st = to_device(base + o_out_blk, P.src[4], (size_t)H * out_row_bytes, s))) return st;
        L.in_blocks = in_blk;
        L.out_blocks = base + o_out_blk;
    }
    const size_t pbytes[4] = {(size_t)qkv * 4 * 4, (size_t)hv * 4, (size_t)hv * 4, (size_t)d.head_dim * 4};
    const size_t poff[4] = {o_conv, o_a, o_dt, o_hn};
    const float** pdst[4] = {&L.conv1d_w, &L.ssm_a, &L.dt_bias, &L.head_norm};
    for (int i = 0; i < 4; i++) {
        if (P.psrc[i] == nullptr) {
            *pdst[i] = nullptr;  // the reference's NULL handling: no conv, decay 0.99, no norm weight
            continue;
        }
        if ((st = to_device(base + poff[i], P.psrc[i], pbytes[i], s))) return st;
        *pdst[i] = reinterpret_cast<const float*>(base + poff[i]);
    }
    // the staged host copies must land before the caller may free or reuse them
    GDN_CUDA(cudaStreamSynchronize(s));
    return GDN_OK;
}

// The prepared layer for this weight set on the current device (prepared now
// if it is new).  Called with g_mu held.
int find_or_prepare(const void* const* src, const int* type, const float* const* psrc, const gdn_dims& d,
                    cudaStream_t s, const gdn_layer** out) {
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    for (auto& up : g_prepared) {
        Prepared& P = *up;
        if (P.dev != dev || memcmp(&P.dims, &d, sizeof(d)) != 0) continue;
        bool same = true;
        for (int i = 0; i < 5 && same; i++) same = P.src[i] == src[i] && P.type[i] == type[i];
        for (int i = 0; i < 4 && same; i++) same = P.psrc[i] == psrc[i];
        if (same) {
            *out = &P.layer;
            return GDN_OK;
        }
    }
    auto owned = std::make_unique<Prepared>();
    Prepared& P = *owned;
    P.dev = dev;
    P.dims = d;
    for (int i = 0; i < 5; i++) {
        P.src[i] = src[i];
        P.type[i] = type[i];
    }
    for (int i = 0; i < 4; i++) P.psrc[i] = psrc[i];
    const int st = prepare(P, s);
    if (st) {
        if (P.mem) cudaFree(P.mem);
        return st;
    }
    *out = &P.layer;
    g_prepared.push_back(std::move(owned));
    return GDN_OK;
}

// The module's scratch on the current device, grown to `bytes` (the old one is
// freed once the device is idle: calls are stream-ordered, a smaller scratch
// may still be in use by queued work).
int scratch(size_t bytes, void** out, size_t* have) {
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(GDN_ERR_ARG, "device %d out of range", dev);
    Scratch& sc = g_scratch[dev];
    if (sc.bytes < bytes) {
        if (sc.p != nullptr) {
            GDN_CUDA(cudaDeviceSynchronize());
            GDN_CUDA(cudaFree(sc.p));
            sc = Scratch();
        }
        GDN_CUDA(cudaMalloc(&sc.p, bytes));
        sc.bytes = bytes;
    }
    *out = sc.p;
    *have = sc.bytes;
    return GDN_OK;
}

}  // namespace

// The reference's expert-cache module (engine/runtime/gpu_offload.cu) can be
// linked beside this library with its DeltaNet, GQA and lifetime functions
// renamed (include/gpu_offload_coexist.h).  When it is, these weak references
// resolve to its renamed gpu_init / gpu_shutdown / gpu_vram_used_mb, which the
// offload API here forwards to, so its streams and expert buffers exist when
// the engine calls gpu_cache_expert or gpu_expert_ffn_fused.
extern "C" int gdn_ref_offload_init(void) __attribute__((weak, visibility("default")));
extern "C" void gdn_ref_offload_shutdown(void) __attribute__((weak, visibility("default")));
extern "C" float gdn_ref_offload_vram_used_mb(void) __attribute__((weak, visibility("default")));

int ref_offload_init() { return gdn_ref_offload_init ? gdn_ref_offload_init() : 0; }
void ref_offload_shutdown() {
    if (gdn_ref_offload_shutdown) gdn_ref_offload_shutdown();
}
float ref_offload_vram_mb() { return gdn_ref_offload_vram_used_mb ? gdn_ref_offload_vram_used_mb() : 0.0f; }

}  // namespace gdn

using namespace gdn;

extern "C" {

int gdn_dn_init_dims(int ssm_inner_size, int ssm_group_count, int ssm_head_dim) {
    std::lock_guard<std::mutex> lock(g_mu);
    DnDims d;
    d.head_dim = ssm_head_dim > 0 ? ssm_head_dim : 128;
    d.groups = ssm_group_count > 0 ? ssm_group_count : 16;
    d.inner = ssm_inner_size > 0 ? ssm_inner_size : 8192;
    if (d.head_dim != 128 || d.inner % 128 != 0 || (d.inner / 128) % d.groups != 0)
        return fail(GDN_ERR_SHAPE, "dn_init_dims: head_dim must be 128 and inner / 128 a multiple of the groups "
                    "(got inner %d, groups %d, head_dim %d)", d.inner, d.groups, d.head_dim);
    g_dims = d;
    return GDN_OK;
}

int gdn_layer_forward(float* output, const float* x, gdn_dn_state* state, const void* w_qkv, int w_qkv_type,
                      const void* w_gate, int w_gate_type, const void* w_alpha, int w_alpha_type,
                      const void* w_beta, int w_beta_type, const void* w_out, int w_out_type,
                      const float* conv1d_w, const float* a_log, const float* dt_bias, const float* head_norm,
                      int hidden_dim, int64_t batch, int64_t T, void* stream) {
    if (!output || !x || !state || !state->S || !state->conv_pos || !w_qkv || !w_gate || !w_out)
        return fail(GDN_ERR_ARG, "layer_forward: output, x, state (S, conv_pos) and w_qkv / w_gate / w_out must be "
                    "non-NULL");
    if (batch < 1 || T < 1) return fail(GDN_ERR_SHAPE, "layer_forward: batch and T must be >= 1");
    if (batch > 1 && T > 1 && batch * T > ((int64_t)1 << 26))
        return fail(GDN_ERR_SHAPE, "layer_forward: batch x T too large");
    const int t0 = w_qkv_type;
    const int types[5] = {w_qkv_type, w_gate_type, w_alpha_type, w_beta_type, w_out_type};
    const void* src[5] = {w_qkv, w_gate, w_alpha, w_beta, w_out};
    if (t0 != GDN_GGML_Q8_0 && t0 != GDN_GGML_Q4_K)
        return fail(GDN_ERR_TYPE, "layer_forward: GGML type %d is not supported (8 = Q8_0, 12 = Q4_K)", t0);
    for (int i = 1; i < 5; i++)
        if (src[i] != nullptr && types[i] != t0)
            return fail(GDN_ERR_TYPE, "layer_forward: the five projections must share one GGML type (%d and %d)", t0,
                        types[i]);
    gdn_dims d;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        d.hidden = hidden_dim;
        d.num_k_heads = g_dims.groups;
        d.num_v_heads = g_dims.inner / g_dims.head_dim;
        d.head_dim = g_dims.head_dim;
    }
    if (hidden_dim <= 0 || hidden_dim % 256 != 0)
        return fail(GDN_ERR_SHAPE, "layer_forward: hidden_dim must be a positive multiple of 256 (got %d)", hidden_dim);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float* psrc[4] = {conv1d_w, a_log, dt_bias, head_norm};
    const gdn_layer* L = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int st;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if ((st = find_or_prepare(src, types, psrc, d, s, &L))) return st;
        const size_t need = T == 1 ? decode_workspace_bytes_for(*L, batch) : prefill_workspace_bytes(d, T);
        if ((st = scratch(need, &ws, &ws_bytes))) return st;
    }
    float* conv_buf = state->conv_buf;
    if (T == 1)
        return decode_step(L, batch, x, GDN_DTYPE_F32, output, state->S, conv_buf, state->conv_pos, ws, ws_bytes, s);
    const int64_t qkv = 2 * (int64_t)d.num_k_heads * d.head_dim + (int64_t)d.num_v_heads * d.head_dim;
    const int64_t s_elems = (int64_t)d.num_v_heads * d.head_dim * d.head_dim;
    for (int64_t b = 0; b < batch; b++) {
        st = prefill(L, T, x + b * T * hidden_dim, GDN_DTYPE_F32, output + b * T * hidden_dim, nullptr,
                     state->S + b * s_elems, conv_buf ? conv_buf + b * 4 * qkv : nullptr, state->conv_pos + b, ws,
                     ws_bytes, s);
        if (st) return st;
    }
    return GDN_OK;
}

int gdn_layer_release(const void* w_qkv) {
    std::lock_guard<std::mutex> lock(g_mu);
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    int n = 0;
    for (size_t i = 0; i < g_prepared.size();) {
        if (g_prepared[i]->dev == dev && g_prepared[i]->src[0] == w_qkv) {
            GDN_CUDA(cudaDeviceSynchronize());
            GDN_CUDA(cudaFree(g_prepared[i]->mem));
            g_prepared.erase(g_prepared.begin() + (std::ptrdiff_t)i);
            n++;
        } else {
            i++;
        }
    }
    return n > 0 ? GDN_OK : fail(GDN_ERR_ARG, "layer_release: no prepared layer for that w_qkv on this device");
}

int gdn_layer_release_all(void) {
    std::lock_guard<std::mutex> lock(g_mu);
    int dev = 0;
    GDN_CUDA(cudaGetDevice(&dev));
    GDN_CUDA(cudaDeviceSynchronize());
    for (size_t i = 0; i < g_prepared.size();) {
        if (g_prepared[i]->dev == dev) {
            GDN_CUDA(cudaFree(g_prepared[i]->mem));
            g_prepared.erase(g_prepared.begin() + (std::ptrdiff_t)i);
        } else {
            i++;
        }
    }
    if (dev >= 0 && dev < kMaxDevices && g_scratch[dev].p != nullptr) {
        GDN_CUDA(cudaFree(g_scratch[dev].p));
        g_scratch[dev] = Scratch();
    }
    return GDN_OK;
}

int gdn_offload_experts_linked(void) { return gdn_ref_offload_init != nullptr ? 1 : 0; }

}  // extern "C"
