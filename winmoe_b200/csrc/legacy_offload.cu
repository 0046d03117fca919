// The reference engine's DeltaNet and GQA offload API (engine/runtime/
// gpu_offload.h:19-67), re-implemented on this library's kernels so that the
// engine (engine/runtime/winmoe_inference.c:868, 938-942, 956-960, 1215-1226,
// 1437-1440, 1485-1486, 1624) can link against it unchanged.
//
// Kept from the reference (gpu_offload.cu:997-1209): one host thread; module
// state; weights copied to module-owned device memory at upload; three
// streams (compute, H2D, D2H); pinned double-buffered slots; async
// launch/wait pairs whose results stay valid in the slot until the next launch
// on it; 0 = ok, -1 = error (detail in gdn_last_error()).
// Different by design: the GPU is the current device (cudaSetDevice is left to
// the caller, one process per GPU); Q8_0 weights are stored as planes
// (gdn_q8_0_repack) and multiplied by this library's GEMV; the pinned slots
// are sized from the uploaded dims instead of fixed 8192/16384-float buffers;
// async launch errors are checked.
#include <stdio.h>
#include <string.h>
#include <vector>

#include "gdn_common.cuh"
#include "quant.cuh"
#include "../../include/gpu_offload_gdn.h"

namespace gdn {

// The reference's expert-cache module, when linked beside this library with
// its lifetime functions renamed (layer_api.cu): initialised, shut down and
// counted together with this module; no-ops when it is not linked.
int ref_offload_init();
void ref_offload_shutdown();
float ref_offload_vram_mb();

namespace {

constexpr int kMaxLayers = 256;
constexpr int kSlots = 2;

struct Proj {
    int8_t* qs = nullptr;
    uint16_t* d = nullptr;
    int in_dim = 0, out_dim = 0;
};

struct LayerGPU {
    Proj qkv, gate, out;
    bool loaded = false;
    // A full-attention (GQA) layer: Q+gate, K and V share their input and are
    // stored as one [q_gate + k + v][hidden] projection (one GEMV per call); O.
    Proj wqkv, wo;
    int q_dim = 0, k_dim = 0, v_dim = 0;
    bool gqa_loaded = false;
};

// Staging of the synchronous GQA calls: pinned input, device input, device and
// pinned outputs (grown on demand).
struct GqaIO {
    float *h_in = nullptr, *d_in = nullptr, *h_out = nullptr, *d_out = nullptr;
    size_t cap_in = 0, cap_out = 0;
};

struct Slot {
    float *h_normed = nullptr, *h_qkv = nullptr, *h_gate = nullptr, *h_gated = nullptr, *h_ssm = nullptr;
    float *d_normed = nullptr, *d_qkv = nullptr, *d_gate = nullptr, *d_gated = nullptr, *d_ssm = nullptr;
    cudaEvent_t ev_h2d_normed{}, ev_qkv_gate{}, ev_d2h_qkv_gate{}, ev_h2d_gated{}, ev_ssm{}, ev_d2h_ssm{};
    size_t cap_in = 0, cap_qkv = 0, cap_gate = 0, cap_gated = 0, cap_out = 0;  // float capacities
};

struct Module {
    bool initialized = false;
    LayerGPU layers[kMaxLayers];
    Slot slots[kSlots];
    GqaIO gqa;
    cudaStream_t compute{}, h2d{}, d2h{};
    double vram_bytes = 0;
} g;

int legacy(int st) { return st == GDN_OK ? 0 : -1; }

void free_proj(Proj& p) {
    if (p.qs) cudaFree(p.qs);
    if (p.d) cudaFree(p.d);
    p = Proj();
}

// Uploads the row blocks parts[i] (out_dims[i] rows of in_dim Q8_0 weights
// each, GGUF bytes) one after the other as a single projection.
int upload_rows(Proj& p, const void* const* parts, const int* out_dims, int nparts, int in_dim) {
    int out_dim = 0;
    for (int i = 0; i < nparts; i++) {
        if (out_dims[i] <= 0) return fail(GDN_ERR_SHAPE, "upload: out_dim %d", out_dims[i]);
        out_dim += out_dims[i];
    }
    if (in_dim <= 0 || in_dim % 32 != 0)
        return fail(GDN_ERR_SHAPE, "upload: in_dim must be a positive multiple of 32 (got %d x %d)", in_dim, out_dim);
    free_proj(p);
    const size_t nb = (size_t)in_dim / 32 * out_dim;
    void* raw = nullptr;
    GDN_CUDA(cudaMalloc(&raw, nb * 34));
    cudaError_t e = cudaSuccess;
    size_t off = 0;
    for (int i = 0; i < nparts && e == cudaSuccess; i++) {
        const size_t bytes = (size_t)in_dim / 32 * out_dims[i] * 34;
        e = cudaMemcpy(static_cast<char*>(raw) + off, parts[i], bytes, cudaMemcpyHostToDevice);
        off += bytes;
    }
    if (e == cudaSuccess) e = cudaMalloc(&p.qs, nb * 32);
    if (e == cudaSuccess) e = cudaMalloc(&p.d, nb * 2);
    if (e != cudaSuccess) {
        cudaFree(raw);
        free_proj(p);
        return cuda_status(e, "upload");
    }
    int st = launch_q8_0_repack(raw, p.qs, p.d, out_dim, in_dim, 0);
    cudaError_t e2 = cudaDeviceSynchronize();
    cudaFree(raw);
    if (st) return st;
    if (e2 != cudaSuccess) return cuda_status(e2, "upload repack");
    p.in_dim = in_dim;
    p.out_dim = out_dim;
    g.vram_bytes += (double)nb * 34;
    return GDN_OK;
}

int upload_proj(Proj& p, const void* host_blocks, int in_dim, int out_dim) {
    return upload_rows(p, &host_blocks, &out_dim, 1, in_dim);
}

// Grows a slot's pinned + device buffer pair to at least `count` floats.
int ensure(float** h, float** dv, size_t* cap, size_t count) {
    if (*cap >= count) return GDN_OK;
    if (*h) cudaFreeHost(*h);
    if (*dv) cudaFree(*dv);
    *h = nullptr;
    *dv = nullptr;
    *cap = 0;
    GDN_CUDA(cudaMallocHost(reinterpret_cast<void**>(h), count * sizeof(float)));
    GDN_CUDA(cudaMalloc(reinterpret_cast<void**>(dv), count * sizeof(float)));
    *cap = count;
    return GDN_OK;
}

int check_slot(int slot) {
    if (!g.initialized) return fail(GDN_ERR_STATE, "gpu_init has not been called");
    if (slot < 0 || slot >= kSlots) return fail(GDN_ERR_ARG, "slot %d out of range", slot);
    return GDN_OK;
}

int check_layer(int layer) {
    if (!g.initialized) return fail(GDN_ERR_STATE, "gpu_init has not been called");
    if (layer < 0 || layer >= kMaxLayers || !g.layers[layer].loaded)
        return fail(GDN_ERR_STATE, "layer %d has no uploaded DeltaNet weights", layer);
    return GDN_OK;
}

int check_gqa(int layer) {
    if (!g.initialized) return fail(GDN_ERR_STATE, "gpu_init has not been called");
    if (layer < 0 || layer >= kMaxLayers || !g.layers[layer].gqa_loaded)
        return fail(GDN_ERR_STATE, "layer %d has no uploaded GQA weights", layer);
    return GDN_OK;
}

int check_dims(const Proj& p, const char* name, int in_dim, int out_dim) {
    if (p.in_dim != in_dim || p.out_dim != out_dim)
        return fail(GDN_ERR_SHAPE, "%s: called with %d -> %d, uploaded as %d -> %d", name, in_dim, out_dim, p.in_dim,
                    p.out_dim);
    return GDN_OK;
}

// x (host, in_dim floats) through projection p on the compute stream; its
// out_dim results go to the host buffers outs[i] (splits[i] floats each, in
// order).  Returns after the copies are done (the reference's calls are
// synchronous).
int gqa_run(const Proj& p, float* const* outs, const int* splits, int n, const float* x, int in_dim) {
    GqaIO& io = g.gqa;
    int st = ensure(&io.h_in, &io.d_in, &io.cap_in, (size_t)in_dim);
    if (!st) st = ensure(&io.h_out, &io.d_out, &io.cap_out, (size_t)p.out_dim);
    if (st) return st;
    memcpy(io.h_in, x, sizeof(float) * in_dim);
    GDN_CUDA(cudaMemcpyAsync(io.d_in, io.h_in, sizeof(float) * in_dim, cudaMemcpyHostToDevice, g.compute));
    if ((st = launch_q8_0_gemv(p.qs, p.d, p.out_dim, p.in_dim, io.d_in, GDN_DTYPE_F32, 1, io.d_out, p.out_dim,
                               g.compute)))
        return st;
    GDN_CUDA(cudaMemcpyAsync(io.h_out, io.d_out, sizeof(float) * p.out_dim, cudaMemcpyDeviceToHost, g.compute));
    GDN_CUDA(cudaStreamSynchronize(g.compute));
    size_t off = 0;
    for (int i = 0; i < n; i++) {
        memcpy(outs[i], io.h_out + off, sizeof(float) * splits[i]);
        off += (size_t)splits[i];
    }
    return GDN_OK;
}

int launch_qkv_gate(int layer, int si, const float* normed, int hidden, int qkv_dim, int gate_dim) {
    int st = check_layer(layer);
    if (!st) st = check_slot(si);
    if (st) return st;
    LayerGPU& L = g.layers[layer];
    if (hidden != L.qkv.in_dim || qkv_dim != L.qkv.out_dim || gate_dim != L.gate.out_dim)
        return fail(GDN_ERR_SHAPE, "dims (%d, %d, %d) differ from the uploaded weights (%d, %d, %d)", hidden, qkv_dim,
                    gate_dim, L.qkv.in_dim, L.qkv.out_dim, L.gate.out_dim);
    Slot& s = g.slots[si];
    if ((st = ensure(&s.h_normed, &s.d_normed, &s.cap_in, hidden))) return st;
    if ((st = ensure(&s.h_qkv, &s.d_qkv, &s.cap_qkv, qkv_dim))) return st;
    if ((st = ensure(&s.h_gate, &s.d_gate, &s.cap_gate, gate_dim))) return st;
    memcpy(s.h_normed, normed, sizeof(float) * hidden);
    GDN_CUDA(cudaMemcpyAsync(s.d_normed, s.h_normed, sizeof(float) * hidden, cudaMemcpyHostToDevice, g.h2d));
    GDN_CUDA(cudaEventRecord(s.ev_h2d_normed, g.h2d));
    GDN_CUDA(cudaStreamWaitEvent(g.compute, s.ev_h2d_normed, 0));
    if ((st = launch_q8_0_gemv(L.qkv.qs, L.qkv.d, qkv_dim, hidden, s.d_normed, GDN_DTYPE_F32, 1, s.d_qkv, qkv_dim, g.compute)))
        return st;
    if ((st = launch_q8_0_gemv(L.gate.qs, L.gate.d, gate_dim, hidden, s.d_normed, GDN_DTYPE_F32, 1, s.d_gate,
                               gate_dim, g.compute)))
        return st;
    GDN_CUDA(cudaEventRecord(s.ev_qkv_gate, g.compute));
    GDN_CUDA(cudaStreamWaitEvent(g.d2h, s.ev_qkv_gate, 0));
    GDN_CUDA(cudaMemcpyAsync(s.h_qkv, s.d_qkv, sizeof(float) * qkv_dim, cudaMemcpyDeviceToHost, g.d2h));
    GDN_CUDA(cudaMemcpyAsync(s.h_gate, s.d_gate, sizeof(float) * gate_dim, cudaMemcpyDeviceToHost, g.d2h));
    GDN_CUDA(cudaEventRecord(s.ev_d2h_qkv_gate, g.d2h));
    return GDN_OK;
}

int launch_ssm_out(int layer, int si, const float* gated, int gated_dim, int out_dim) {
    int st = check_layer(layer);
    if (!st) st = check_slot(si);
    if (st) return st;
    LayerGPU& L = g.layers[layer];
    if (gated_dim != L.out.in_dim || out_dim != L.out.out_dim)
        return fail(GDN_ERR_SHAPE, "dims (%d, %d) differ from the uploaded ssm_out (%d, %d)", gated_dim, out_dim,
                    L.out.in_dim, L.out.out_dim);
    Slot& s = g.slots[si];
    if ((st = ensure(&s.h_gated, &s.d_gated, &s.cap_gated, gated_dim))) return st;
    if ((st = ensure(&s.h_ssm, &s.d_ssm, &s.cap_out, out_dim))) return st;
    memcpy(s.h_gated, gated, sizeof(float) * gated_dim);
    GDN_CUDA(cudaMemcpyAsync(s.d_gated, s.h_gated, sizeof(float) * gated_dim, cudaMemcpyHostToDevice, g.h2d));
    GDN_CUDA(cudaEventRecord(s.ev_h2d_gated, g.h2d));
    GDN_CUDA(cudaStreamWaitEvent(g.compute, s.ev_h2d_gated, 0));
    if ((st = launch_q8_0_gemv(L.out.qs, L.out.d, out_dim, gated_dim, s.d_gated, GDN_DTYPE_F32, 1, s.d_ssm,
                               out_dim, g.compute)))
        return st;
    GDN_CUDA(cudaEventRecord(s.ev_ssm, g.compute));
    GDN_CUDA(cudaStreamWaitEvent(g.d2h, s.ev_ssm, 0));
    GDN_CUDA(cudaMemcpyAsync(s.h_ssm, s.d_ssm, sizeof(float) * out_dim, cudaMemcpyDeviceToHost, g.d2h));
    GDN_CUDA(cudaEventRecord(s.ev_d2h_ssm, g.d2h));
    return GDN_OK;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" {

int gpu_init(void) {
    if (g.initialized) return 0;
    if (ref_offload_init() != 0) {
        fail(GDN_ERR_CUDA, "gpu_init: the linked expert-cache module failed to initialise");
        return -1;
    }
    if (cudaStreamCreateWithFlags(&g.compute, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&g.h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&g.d2h, cudaStreamNonBlocking) != cudaSuccess) {
        fail(GDN_ERR_CUDA, "gpu_init: stream creation failed");
        return -1;
    }
    for (Slot& s : g.slots) {
        cudaEvent_t* evs[6] = {&s.ev_h2d_normed, &s.ev_qkv_gate, &s.ev_d2h_qkv_gate,
                               &s.ev_h2d_gated, &s.ev_ssm, &s.ev_d2h_ssm};
        for (cudaEvent_t* e : evs)
            if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) {
                fail(GDN_ERR_CUDA, "gpu_init: event creation failed");
                return -1;
            }
    }
    g.initialized = true;
    return 0;
}

void gpu_shutdown(void) {
    if (!g.initialized) return;
    ref_offload_shutdown();
    cudaDeviceSynchronize();
    for (LayerGPU& L : g.layers) {
        free_proj(L.qkv);
        free_proj(L.gate);
        free_proj(L.out);
        L.loaded = false;
        free_proj(L.wqkv);
        free_proj(L.wo);
        L.gqa_loaded = false;
    }
    if (g.gqa.h_in) cudaFreeHost(g.gqa.h_in);
    if (g.gqa.h_out) cudaFreeHost(g.gqa.h_out);
    if (g.gqa.d_in) cudaFree(g.gqa.d_in);
    if (g.gqa.d_out) cudaFree(g.gqa.d_out);
    g.gqa = GqaIO();
    for (Slot& s : g.slots) {
        float* hs[5] = {s.h_normed, s.h_qkv, s.h_gate, s.h_gated, s.h_ssm};
        float* ds[5] = {s.d_normed, s.d_qkv, s.d_gate, s.d_gated, s.d_ssm};
        for (float* p : hs)
            if (p) cudaFreeHost(p);
        for (float* p : ds)
            if (p) cudaFree(p);
        cudaEvent_t evs[6] = {s.ev_h2d_normed, s.ev_qkv_gate, s.ev_d2h_qkv_gate, s.ev_h2d_gated, s.ev_ssm, s.ev_d2h_ssm};
        for (cudaEvent_t e : evs) cudaEventDestroy(e);
        s = Slot();
    }
    cudaStreamDestroy(g.compute);
    cudaStreamDestroy(g.h2d);
    cudaStreamDestroy(g.d2h);
    g.vram_bytes = 0;
    g.initialized = false;
}

int gpu_is_initialized(void) { return g.initialized ? 1 : 0; }

float gpu_vram_used_mb(void) { return (float)(g.vram_bytes / (1024.0 * 1024.0)) + ref_offload_vram_mb(); }

// rows = in_dim, cols = out_dim, as the engine passes them (winmoe_inference.c:938-942).
int gpu_upload_deltanet_weights(int layer, const void* qkv_q8, int qkv_rows, int qkv_cols, const void* gate_q8,
                                int gate_rows, int gate_cols, const void* ssm_out_q8, int ssm_rows, int ssm_cols) {
    if (!g.initialized) return legacy(fail(GDN_ERR_STATE, "gpu_init has not been called"));
    if (layer < 0 || layer >= kMaxLayers) return legacy(fail(GDN_ERR_ARG, "layer %d out of range", layer));
    if (!qkv_q8 || !gate_q8 || !ssm_out_q8) return legacy(fail(GDN_ERR_ARG, "NULL weight pointer"));
    LayerGPU& L = g.layers[layer];
    L.loaded = false;
    int st = upload_proj(L.qkv, qkv_q8, qkv_rows, qkv_cols);
    if (!st) st = upload_proj(L.gate, gate_q8, gate_rows, gate_cols);
    if (!st) st = upload_proj(L.out, ssm_out_q8, ssm_rows, ssm_cols);
    if (st) return legacy(st);
    L.loaded = true;
    return 0;
}

int gpu_launch_qkv_gate(int layer, int slot, const float* normed, int hidden_dim, int qkv_dim, int gate_dim) {
    return legacy(launch_qkv_gate(layer, slot, normed, hidden_dim, qkv_dim, gate_dim));
}

int gpu_wait_qkv_gate(int slot) {
    int st = check_slot(slot);
    if (st) return legacy(st);
    return legacy(cuda_status(cudaEventSynchronize(g.slots[slot].ev_d2h_qkv_gate), "gpu_wait_qkv_gate"));
}

int gpu_launch_ssm_out(int layer, int slot, const float* gated, int gated_dim, int output_dim) {
    return legacy(launch_ssm_out(layer, slot, gated, gated_dim, output_dim));
}

int gpu_wait_ssm_out(int slot) {
    int st = check_slot(slot);
    if (st) return legacy(st);
    return legacy(cuda_status(cudaEventSynchronize(g.slots[slot].ev_d2h_ssm), "gpu_wait_ssm_out"));
}

float* gpu_get_qkv_out(int slot) { return (slot >= 0 && slot < kSlots) ? g.slots[slot].h_qkv : nullptr; }
float* gpu_get_gate_out(int slot) { return (slot >= 0 && slot < kSlots) ? g.slots[slot].h_gate : nullptr; }
float* gpu_get_ssm_out_buf(int slot) { return (slot >= 0 && slot < kSlots) ? g.slots[slot].h_ssm : nullptr; }

int gpu_deltanet_projections(int layer, const float* normed, int hidden_dim, float* qkv_out, int qkv_dim,
                             float* gate_out, int gate_dim) {
    if (gpu_launch_qkv_gate(layer, 0, normed, hidden_dim, qkv_dim, gate_dim) != 0) return -1;
    if (gpu_wait_qkv_gate(0) != 0) return -1;
    memcpy(qkv_out, g.slots[0].h_qkv, sizeof(float) * qkv_dim);
    memcpy(gate_out, g.slots[0].h_gate, sizeof(float) * gate_dim);
    return 0;
}

int gpu_ssm_out_projection(int layer, const float* gated, int gated_dim, float* output, int output_dim) {
    if (gpu_launch_ssm_out(layer, 0, gated, gated_dim, output_dim) != 0) return -1;
    if (gpu_wait_ssm_out(0) != 0) return -1;
    memcpy(output, g.slots[0].h_ssm, sizeof(float) * output_dim);
    return 0;
}

// rows = in_dim, cols = out_dim, as the engine passes them (winmoe_inference.c:956-960:
// Q+gate and K/V [H -> out], O [attn -> H]); the reference's q8_matvec_kernel
// (gpu_offload.cu:870-943) is this library's fp32-activation Q8_0 GEMV.
int gpu_upload_gqa_weights(int layer, const void* wq_q8, int wq_rows, int wq_cols, const void* wk_q8, int wk_rows,
                           int wk_cols, const void* wv_q8, int wv_rows, int wv_cols, const void* wo_q8, int wo_rows,
                           int wo_cols) {
    if (!g.initialized) return legacy(fail(GDN_ERR_STATE, "gpu_init has not been called"));
    if (layer < 0 || layer >= kMaxLayers) return legacy(fail(GDN_ERR_ARG, "layer %d out of range", layer));
    if (!wq_q8 || !wk_q8 || !wv_q8 || !wo_q8) return legacy(fail(GDN_ERR_ARG, "NULL weight pointer"));
    if (wk_rows != wq_rows || wv_rows != wq_rows)
        return legacy(fail(GDN_ERR_SHAPE, "Q, K and V must share their input width (%d, %d, %d)", wq_rows, wk_rows,
                           wv_rows));
    LayerGPU& L = g.layers[layer];
    L.gqa_loaded = false;
    const void* parts[3] = {wq_q8, wk_q8, wv_q8};
    const int outs[3] = {wq_cols, wk_cols, wv_cols};
    int st = upload_rows(L.wqkv, parts, outs, 3, wq_rows);
    if (!st) st = upload_proj(L.wo, wo_q8, wo_rows, wo_cols);
    if (st) return legacy(st);
    L.q_dim = wq_cols;
    L.k_dim = wk_cols;
    L.v_dim = wv_cols;
    L.gqa_loaded = true;
    return 0;
}

int gpu_gqa_projections(int layer, const float* normed, int hidden_dim, float* q_gate_out, int q_gate_dim,
                        float* k_out, int k_dim, float* v_out, int v_dim) {
    int st = check_gqa(layer);
    if (st) return legacy(st);
    if (!normed || !q_gate_out || !k_out || !v_out) return legacy(fail(GDN_ERR_ARG, "gpu_gqa_projections: NULL"));
    const LayerGPU& L = g.layers[layer];
    if (L.wqkv.in_dim != hidden_dim || L.q_dim != q_gate_dim || L.k_dim != k_dim || L.v_dim != v_dim)
        return legacy(fail(GDN_ERR_SHAPE, "gpu_gqa_projections: called with %d -> %d / %d / %d, uploaded as %d -> %d / "
                           "%d / %d", hidden_dim, q_gate_dim, k_dim, v_dim, L.wqkv.in_dim, L.q_dim, L.k_dim, L.v_dim));
    const int splits[3] = {q_gate_dim, k_dim, v_dim};
    float* outs[3] = {q_gate_out, k_out, v_out};
    return legacy(gqa_run(L.wqkv, outs, splits, 3, normed, hidden_dim));
}

int gpu_gqa_output(int layer, const float* attn_out, int attn_dim, float* output, int hidden_dim) {
    int st = check_gqa(layer);
    if (st) return legacy(st);
    if (!attn_out || !output) return legacy(fail(GDN_ERR_ARG, "gpu_gqa_output: NULL"));
    const LayerGPU& L = g.layers[layer];
    if ((st = check_dims(L.wo, "gpu_gqa_output", attn_dim, hidden_dim))) return legacy(st);
    float* outs[1] = {output};
    return legacy(gqa_run(L.wo, outs, &hidden_dim, 1, attn_out, attn_dim));
}

}  // extern "C"
