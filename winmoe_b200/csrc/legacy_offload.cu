// The reference engine's DeltaNet offload API (engine/runtime/gpu_offload.h:
// 19-53), re-implemented on this library's kernels so that the engine
// (engine/runtime/winmoe_inference.c:868, 938-942, 1215-1226, 1437-1440) can
// link against it unchanged.
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
    cudaStream_t compute{}, h2d{}, d2h{};
    double vram_bytes = 0;
} g;

int legacy(int st) { return st == GDN_OK ? 0 : -1; }

void free_proj(Proj& p) {
    if (p.qs) cudaFree(p.qs);
    if (p.d) cudaFree(p.d);
    p = Proj();
}

int upload_proj(Proj& p, const void* host_blocks, int in_dim, int out_dim) {
    if (in_dim <= 0 || out_dim <= 0 || in_dim % 32 != 0)
        return fail(GDN_ERR_SHAPE, "upload: in_dim must be a positive multiple of 32 (got %d x %d)", in_dim, out_dim);
    free_proj(p);
    const size_t nb = (size_t)in_dim / 32 * out_dim;
    void* raw = nullptr;
    GDN_CUDA(cudaMalloc(&raw, nb * 34));
    cudaError_t e = cudaMemcpy(raw, host_blocks, nb * 34, cudaMemcpyHostToDevice);
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
    cudaDeviceSynchronize();
    for (LayerGPU& L : g.layers) {
        free_proj(L.qkv);
        free_proj(L.gate);
        free_proj(L.out);
        L.loaded = false;
    }
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

float gpu_vram_used_mb(void) { return (float)(g.vram_bytes / (1024.0 * 1024.0)); }

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

}  // extern "C"
