#!/usr/bin/env python
"""Benchmark of the B200 Gated DeltaNet hot path; prints ONE JSON line.

Default workload (N=1): batched decode, B = 256 independent sequences per GPU,
each with its own fp32 32x128x128 state pre-filled N(0, 0.05^2) and bf16
activations N(0,1), through one DeltaNet layer of the 35B-class dims with
seeded Q8_0 weights.  A step is one decode token for all 256 sequences; K
timed steps after W warm-up steps.  Every step streams the 512 MiB of state
in and out of HBM (inputs larger than L2, so no flush is needed).

Multi-GPU (torchrun): every rank runs its own 256 sequences -- the decode
path shards by sequence with no collective ("scaling": "weak"); the only
collectives are the barrier and the max-over-ranks of the timing.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

--impl reference times the reference's own CPU implementation of the path
(the in-place build in oracle/_ref, unmodified dispatch; else the bit-identical
port) on this host's cores, a bounded sample of sequences per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "gated-DeltaNet tok/s (decode B=256, prefill T=4k); % of HBM/TC roofline"
BATCH = 256
# dram__bytes_read.sum + dram__bytes_write.sum of one gdn_state_kernel launch at
# B = 256 (35B-class dims), read from one ncu capture of that launch; the bench
# cannot count DRAM bytes itself, so the line labels this figure as captured.
NCU_STATE_TRAFFIC = 549_619_712 + 479_335_680
NCU_STATE_TRAFFIC_SOURCE = ("ncu capture of one gdn_state_kernel launch at B=256: dram__bytes_read.sum + "
                            "dram__bytes_write.sum (not measured in this run)")


def host_cpu():
    """Threads the CPU baselines use and the host's CPU model (/proc/cpuinfo)."""
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)), model


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the T=4096 prefill leg")
    ap.add_argument("--no-stack", action="store_true", help="skip the 48-layer T=32768 stack leg (config 5)")
    ap.add_argument("--stack-mode", default="p2p", choices=["p2p", "gather"],
                    help="N>1 stack leg: exchanges fused into the kernels as peer stores over NVLink, or NCCL "
                         "all-gathers between the kernels")
    ap.add_argument("--no-extra-legs", action="store_true",
                    help="skip the batch-1 decode (config 1) and Q4_K sweep (config 4) legs")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the T=4096 prefill leg (one GPU); the line's value is the prefill's tok/s")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


_json_out = None


def reserve_stdout():
    """Keeps file descriptor 1 for the JSON line alone: everything else written to stdout,
    by Python or by native libraries (NCCL prints its version banner there whenever NCCL_DEBUG
    is set), goes to stderr from here on."""
    global _json_out
    sys.stdout.flush()
    _json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr


def emit(line):
    out = _json_out if _json_out is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str):
        self.index = index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.tmp.flush()
        rows = [r.split(",") for r in Path(self.tmp.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if len(r) > 8 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 8 and r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            if len(r) > 8:
                for i, n in enumerate(names):
                    if r[5 + i].strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def state_kernel_bytes(cfg, B):
    """Algorithmic HBM bytes of one gdn_state_kernel launch: state read + write,
    the conv'd q/k/v, z, gates read once, the fp16 gated output written once."""
    d2 = cfg.head_dim * cfg.head_dim
    return (B * cfg.num_v_heads * d2 * 4 * 2 + B * cfg.qkv_dim * 4 + B * cfg.inner * 4 + B * 2 * cfg.num_v_heads * 4
            + B * cfg.inner * 2)


def step_bytes(cfg, B):
    """Algorithmic HBM bytes of one decode step at batch B (the per-step
    figure of the roofline): state r+w, conv window (3 rows read, 1 written),
    conv weights, Q8_0 weights once, activations in/out."""
    w = (cfg.in_proj_rows * cfg.hidden + cfg.hidden * cfg.inner) // 32 * 34
    return (B * cfg.num_v_heads * cfg.head_dim * cfg.head_dim * 8 + B * 4 * cfg.qkv_dim * 4 + cfg.qkv_dim * 16 + w
            + B * cfg.hidden * 2 + B * cfg.hidden * 4)


def prefill_flops_per_token(cfg, chunk=64):
    """Algorithmic FLOP per prompt token: the projections plus the chunked
    recurrence (5 C^2 d + 3 C d^2 multiply-adds and the C^3/3 triangular solve
    per chunk and value head)."""
    proj = 2 * cfg.hidden * (cfg.qkv_dim + cfg.inner + 2 * cfg.num_v_heads) + 2 * cfg.inner * cfg.hidden
    d, C = cfg.head_dim, chunk
    rec = cfg.num_v_heads * (5 * 2 * C * C * d + 3 * 2 * C * d * d + 2 * C ** 3 / 3) / C
    return proj + rec


def run_prefill(cfg, w, dev, steps, warmup, peak_tflops, peak_src):
    """Config 3: one sequence, T = 4096 bf16 prompt tokens per step (chunk 64)."""
    import ctypes as C
    import torch
    from winmoe_b200 import layer as L
    from winmoe_b200._lib import lib
    T = 4096
    gen = torch.Generator(device=dev).manual_seed(3)
    xs = torch.randn((warmup + steps, T, cfg.hidden), generator=gen, device=dev).to(torch.bfloat16)
    st = L.DeltaNetState.zeros(cfg, 1, dev)
    out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for i in range(warmup):
        L.prefill(w, st, xs[i], out=out, stream=stream)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        L.prefill(w, st, xs[warmup + i], out=out, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    h = lib()
    h.gdn_profile_enable(1)
    buf = (C.c_float * 4)()
    ph = []
    for i in range(steps):
        L.prefill(w, st, xs[warmup + i], out=out, stream=stream)
        n = h.gdn_decode_phase_ms(buf, 4)
        ph.append([buf[j] for j in range(n)])
    h.gdn_profile_enable(0)
    ph = np.mean(np.array(ph), axis=0)
    flops = prefill_flops_per_token(cfg) * T
    in_flops = 2.0 * T * cfg.hidden * (cfg.qkv_dim + cfg.inner + 2 * cfg.num_v_heads)
    ach = in_flops / (ph[0] / 1e3) / 1e12
    return {
        "workload": "prefill T=4096 (config 3): one sequence, chunk 64, bf16 prompt, fp32 state",
        "value": T / (ms / 1e3), "unit": "tok/s", "ms_per_prefill": ms, "steps": steps, "warmup": warmup,
        "algorithmic_flop_per_token": prefill_flops_per_token(cfg),
        "whole_prefill": {"achieved_tflops": flops / (ms / 1e3) / 1e12, "peak": peak_tflops,
                          "frac": flops / (ms / 1e3) / 1e12 / peak_tflops, "peak_source": peak_src},
        "roofline": {"bound": "tensor", "kernel": "q8_0_gemm_tc (input projection)", "achieved": ach,
                     "peak": peak_tflops, "unit": "TFLOP/s", "frac": ach / peak_tflops, "peak_source": peak_src,
                     "algorithmic_flop_per_launch": in_flops, "launch_ms": float(ph[0])},
        "phases_ms": {"in_proj": float(ph[0]), "prep": float(ph[1]), "chunked_recurrence": float(ph[2]),
                      "out_proj": float(ph[3])},
    }


def decode_b1_bytes(cfg):
    """Algorithmic HBM bytes of one batch-1 decode token (config 1): Q8_0 weights
    once, state read + write, conv window (3 rows read, 1 written), conv weights,
    activations."""
    w = (cfg.in_proj_rows * cfg.hidden + cfg.hidden * cfg.inner) // 32 * 34
    d2 = cfg.head_dim * cfg.head_dim
    act = (cfg.hidden + cfg.in_proj_rows + cfg.qkv_dim + cfg.inner + cfg.hidden) * 4
    return w + cfg.num_v_heads * d2 * 8 + 4 * cfg.qkv_dim * 4 + cfg.qkv_dim * 16 + act


B1_LAYERS = 8  # distinct weight sets cycled by the batch-1 legs: 8 x 36 MB > the 126 MB L2


def run_decode_b1(cfg, w, dev, hbm_peak, peak_src, tensors, with_cpu):
    """Config 1: one sequence from a zero state, 64 fp32 tokens (seed 0), one token per
    step.  Step i runs layer i % 8 of eight layers with distinct copies of the weights
    (and their own states), as a model's layers follow one another: 8 x 36 MB of Q8_0
    exceed the L2, so every step's weights stream from HBM."""
    import torch
    from winmoe_b200 import layer as L, synth
    steps = 64
    t = tensors
    ws = [w] + [L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                         device=dev) for _ in range(B1_LAYERS - 1)]
    xs = torch.from_numpy(synth.hidden_states(steps, cfg.hidden)).to(dev)
    out = torch.empty((1, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    warm = [L.DeltaNetState.zeros(cfg, 1, dev) for _ in ws]
    for i in range(2 * B1_LAYERS):
        L.decode_step(ws[i % B1_LAYERS], warm[i % B1_LAYERS], xs[i:i + 1], out, stream)
    st = [L.DeltaNetState.zeros(cfg, 1, dev) for _ in ws]
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # host-paced: each step launched as the previous one's launches return
    e0.record(stream)
    for i in range(steps):
        L.decode_step(ws[i % B1_LAYERS], st[i % B1_LAYERS], xs[i:i + 1], out, stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_host = e0.elapsed_time(e1) / steps
    # device-paced: the 64 steps queued behind a GPU sleep, so the events time the kernels
    # (the pace of a captured or pre-queued decode loop)
    st = [L.DeltaNetState.zeros(cfg, 1, dev) for _ in ws]
    torch.cuda.synchronize(dev)
    torch.cuda._sleep(20_000_000)
    e0.record(stream)
    for i in range(steps):
        L.decode_step(ws[i % B1_LAYERS], st[i % B1_LAYERS], xs[i:i + 1], out, stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    # the step as one CUDA graph launch per token (DecodeGraph per layer), launched from Python
    gs = [L.DecodeGraph(wl, L.DeltaNetState.zeros(cfg, 1, dev), x_dtype=xs.dtype) for wl in ws]
    for i in range(2 * B1_LAYERS):
        g = gs[i % B1_LAYERS]
        g.x.copy_(xs[i:i + 1])
        g.replay()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for i in range(steps):
        g = gs[i % B1_LAYERS]
        g.x.copy_(xs[i:i + 1])
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_graph = e0.elapsed_time(e1) / steps
    del gs, ws, st, warm
    nb = decode_b1_bytes(cfg)
    ach = nb / (ms / 1e3) / 1e9
    res = {"workload": "decode B=1 (config 1): 64 tokens of one sequence from a zero state, fp32 x, step i "
                       "through layer i % 8 of eight layers with distinct weight copies (8 x 36 MB of Q8_0 > L2: "
                       "every step's weights come from HBM); steps queued behind a GPU sleep (device pace); "
                       "ms_per_token_host_paced launches each step from Python as the previous returns; "
                       "ms_per_token_graph replays each layer's step captured as a CUDA graph, one launch per token",
           "value": 1e3 / ms, "unit": "tok/s", "ms_per_token": ms, "ms_per_token_host_paced": ms_host,
           "ms_per_token_graph": ms_graph,
           "steps": steps, "warmup": 3,
           "roofline": {"bound": "hbm", "kernel": "whole decode step", "achieved": ach, "peak": hbm_peak,
                        "unit": "GB/s", "frac": ach / hbm_peak, "peak_source": peak_src,
                        "algorithmic_bytes_per_token": nb}}
    if with_cpu:
        dt, kind = cpu_reference_run(cfg, tensors, 64, 1, 0, zero_state=True)
        res["cpu_baseline"] = {"value": 64 / dt, "unit": "tok/s",
                               "cores": host_cpu()[0], "cpu_model": host_cpu()[1], "kind": kind,
                               "sample": "the same 64 tokens through the reference's deltanet_forward (unmodified "
                                         "Q8_0/Q8_K dispatch)"}
    return res


GQA_DIMS = {"hidden": 2048, "q_gate": 2 * 16 * 256, "kv": 2 * 256, "attn": 16 * 256}  # 35B-class full-attention layer


def run_gqa(dev, hbm_peak, peak_src, with_cpu):
    """The full-attention (GQA) layers' Q8_0 projections per token (Q+gate, K, V, then O),
    through the reference's own offload calls (host buffers in and out, synchronous) and,
    device-resident, as the same GEMVs on the library's stream."""
    import ctypes as C
    import torch
    from winmoe_b200 import layer as L, synth
    from winmoe_b200._lib import lib
    D = GQA_DIMS
    H, QG, KV, A = D["hidden"], D["q_gate"], D["kv"], D["attn"]
    ws = [synth.q8_0_blocks(n, k, seed=60 + i) for i, (n, k) in enumerate([(QG, H), (KV, H), (KV, H), (H, A)])]
    h = lib()
    own_init = not h.gpu_is_initialized()
    if own_init and h.gpu_init() != 0:
        raise RuntimeError("gpu_init failed")
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    if h.gpu_upload_gqa_weights(0, vp(ws[0]), H, QG, vp(ws[1]), H, KV, vp(ws[2]), H, KV, vp(ws[3]), A, H) != 0:
        raise RuntimeError("gpu_upload_gqa_weights failed")
    n_tok = 64
    xs = synth.hidden_states(n_tok, H, seed=70)
    at = synth.hidden_states(n_tok, A, seed=71)
    qg, k, v, o = (np.zeros(n, np.float32) for n in (QG, KV, KV, H))

    def token(i):
        if h.gpu_gqa_projections(0, vp(xs[i]), H, vp(qg), QG, vp(k), KV, vp(v), KV) != 0:
            raise RuntimeError("gpu_gqa_projections failed")
        if h.gpu_gqa_output(0, vp(at[i]), A, vp(o), H) != 0:
            raise RuntimeError("gpu_gqa_output failed")
    for i in range(3):
        token(i)
    t0 = time.perf_counter()
    for i in range(n_tok):
        token(i)
    e2e_us = (time.perf_counter() - t0) / n_tok * 1e6
    # device-resident: the library's two GEMVs of a token (Q+gate|K|V as one projection, as
    # gpu_upload_gqa_weights stores them, then O), queued behind a GPU sleep so that the
    # events time the kernels and not the host's launches
    # eight copies of the weights cycled over the tokens (8 x 29 MB > L2), as eight layers' weights
    qkv_blocks = np.concatenate(ws[:3])
    sets = [[L.q8_0_planes(qkv_blocks, QG + 2 * KV, H, dev), L.q8_0_planes(ws[3], H, A, dev)]
            for _ in range(B1_LAYERS)]
    xd = torch.from_numpy(xs).to(dev)
    ad = torch.from_numpy(at).to(dev)
    yq = torch.empty((1, QG + 2 * KV), dtype=torch.float32, device=dev)
    yo = torch.empty((1, H), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def dev_token(i):
        planes = sets[i % B1_LAYERS]
        L.gemm_q8_0(planes[0][0], planes[0][1], xd[i:i + 1], out=yq, stream=stream)
        L.gemm_q8_0(planes[1][0], planes[1][1], ad[i:i + 1], out=yo, stream=stream)
    for i in range(2 * B1_LAYERS):
        dev_token(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(20_000_000)  # ~10 ms of GPU time while the host queues 128 launches
    e0.record(stream)
    for i in range(n_tok):
        dev_token(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dev_us = e0.elapsed_time(e1) / n_tok * 1e3
    del sets
    nb = sum(w.nbytes for w in ws) + (3 * H + A + QG + 2 * KV + H) * 4
    if own_init:
        h.gpu_shutdown()
    res = {"workload": "GQA projections per token (35B-class full-attention layer: Q+gate 2048->8192, K and V "
                       "2048->512, O 4096->2048, Q8_0, fp32 activations)",
           "value": 1e6 / e2e_us, "unit": "tok/s", "us_per_token": e2e_us, "tokens": n_tok,
           "path": "gpu_gqa_projections + gpu_gqa_output (host buffers, synchronous, as the engine calls them)",
           "device_us_per_token": dev_us,
           "device_path": "the library's two GEMVs per token on device buffers, token i on weight copy i % 8 "
                          "(8 x 29 MB > L2: weights from HBM), queued behind a GPU sleep",
           "roofline": {"bound": "hbm", "kernel": "gemv_stream_kernel<q8_0> x 2", "achieved": nb / (dev_us / 1e6) / 1e9,
                        "peak": hbm_peak, "unit": "GB/s", "frac": nb / (dev_us / 1e6) / 1e9 / hbm_peak,
                        "peak_source": peak_src, "algorithmic_bytes_per_token": nb}}
    if with_cpu:
        from oracle import oracle as O
        orc = O.ref() if O.ref_available() else O.port()
        n_cpu = 16
        t0 = time.perf_counter()
        for i in range(n_cpu):
            for w, (n, kk), x in zip(ws, [(QG, H), (KV, H), (KV, H), (H, A)], (xs[i], xs[i], xs[i], at[i])):
                orc.quant_matvec(w, x, n, kk, 8, 0)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": n_cpu / dt, "unit": "tok/s",
                               "cores": host_cpu()[0], "cpu_model": host_cpu()[1],
                               "kind": "reference" if O.ref_available() else "port",
                               "sample": f"{n_cpu} tokens through the reference's quant_matvec (type 8, unmodified "
                                         "Q8_K dispatch) for the four projections"}
    return res


EXPERT_HIDDEN, EXPERT_INTER, EXPERT_TOPK, EXPERT_POOL = 2048, 512, 8, 128


def run_expert_ffn(dev, hbm_peak, peak_src, with_cpu):
    """(f)4: the MoE experts of one token, the reference's batched GPU route
    (gpu_expert_batch_start / _add / _finish, gpu_offload.cu:756-809): 8 experts,
    each Q4_K gate / up, SwiGLU, Q5_K down, weighted into the token's output --
    one gdn_experts_ffn call per token (two launches).  Token i uses experts
    8i .. 8i+7 of a pool of 128 distinct experts (243 MB > L2: weights from HBM),
    weights 1/8.  Beside it, the same tokens as 8 single-expert accumulating
    calls each (the reference's call pattern, two launches per expert)."""
    import torch
    from winmoe_b200 import layer as L, synth
    from winmoe_b200._lib import lib
    H, I, K, NP = EXPERT_HIDDEN, EXPERT_INTER, EXPERT_TOPK, EXPERT_POOL
    g = torch.Generator(device=dev).manual_seed(77)

    def blocks(rows, cols, nbytes):
        t = torch.randint(0, 256, (rows * (cols // 256) * nbytes,), generator=g, device=dev, dtype=torch.uint8)
        sb = t.view(rows * (cols // 256), nbytes)
        sb[:, 0:4] = torch.tensor([0x00, 0x20, 0x00, 0x20], dtype=torch.uint8, device=dev)  # d = dmin = fp16 0.0078
        return t
    pool = [(blocks(I, H, 144), blocks(I, H, 144), blocks(H, I, 176)) for _ in range(NP)]
    n_tok = 16
    xs = torch.from_numpy(synth.hidden_states(n_tok, H, seed=78)).to(dev)
    out = torch.zeros((n_tok, H), dtype=torch.float32, device=dev)
    ws = torch.empty(lib().gdn_experts_ffn_workspace_size(K, 1, H, I), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    wts = [1.0 / K] * K

    def token_batched(i):
        sel = [pool[(K * i + e) % NP] for e in range(K)]
        L.experts_ffn([w[0] for w in sel], [w[1] for w in sel], [w[2] for w in sel], 12, 13, H, I, xs[i:i + 1],
                      weights=wts, out=out[i:i + 1], accumulate=True, workspace=ws, stream=stream)

    def token_single(i):
        for e in range(K):
            wg, wu, wd = pool[(K * i + e) % NP]
            L.expert_ffn(wg, wu, wd, 12, 13, H, I, xs[i:i + 1], out=out[i:i + 1], weight=1.0 / K, accumulate=True,
                         workspace=ws, stream=stream)

    def timed(token):
        for i in range(4):
            token(i)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)  # the calls queue behind ~10 ms of GPU time: events time the kernels
        e0.record(stream)
        for i in range(n_tok):
            token(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n_tok * 1e3
    us_single = timed(token_single)
    us = timed(token_batched)
    nb = K * (2 * I * (H // 256) * 144 + H * (I // 256) * 176) + (H + K * (3 * I + 2 * H)) * 4
    res = {"workload": "MoE experts of one token (35B-class: hidden 2048, expert intermediate 512, top-8): Q4_K "
                       "gate + up, SwiGLU, Q5_K down, weighted accumulation, 8 experts per token from a pool of "
                       "128 (243 MB > L2: weights from HBM); one gdn_experts_ffn call (2 launches) per token; "
                       "16 tokens queued behind a GPU sleep",
           "value": 1e6 / us, "unit": "tok/s", "us_per_token": us, "us_per_expert": us / K,
           "us_per_token_single_expert_calls": us_single,
           "roofline": {"bound": "hbm", "kernel": "gemv_stream_kernel<q4_k> (gate + up) + gemv_stream_kernel<q5_k> (down, k-segments) per token",
                        "achieved": nb / (us / 1e6) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                        "frac": nb / (us / 1e6) / 1e9 / hbm_peak, "peak_source": peak_src,
                        "algorithmic_bytes_per_token": nb}}
    if with_cpu:
        from oracle import oracle as O
        orc = O.ref() if O.ref_available() else O.port()
        host = [tuple(t.cpu().numpy() for t in pool[e]) for e in range(K)]
        x0 = xs[0].cpu().numpy()
        n_cpu = 4
        t0 = time.perf_counter()
        for _ in range(n_cpu):
            acc = np.zeros(H, np.float32)
            for wg, wu, wd in host:  # the reference's own q4k / q5k matvecs around the SwiGLU
                gg = orc.quant_matvec(wg, x0, I, H, 12, O.ACT_EXACT)
                uu = orc.quant_matvec(wu, x0, I, H, 12, O.ACT_EXACT)
                a = (gg * (1.0 / (1.0 + np.exp(-gg)))).astype(np.float32) * uu
                acc += np.float32(1.0 / K) * orc.quant_matvec(wd, a, H, I, 13, O.ACT_EXACT)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": n_cpu / dt, "unit": "tok/s", "cores": host_cpu()[0],
                               "cpu_model": host_cpu()[1], "kind": "reference" if O.ref_available() else "port",
                               "sample": f"{n_cpu} tokens x 8 experts through the reference's q4k_matvec / "
                                         "q5k_matvec (Q8_K activations) and a numpy SwiGLU"}
    del pool
    return res


def q4k_call_bytes(cfg, B):
    """Config 4: Q4_K bytes of the four projections plus fp32 activations in and out."""
    w = (cfg.in_proj_rows * cfg.hidden + cfg.hidden * cfg.inner) // 256 * 144
    return w + B * (cfg.hidden + cfg.inner) * 4 * 2


def run_q4k_sweep(cfg, dev, hbm_peak, peak_src, with_cpu):
    """Config 4: the four projections as Q4_K, dequant-GEMV at batch 1 / 8 / 32."""
    import torch
    from winmoe_b200 import layer as L, synth
    t = synth.layer_tensors(cfg, weight_type=12)
    # ten copies of the weights cycled over the calls (10 x 19 MB > L2): weights from HBM
    n_sets = 10
    w_in = [torch.from_numpy(t.in_proj).to(dev) for _ in range(n_sets)]
    w_out = [torch.from_numpy(t.out_proj).to(dev) for _ in range(n_sets)]
    stream = torch.cuda.current_stream(dev)
    rows = {}
    for B, half in ((1, False), (8, False), (32, False), (8, True), (32, True)):
        gen = torch.Generator().manual_seed(40 + B)
        xi = torch.randn((B, cfg.hidden), generator=gen).to(dev)
        xo = torch.randn((B, cfg.inner), generator=gen).to(dev)
        if half:  # fp16 activations: from 32 rows the tcgen05 GEMM (exact hi + lo weights), below the GEMV
            xi, xo = xi.half(), xo.half()
        yi = torch.empty((B, cfg.in_proj_rows), dtype=torch.float32, device=dev)
        yo = torch.empty((B, cfg.hidden), dtype=torch.float32, device=dev)

        def call(i):
            L.gemm_q4_k(w_in[i % n_sets], cfg.in_proj_rows, cfg.hidden, xi, out=yi, stream=stream)
            L.gemm_q4_k(w_out[i % n_sets], cfg.hidden, cfg.inner, xo, out=yo, stream=stream)
        for i in range(n_sets):
            call(i)
        reps = 50
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)  # the calls queue behind ~10 ms of GPU time: events time the kernels
        e0.record(stream)
        for i in range(reps):
            call(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
        nb = q4k_call_bytes(cfg, B)
        ach = nb / (ms / 1e3) / 1e9
        path = "" if not half else " fp16 x (tcgen05 GEMM)" if B >= 32 else " fp16 x (fp16-MMA GEMV)"
        rows[f"B={B}" + path] = {
            "us_per_call": ms * 1e3, "tok_per_s": B / (ms / 1e3), "achieved_gbs": ach, "frac": ach / hbm_peak,
            "algorithmic_bytes_per_call": nb}
    res = {"workload": "Q4_K projection sweep (config 4): in_proj (qkvz + ba rows) and out_proj, dequant-GEMV, "
                       "fp32 activations (m <= 2: dp4a GEMV, m >= 3: fp16-MMA GEMV); one call = the four projections "
                       "for B tokens; the 'fp16 x' rows take the same batches as fp16 activations (B = 32: the "
                       "tcgen05 GEMM); 50 calls queued behind "
                       "a GPU sleep, so the events time the kernels rather than the host's launches; call i uses "
                       "weight copy i % 10 (10 x 19 MB > L2: weights from HBM)",
           "roofline_peak": {"unit": "GB/s", "peak": hbm_peak, "peak_source": peak_src}, "batches": rows}
    if with_cpu:
        from oracle import oracle as O
        orc = O.ref() if O.ref_available() else O.port()
        x = synth.hidden_states(2, cfg.inner, seed=45)
        t0 = time.perf_counter()
        n = 4
        for i in range(n):
            orc.quant_matvec(t.in_proj, x[i % 2, :cfg.hidden], cfg.in_proj_rows, cfg.hidden, 12, O.ACT_EXACT)
            orc.quant_matvec(t.out_proj, x[i % 2], cfg.hidden, cfg.inner, 12, O.ACT_EXACT)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": n / dt, "unit": "tok/s",
                               "cores": host_cpu()[0], "cpu_model": host_cpu()[1],
                               "kind": "reference" if O.ref_available() else "port",
                               "sample": f"{n} tokens through the reference's quant_matvec type 12 (q4k_matvec with "
                                         "Q8_K activations) for the four projections; the reference has no batched "
                                         "Q4_K GEMM, so B tokens cost B times this"}
    return res


STACK_T, STACK_LAYERS = 32768, 48


def run_stack(cfg, dev, world, rank, steps, warmup, tc_peak, peak_src, with_cpu, barrier, max_over_ranks,
              mode="p2p"):
    """Config 5: T = 32768 prompt tokens through 48 residual DeltaNet layers
    (x <- x + DN_l(rmsnorm(x))), value heads sharded over the ranks (strong
    scaling: the same total work at every N).  mode "p2p": the residual sharded
    by tokens, the RMSNorm and the prefill's last kernel storing their rows
    into the ranks that read them over NVLink (CUDA IPC); "gather": NCCL
    all-gathers of the gated heads and of the out_proj rows."""
    import torch
    from winmoe_b200 import synth
    from winmoe_b200.stack import PeerStack, StackLayer, prefill_stack
    T, NL = STACK_T, STACK_LAYERS
    layers = []
    for l in range(NL):
        t = synth.layer_tensors_device(cfg, l, dev)
        layers.append(StackLayer.upload(cfg, t, rank, world, dev))
        del t
    gen = torch.Generator(device=dev).manual_seed(5)
    x0 = torch.randn((T, cfg.hidden), generator=gen, device=dev)
    runs = warmup + steps
    xs = [x0.clone() for _ in range(runs)]
    states = [[lay.state(dev) for lay in layers] for _ in range(runs)]
    stream = torch.cuda.current_stream(dev)
    peers = PeerStack(cfg, T, rank, world, None, dev) if world > 1 and mode == "p2p" else None
    for i in range(warmup):
        prefill_stack(layers, states[i], xs[i], None, rank, world, peers=peers)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(warmup, runs):
        prefill_stack(layers, states[i], xs[i], None, rank, world, peers=peers)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    if peers is not None:
        peers.close()
    ms = max_over_ranks(e0.elapsed_time(e1)) / steps
    flops = prefill_flops_per_token(cfg) * T * NL
    ach = flops / (ms / 1e3) / 1e12
    how = ("the residual sharded by tokens and the exchanges fused into the kernels: the RMSNorm stores each GPU's "
           "rows into every GPU's layer input, the prefill's last kernel each token slice's head columns into the "
           "out_proj operand of the GPU that owns the slice (peer stores over NVLink, CUDA IPC)"
           if peers is not None else "NCCL all-gathers of the gated heads and of the out_proj token slices")
    res = {"workload": f"long prefill (config 5): T={T} tokens through {NL} residual DeltaNet layers "
                       "(rmsnorm, chunked prefill, out_proj), bf16 layer inputs, value heads sharded over the GPUs "
                       f"with {how}", "stack_mode": mode if world > 1 else "single",
           "value": T / (ms / 1e3), "unit": "tok/s", "ms_per_prompt": ms, "steps": steps, "warmup": warmup,
           "n_gpus": world, "scaling": "strong", "layers": NL, "tokens": T,
           "weights": "Q8_0, independent per layer, drawn on the device with torch's generator (same "
                      "distributions and seeds as the parity tests' numpy draws, different values)",
           "exchanged_bytes_per_layer_per_gpu": (
               (world - 1) * (T * cfg.hidden * 2 + (T // world) * cfg.inner * 2) // world if peers is not None
               else (world - 1) * (T * cfg.inner * 2 + T * cfg.hidden * 4) // world),
           "roofline": {"bound": "tensor", "kernel": "whole stack", "achieved": ach, "peak": tc_peak * world,
                        "unit": "TFLOP/s", "frac": ach / (tc_peak * world), "peak_source": peak_src,
                        "algorithmic_flop_per_prompt": flops}}
    if with_cpu and rank == 0 and world == 1:
        from oracle import oracle as O
        orc = O.ref() if O.ref_available() else O.port()
        n_tok, n_layers = 64, 2
        tensors = [synth.layer_tensors(cfg, layer=l) for l in range(n_layers)]
        S = [np.zeros((cfg.num_v_heads, 128, 128), np.float32) for _ in range(n_layers)]
        cb = [np.zeros((4, cfg.qkv_dim), np.float32) for _ in range(n_layers)]
        pos = [np.zeros(1, np.int32) for _ in range(n_layers)]
        ones = np.ones(cfg.hidden, np.float32)
        xs_h = synth.hidden_states(n_tok, cfg.hidden, seed=5)
        t0 = time.perf_counter()
        for x in xs_h:
            for l in range(n_layers):
                x = x + orc.deltanet_forward(cfg, orc.rmsnorm(x, ones), S[l], cb[l], pos[l], tensors[l], act_mode=0)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": n_tok * n_layers / dt, "unit": "token-layers/s",
                               "cores": host_cpu()[0], "cpu_model": host_cpu()[1],
                               "kind": "reference" if O.ref_available() else "port",
                               "sample": f"prefix of {n_tok} tokens through layers 0-1 (rmsnorm + the reference's "
                                         "deltanet_forward per token); the GPU figure in the same unit is "
                                         f"value x {NL}"}
    return res


def cpu_reference_run(cfg, tensors, n_calls, seqs, act_mode, zero_state=False):
    """Times n_calls of the reference's deltanet_forward over `seqs` prefilled sequences."""
    from oracle import oracle as O
    from winmoe_b200 import synth
    orc = O.ref() if O.ref_available() else O.port()
    kind = "reference" if O.ref_available() else "port"
    states = [np.zeros((cfg.num_v_heads, cfg.head_dim, cfg.head_dim), np.float32) if zero_state
              else synth.prefilled_state(cfg, b) for b in range(seqs)]
    convs = [np.zeros((4, cfg.qkv_dim), np.float32) for _ in range(seqs)]
    poss = [np.zeros(1, np.int32) for _ in range(seqs)]
    xs = synth.hidden_states(n_calls, cfg.hidden, seed=11)
    orc.deltanet_forward(cfg, xs[0], states[0].copy(), convs[0].copy(), poss[0].copy(), tensors, act_mode=act_mode)
    t0 = time.perf_counter()
    for i in range(n_calls):
        b = i % seqs
        orc.deltanet_forward(cfg, xs[i], states[b], convs[b], poss[b], tensors, act_mode=act_mode)
    dt = time.perf_counter() - t0
    return dt, kind


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from winmoe_b200 import synth
    from winmoe_b200.config import DIMS_35B as cfg
    tensors = synth.layer_tensors(cfg)
    per_step = 4  # sequence-tokens of the B=256 workload timed per step
    dt_w, kind = cpu_reference_run(cfg, tensors, per_step * args.warmup, per_step, 0) if args.warmup else (0, None)
    dt, kind = cpu_reference_run(cfg, tensors, per_step * args.steps, per_step, 0)
    toks = per_step * args.steps
    v = toks / dt
    cores, cpu_model = host_cpu()
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode B=256 (config 2), reference deltanet_forward per sequence-token",
                   "hidden": cfg.hidden, "k_heads": cfg.num_k_heads, "v_heads": cfg.num_v_heads,
                   "head_dim": cfg.head_dim, "weights": "Q8_0"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "cpu_model": cpu_model, "kind": kind,
                         "sample": f"{per_step} sequence-tokens per step x {args.steps} steps of the B=256 decode "
                                   "workload (prefilled states), engine/runtime/deltanet_impl.h:deltanet_forward "
                                   "with its unmodified Q8_0/Q8_K dispatch, OpenMP over all host threads"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def run_ours(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world, rank, local = dist_env()
    if world > 1:
        # NCCL's communicator log (INIT lines: rank, nranks, device, ring/tree setup) on stderr,
        # raised to INFO where the environment leaves it off or lower (VERSION / WARN); its version
        # banner goes to fd 1, which reserve_stdout() points at stderr too
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        # one communicator line per rank on stderr (stdout carries only the JSON line)
        nv = ".".join(str(v) for v in torch.cuda.nccl.version())
        print(f"[bench] nccl {nv} communicator: rank {dist.get_rank()} of {dist.get_world_size()}, local rank "
              f"{local}, device {torch.cuda.get_device_name(local)} ({torch.cuda.get_device_properties(local).uuid})",
              file=sys.stderr, flush=True)
    dev = torch.device("cuda", torch.cuda.current_device())

    from winmoe_b200 import layer as L, synth
    from winmoe_b200._lib import lib
    from winmoe_b200.config import DIMS_35B as cfg

    B, K, W = BATCH, args.steps, args.warmup
    tensors = synth.layer_tensors(cfg)
    w = L.DeltaNetWeights.upload(cfg, tensors.in_proj, tensors.out_proj, tensors.conv1d_w, tensors.ssm_a,
                                 tensors.dt_bias, tensors.head_norm, device=dev)
    if args.prefill_only:
        if world > 1:
            raise SystemExit("--prefill-only runs on one GPU")
        hbm_peak, tc_peak, peak_src = measured_peaks()
        pre = run_prefill(cfg, w, dev, K, W, tc_peak, peak_src)
        line = {"metric": METRIC, "value": pre["value"], "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W,
                "ms_per_step": pre["ms_per_prefill"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": pre["workload"], "hidden": cfg.hidden, "k_heads": cfg.num_k_heads,
                           "v_heads": cfg.num_v_heads, "head_dim": cfg.head_dim, "weights": "Q8_0 (seeded)"},
                # per prefill: x -> fp16, in_proj GEMM (with conv1d + SiLU + L2 in its epilogue), gate-row
                # GEMM + its split-K sum into the gates, edge rows + conv window, chunk_local, chunk_scan,
                # chunk_out, out_proj GEMM
                "gpu_launches": 9 * K, "roofline": pre["roofline"], "prefill": pre}
        emit(line)
        return

    gen = torch.Generator(device=dev).manual_seed(7 + 1000 * rank)
    st = L.DeltaNetState.zeros(cfg, B, dev)
    st.S.normal_(0.0, 0.05, generator=gen)
    xs = torch.randn((W + K, B, cfg.hidden), generator=gen, device=dev).to(torch.bfloat16)
    out = torch.empty((B, cfg.hidden), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    # --- device-resident inputs (value)
    for i in range(W):
        L.decode_step(w, st, xs[i], out, stream)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    smi_id = vis[torch.cuda.current_device()] if vis else str(torch.cuda.current_device())
    with ClockSampler(smi_id) as clk:
        # the K steps queue behind ~1 ms of GPU time, so the events time the device and not the
        # host's issue of the first step (which matters most for short runs, --steps 4)
        torch.cuda._sleep(2_000_000)
        e0.record(stream)
        for i in range(K):
            L.decode_step(w, st, xs[W + i], out, stream)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clocks = clk.summary()
    value = B * K * world / (ms / 1e3)

    # --- end to end through the public API: every step's x copied in from pinned host memory
    # and its output copied back to pinned host memory, as a serving loop runs it: the copies
    # on their own streams, double-buffered, so step i+1's input and step i-1's output move
    # while step i computes (events order each copy against the steps that use its buffers)
    xh = torch.empty((K + W, B, cfg.hidden), dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(xs.cpu())
    oh = torch.empty((2, B, cfg.hidden), dtype=torch.float32, pin_memory=True)
    xd = torch.empty((2, B, cfg.hidden), dtype=torch.bfloat16, device=dev)
    od = torch.empty((2, B, cfg.hidden), dtype=torch.float32, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    # three events per buffer, created once and re-recorded (a wait uses the most
    # recent record, issued in stream order before it)
    ev_h2d = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_d2h = [torch.cuda.Event() for _ in range(2)]

    def pipelined(first, n, start_ev):
        s_in.wait_event(start_ev)
        for i in range(first, first + n):
            b = i % 2
            if i - 2 >= first:
                s_in.wait_event(ev_comp[b])  # xd[b] was step i-2's input
                # od[b] held step i-2's output: the compute stream is ordered behind its read-out
                # through ev_h2d[b] below, so it waits on one copy-engine event per step, not two
                # (each such wait costs the compute engine ~10 us here, however early the copy ended)
                s_in.wait_event(ev_d2h[b])
            with torch.cuda.stream(s_in):
                xd[b].copy_(xh[i], non_blocking=True)
            ev_h2d[b].record(s_in)
            stream.wait_event(ev_h2d[b])
            L.decode_step(w, st, xd[b], od[b], stream)
            ev_comp[b].record(stream)
            s_out.wait_event(ev_comp[b])
            with torch.cuda.stream(s_out):
                oh[b].copy_(od[b], non_blocking=True)
            ev_d2h[b].record(s_out)
        stream.wait_event(ev_d2h[(first + n - 1) % 2])  # the last output is on the host
    e_w = torch.cuda.Event()
    e_w.record(stream)
    pipelined(0, W, e_w)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda._sleep(2_000_000)  # as above: the steps and their copies queue behind ~1 ms of GPU time
    e0.record(stream)
    pipelined(W, K, e0)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    e2e = B * K * world / (ms_e2e / 1e3)

    # --- per-kernel durations (separate pass: events around each phase, per step)
    import ctypes as C
    h = lib()
    h.gdn_profile_enable(1)
    phases = []
    buf = (C.c_float * 4)()
    for i in range(K):
        L.decode_step(w, st, xs[W + i], out, stream)
        n = h.gdn_decode_phase_ms(buf, 4)
        phases.append([buf[j] for j in range(n)])
    h.gdn_profile_enable(0)
    ph = np.mean(np.array(phases), axis=0)
    state_ms = float(ph[2])
    hbm_peak, tc_peak, peak_src = measured_peaks()
    sk_bytes = state_kernel_bytes(cfg, B)
    achieved = sk_bytes / (state_ms / 1e3) / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "operand_dtypes": {"state": "f32", "x": "bf16", "projections": "f16 x f16 -> f32 (tcgen05, TMEM)"},
        "data": "synthetic",
        "config": {"workload": "decode B=256 per GPU (config 2): one DeltaNet layer, one token for 256 sequences "
                               "per step", "batch_per_gpu": B, "hidden": cfg.hidden, "k_heads": cfg.num_k_heads,
                   "v_heads": cfg.num_v_heads, "head_dim": cfg.head_dim, "weights": "Q8_0 (seeded)",
                   "state": "fp32 N(0,0.05^2) prefilled", "parallelism": f"sequence-sharded x{world}, no collective",
                   "l2": "inputs larger than L2: 512 MiB of state read+written per step"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": B * cfg.hidden * 2,
                "d2h_bytes_per_step": B * cfg.hidden * 4,
                "path": "decode_step on device buffers; each step's x copied in from pinned host memory and its "
                        "output copied back on two copy streams, double-buffered, overlapping the neighbouring "
                        "steps' kernels"},
        # per step: x -> fp16, in_proj GEMM (tcgen05), prep, state, out_proj GEMM (tcgen05), split-K sum
        "gpu_launches": 6 * K,
        "roofline": {"bound": "hbm", "kernel": "gdn_state_kernel", "achieved": achieved, "peak": hbm_peak,
                     "unit": "GB/s", "frac": achieved / hbm_peak, "peak_source": peak_src,
                     "traffic": NCU_STATE_TRAFFIC, "traffic_source": NCU_STATE_TRAFFIC_SOURCE,
                     "algorithmic_bytes_per_launch": sk_bytes,
                     "launch_ms": state_ms},
        "phases_ms": {"in_proj": float(ph[0]), "prep": float(ph[1]), "state": float(ph[2]),
                      "out_proj": float(ph[3])},
        "step_roofline": {"algorithmic_bytes_per_step": step_bytes(cfg, B),
                          "achieved_gbs": step_bytes(cfg, B) / (ms / K / 1e3) / 1e9,
                          "frac": step_bytes(cfg, B) / (ms / K / 1e3) / 1e9 / hbm_peak},
        "clocks": clocks,
    }
    if world == 1 and not args.no_prefill:
        line["prefill"] = run_prefill(cfg, w, dev, min(K, 8), W, tc_peak, peak_src)
    if not args.no_stack:
        line["stack"] = run_stack(cfg, dev, world, rank, min(K, 2), W, tc_peak, peak_src,
                                  not args.no_cpu_baseline, barrier, max_over_ranks, args.stack_mode)
    if world == 1 and not args.no_extra_legs:
        line["decode_b1"] = run_decode_b1(cfg, w, dev, hbm_peak, peak_src, tensors, not args.no_cpu_baseline)
        line["q4k_sweep"] = run_q4k_sweep(cfg, dev, hbm_peak, peak_src, not args.no_cpu_baseline)
        line["gqa"] = run_gqa(dev, hbm_peak, peak_src, not args.no_cpu_baseline)
        line["expert_ffn"] = run_expert_ffn(dev, hbm_peak, peak_src, not args.no_cpu_baseline)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, kind = cpu_reference_run(cfg, tensors, 64, 4, 0)
        cores, cpu_model = host_cpu()
        line["cpu_baseline"] = {
            "value": 64 / dt, "unit": "tok/s", "cores": cores, "cpu_model": cpu_model,
            "kind": kind, "sample": "64 sequence-tokens (4 prefilled sequences x 16 tokens) of the B=256 decode "
                                    "workload through the reference's deltanet_forward, unmodified dispatch"}
        if "prefill" in line:
            dtp, kindp = cpu_reference_run(cfg, tensors, 64, 1, 0)
            line["prefill"]["cpu_baseline"] = {
                "value": 64 / dtp, "unit": "tok/s", "cores": cores, "cpu_model": cpu_model, "kind": kindp,
                "sample": "64 consecutive prompt tokens of one sequence through the reference's deltanet_forward "
                          "(the reference has no chunked prefill; tokens go one by one)"}
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        emit(line)


def main():
    args = parse()
    reserve_stdout()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
