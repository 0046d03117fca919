"""GPU parity of the decode step against the CPU oracle (the reference's own
deltanet_forward, compiled in place when the host can run it, else the
bit-identical plain-C port), on the benchmark configs' seeded inputs.

Tolerance (north star): decode outputs and final state within 1e-3 relative
L2, in fp32, against the fp32-activation oracle ("ref-fp32act").
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from winmoe_b200 import GDNConfig, HEAD_MAP_INTERLEAVED, layer as L, synth
from winmoe_b200.config import DIMS_35B

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def t35():
    return synth.layer_tensors(DIMS_35B)


@pytest.fixture(scope="module")
def w35(t35):
    return L.DeltaNetWeights.upload(DIMS_35B, t35.in_proj, t35.out_proj, t35.conv1d_w, t35.ssm_a, t35.dt_bias,
                                    t35.head_norm, device=DEV)


def run_oracle(cfg, t, xs, S0=None, head_map=0):
    """Sequential oracle over xs [T][hidden] for one sequence; returns (outs, S, conv_buf, pos)."""
    orc = O.best() if head_map == 0 else O.port()
    S = np.zeros((cfg.num_v_heads, cfg.head_dim, cfg.head_dim), np.float32) if S0 is None else S0.copy()
    cb = np.zeros((4, cfg.qkv_dim), np.float32)
    pos = np.zeros(1, np.int32)
    outs = []
    for x in xs:
        if head_map == 0:
            outs.append(orc.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=O.ACT_FP32))
        else:
            outs.append(orc.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=O.ACT_FP32, head_map=head_map))
    return np.stack(outs), S, cb, pos


def test_decode_b1_64_steps(t35, w35):
    """Config 1: batch 1, 64 tokens from a zero state, fp32 activations."""
    cfg = DIMS_35B
    xs = synth.hidden_states(64, cfg.hidden)
    want, S_ref, cb_ref, pos_ref = run_oracle(cfg, t35, xs)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    got = []
    for x in xs:
        got.append(L.decode_step(w35, st, torch.from_numpy(x).reshape(1, -1).to(DEV)).cpu().numpy()[0])
    got = np.stack(got)
    for i in range(64):
        assert rel_l2(got[i], want[i]) <= TOL, (i, rel_l2(got[i], want[i]))
    assert rel_l2(st.S.cpu().numpy()[0], S_ref) <= TOL
    assert rel_l2(st.conv_buf.cpu().numpy()[0], cb_ref) <= TOL
    assert int(st.conv_pos.cpu()[0]) == int(pos_ref[0]) == 64


@pytest.mark.parametrize("B,dtype", [(3, torch.float32), (4, torch.bfloat16), (5, torch.bfloat16),
                                     (8, torch.bfloat16), (9, torch.bfloat16),
                                     (32, torch.float16), (40, torch.float32), (64, torch.bfloat16),
                                     (64, torch.float32), (96, torch.float16), (130, torch.bfloat16)])
def test_decode_batched_prefilled(t35, w35, B, dtype):
    """Independent sequences with prefilled states (config 2 style), a few steps:
    CUDA-core projections (fp32 x below 64 sequences, 16-bit x below 5) and the
    tensor-core ones (16-bit x from 5, any x from 64)."""
    cfg = DIMS_35B
    steps = 3
    S0 = np.stack([synth.prefilled_state(cfg, b) for b in range(B)])
    xs = synth.hidden_states(steps * B, cfg.hidden, seed=42).reshape(steps, B, cfg.hidden)
    xs_t = torch.from_numpy(xs).to(dtype)
    xs_in = xs_t.float().numpy()  # the oracle sees the same (rounded) activations
    st = L.DeltaNetState.zeros(cfg, B, DEV)
    st.S.copy_(torch.from_numpy(S0))
    outs = []
    for s in range(steps):
        outs.append(L.decode_step(w35, st, xs_t[s].to(DEV).contiguous()).cpu().numpy())
    check = range(B) if B <= 8 else [0, 1, B // 2, B - 1]
    for b in check:
        want, S_ref, _, _ = run_oracle(cfg, t35, xs_in[:, b], S0=S0[b])
        for s in range(steps):
            assert rel_l2(outs[s][b], want[s]) <= TOL, (b, s, rel_l2(outs[s][b], want[s]))
        assert rel_l2(st.S[b].cpu().numpy(), S_ref) <= TOL, b


def test_decode_b256_tensor_core_subset(t35, w35):
    """Config 2 as specified: B = 256 sequences (tensor-core projections), bf16
    activations, prefilled states, 32 steps; a fixed subset of 8 sequences is
    compared with the oracle at every step (outputs) and at the end (S, conv
    window), so drift of the projections and of the fp16 gated heads over the
    32 steps shows."""
    cfg = DIMS_35B
    B, steps = 256, 32
    check = [0, 1, 37, 100, 128, 129, 200, 255]
    gen = torch.Generator().manual_seed(7)
    S0 = (torch.randn((B, cfg.num_v_heads, 128, 128), generator=gen) * 0.05)
    xs_t = torch.randn((steps, B, cfg.hidden), generator=gen).to(torch.bfloat16)
    st = L.DeltaNetState.zeros(cfg, B, DEV)
    st.S.copy_(S0)
    outs = [L.decode_step(w35, st, xs_t[s].to(DEV).contiguous()).cpu().numpy() for s in range(steps)]
    xs_in = xs_t.float().numpy()
    for b in check:
        want, S_ref, cb_ref, pos_ref = run_oracle(cfg, t35, xs_in[:, b], S0=S0[b].numpy())
        for s in range(steps):
            assert rel_l2(outs[s][b], want[s]) <= TOL, (b, s, rel_l2(outs[s][b], want[s]))
        assert rel_l2(st.S[b].cpu().numpy(), S_ref) <= TOL, b
        assert rel_l2(st.conv_buf[b].cpu().numpy(), cb_ref) <= TOL, b
        assert int(st.conv_pos[b]) == int(pos_ref[0]) == steps


def test_decode_interleaved_head_map():
    """g = h % Hk (winmoe_inference.c:1330) against the oracle's interleaved map."""
    cfg = GDNConfig(512, 2, 8, 128)
    t = synth.layer_tensors(cfg, layer=3)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 head_map=HEAD_MAP_INTERLEAVED, device=DEV)
    xs = synth.hidden_states(5, cfg.hidden, seed=9)
    want, S_ref, _, _ = run_oracle(cfg, t, xs, head_map=1)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    for i, x in enumerate(xs):
        y = L.decode_step(w, st, torch.from_numpy(x).reshape(1, -1).to(DEV)).cpu().numpy()[0]
        assert rel_l2(y, want[i]) <= TOL
    assert rel_l2(st.S.cpu().numpy()[0], S_ref) <= TOL


def test_decode_q4_k_layer():
    """A layer whose projections are Q4_K (quant_matvec type 12)."""
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, weight_type=12)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 weight_type=12, device=DEV)
    xs = synth.hidden_states(4, cfg.hidden, seed=5)
    want, S_ref, _, _ = run_oracle(cfg, t, xs)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    for i, x in enumerate(xs):
        y = L.decode_step(w, st, torch.from_numpy(x).reshape(1, -1).to(DEV)).cpu().numpy()[0]
        assert rel_l2(y, want[i]) <= TOL


def test_reference_signature_mirror(t35):
    """deltanet_forward with the reference's argument list (host GGUF tensors)."""
    cfg = DIMS_35B
    parts = t35.split_in_proj()
    xs = synth.hidden_states(3, cfg.hidden, seed=77)
    want, _, _, _ = run_oracle(cfg, t35, xs)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    out = np.zeros(cfg.hidden, np.float32)
    for i, x in enumerate(xs):
        L.deltanet_forward(out, x, st, parts["w_qkv"], 8, parts["w_gate"], 8, parts["w_alpha"], 8,
                           parts["w_beta"], 8, t35.out_proj, 8, t35.conv1d_w, t35.ssm_a, t35.dt_bias,
                           t35.head_norm, cfg.hidden)
        assert rel_l2(out, want[i]) <= TOL


def test_legacy_offload_api(t35):
    """gpu_init / gpu_upload_deltanet_weights / async launch+wait, as the engine calls them."""
    import ctypes as C
    from winmoe_b200._lib import lib
    cfg = DIMS_35B
    parts = t35.split_in_proj()
    h = lib()
    assert h.gpu_init() == 0
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    assert h.gpu_upload_deltanet_weights(0, vp(parts["w_qkv"]), cfg.hidden, cfg.qkv_dim, vp(parts["w_gate"]),
                                         cfg.hidden, cfg.inner, vp(t35.out_proj), cfg.inner, cfg.hidden) == 0
    x = synth.hidden_states(1, cfg.hidden, seed=3)[0]
    assert h.gpu_launch_qkv_gate(0, 1, vp(x), cfg.hidden, cfg.qkv_dim, cfg.inner) == 0
    assert h.gpu_wait_qkv_gate(1) == 0
    qkv = np.ctypeslib.as_array(h.gpu_get_qkv_out(1), shape=(cfg.qkv_dim,)).copy()
    gate = np.ctypeslib.as_array(h.gpu_get_gate_out(1), shape=(cfg.inner,)).copy()
    P = O.port()
    assert rel_l2(qkv, P.quant_matvec(parts["w_qkv"], x, cfg.qkv_dim, cfg.hidden, 8, O.ACT_FP32)) <= 1e-5
    assert rel_l2(gate, P.quant_matvec(parts["w_gate"], x, cfg.inner, cfg.hidden, 8, O.ACT_FP32)) <= 1e-5
    g = synth.hidden_states(1, cfg.inner, seed=4)[0]
    outb = np.zeros(cfg.hidden, np.float32)
    assert h.gpu_ssm_out_projection(0, vp(g), cfg.inner, vp(outb), cfg.hidden) == 0
    assert rel_l2(outb, P.quant_matvec(t35.out_proj, g, cfg.hidden, cfg.inner, 8, O.ACT_FP32)) <= 1e-5
    # errors: unknown layer, bad dims -> -1 with a message, as the reference's -1
    assert h.gpu_launch_qkv_gate(5, 0, vp(x), cfg.hidden, cfg.qkv_dim, cfg.inner) == -1
    assert h.gpu_launch_qkv_gate(0, 0, vp(x), cfg.hidden + 32, cfg.qkv_dim, cfg.inner) == -1
    h.gpu_shutdown()
    assert h.gpu_is_initialized() == 0


def test_legacy_gqa_offload():
    """gpu_upload_gqa_weights / gpu_gqa_projections / gpu_gqa_output, as the engine calls them
    for its full-attention layers (35B-class: 16 query heads of 256 with gates, 2 KV heads)."""
    import ctypes as C
    from winmoe_b200._lib import lib
    H, q_gate, kv, attn = 2048, 2 * 16 * 256, 2 * 256, 16 * 256
    wq = synth.q8_0_blocks(q_gate, H, seed=61)
    wk = synth.q8_0_blocks(kv, H, seed=62)
    wv = synth.q8_0_blocks(kv, H, seed=63)
    wo = synth.q8_0_blocks(H, attn, seed=64)
    h = lib()
    assert h.gpu_init() == 0
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    assert h.gpu_upload_gqa_weights(3, vp(wq), H, q_gate, vp(wk), H, kv, vp(wv), H, kv, vp(wo), attn, H) == 0
    P = O.port()
    for seed in (5, 6):  # twice: the staging buffers are reused
        x = synth.hidden_states(1, H, seed=seed)[0]
        qg, k, v = np.zeros(q_gate, np.float32), np.zeros(kv, np.float32), np.zeros(kv, np.float32)
        assert h.gpu_gqa_projections(3, vp(x), H, vp(qg), q_gate, vp(k), kv, vp(v), kv) == 0
        assert rel_l2(qg, P.quant_matvec(wq, x, q_gate, H, 8, O.ACT_FP32)) <= 1e-5
        assert rel_l2(k, P.quant_matvec(wk, x, kv, H, 8, O.ACT_FP32)) <= 1e-5
        assert rel_l2(v, P.quant_matvec(wv, x, kv, H, 8, O.ACT_FP32)) <= 1e-5
        a = synth.hidden_states(1, attn, seed=seed + 10)[0]
        o = np.zeros(H, np.float32)
        assert h.gpu_gqa_output(3, vp(a), attn, vp(o), H) == 0
        assert rel_l2(o, P.quant_matvec(wo, a, H, attn, 8, O.ACT_FP32)) <= 1e-5
    # a layer without GQA weights, or dims other than the uploaded ones: -1 with a message
    assert h.gpu_gqa_output(4, vp(a), attn, vp(o), H) == -1
    assert h.gpu_gqa_projections(3, vp(x), H, vp(qg), q_gate // 2, vp(k), kv, vp(v), kv) == -1
    h.gpu_shutdown()


@pytest.mark.parametrize("cfg,B", [(GDNConfig(256, 1, 3, 128), 2), (GDNConfig(768, 3, 6, 128), 70)])
def test_decode_odd_shapes(cfg, B):
    """Odd value-head counts (padded projection rows) and a batch above the tensor-core threshold."""
    t = synth.layer_tensors(cfg, layer=5)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 device=DEV)
    S0 = np.stack([synth.prefilled_state(cfg, b) for b in range(B)])
    xs = synth.hidden_states(3 * B, cfg.hidden, seed=21).reshape(3, B, cfg.hidden)
    xs_t = torch.from_numpy(xs).to(torch.bfloat16)
    st = L.DeltaNetState.zeros(cfg, B, DEV)
    st.S.copy_(torch.from_numpy(S0))
    outs = [L.decode_step(w, st, xs_t[s].to(DEV).contiguous()).cpu().numpy() for s in range(3)]
    for b in sorted({0, B // 2, B - 1}):
        want, S_ref, cb_ref, _ = run_oracle(cfg, t, xs_t.float().numpy()[:, b], S0=S0[b])
        for s in range(3):
            assert rel_l2(outs[s][b], want[s]) <= TOL, (b, s)
        assert rel_l2(st.S[b].cpu().numpy(), S_ref) <= TOL
        assert rel_l2(st.conv_buf[b].cpu().numpy(), cb_ref) <= TOL
    assert (st.conv_pos.cpu().numpy() == 3).all()


def test_decode_reference_projections():
    """gdn_decode_step_ex(GDN_DECODE_REF_PROJECTIONS): projections as the
    reference's CPU computes them (Q8_K activations) -- far closer to the
    reference's own unmodified layer (ref-exact) than the fp32-activation route."""
    cfg = DIMS_35B
    t = synth.layer_tensors(cfg, layer=1)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 device=DEV)
    B, steps = 3, 8
    xs = np.stack([synth.hidden_states(B, cfg.hidden, seed=50 + i) for i in range(steps)])
    orc = O.best()
    err = {True: [], False: []}
    for ref in (True, False):
        st = L.DeltaNetState.zeros(cfg, B, DEV)
        got = [L.decode_step(w, st, torch.from_numpy(xs[i]).to(DEV), ref_projections=ref).cpu().numpy()
               for i in range(steps)]
        for b in range(B):
            S = np.zeros((cfg.num_v_heads, 128, 128), np.float32)
            cb = np.zeros((4, cfg.qkv_dim), np.float32)
            pos = np.zeros(1, np.int32)
            for i in range(steps):
                want = orc.deltanet_forward(cfg, xs[i, b], S, cb, pos, t, act_mode=O.ACT_EXACT)
                err[ref].append(rel_l2(got[i][b], want))
    assert max(err[True]) <= 1e-4, max(err[True])
    assert max(err[True]) * 10 <= np.median(err[False]), (max(err[True]), np.median(err[False]))


@pytest.mark.parametrize("B,dtype", [(1, torch.float32), (256, torch.bfloat16)])
def test_decode_graph_replay_matches_eager(t35, w35, B, dtype):
    """DecodeGraph: replays of the captured step give the eager step's outputs and
    states bit for bit (same kernels on the same buffers)."""
    cfg = DIMS_35B
    gen = torch.Generator().manual_seed(B)
    S0 = torch.randn((B, cfg.num_v_heads, 128, 128), generator=gen) * 0.05
    xs = torch.randn((4, B, cfg.hidden), generator=gen).to(dtype).to(DEV)
    eager, graphed = L.DeltaNetState.zeros(cfg, B, DEV), L.DeltaNetState.zeros(cfg, B, DEV)
    eager.S.copy_(S0)
    graphed.S.copy_(S0)
    g = L.DecodeGraph(w35, graphed, x_dtype=dtype)
    assert torch.equal(graphed.S, eager.S)  # capturing does not run the step
    for i in range(4):
        want = L.decode_step(w35, eager, xs[i].contiguous())
        g.x.copy_(xs[i])
        got = g.replay()
        torch.cuda.synchronize()
        assert torch.equal(got, want), i
    assert torch.equal(graphed.S, eager.S)
    assert torch.equal(graphed.conv_buf, eager.conv_buf)
    assert torch.equal(graphed.conv_pos, eager.conv_pos)


@pytest.mark.parametrize("B", [16, 32])
def test_decode_q4_k_layer_batched(B):
    """A Q4_K layer with bf16 activations, 3 steps from prefilled states: B = 16 on
    the fp16-MMA GEMV, B = 32 on the tcgen05 GEMM (fp16 operands, exact weights,
    split-K out_proj)."""
    cfg = DIMS_35B
    steps = 3
    t = synth.layer_tensors(cfg, weight_type=12)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 weight_type=12, device=DEV)
    S0 = np.stack([synth.prefilled_state(cfg, b) for b in range(B)])
    xs_t = torch.from_numpy(synth.hidden_states(steps * B, cfg.hidden, seed=77).reshape(steps, B, -1)).to(
        torch.bfloat16)
    xs_in = xs_t.float().numpy()
    st = L.DeltaNetState.zeros(cfg, B, DEV)
    st.S.copy_(torch.from_numpy(S0))
    outs = [L.decode_step(w, st, xs_t[s].to(DEV).contiguous()).cpu().numpy() for s in range(steps)]
    for b in (0, 7, B - 1):
        want, S_ref, _, _ = run_oracle(cfg, t, xs_in[:, b], S0=S0[b])
        for s in range(steps):
            assert rel_l2(outs[s][b], want[s]) <= TOL, (b, s, rel_l2(outs[s][b], want[s]))
        assert rel_l2(st.S[b].cpu().numpy(), S_ref) <= TOL, b
