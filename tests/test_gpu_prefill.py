"""GPU parity of the chunked prefill against the CPU oracle (T sequential
deltanet_forward calls of the reference, which has no prefill path).

Tolerance (north star): bf16-input prefill within 2e-2 relative L2 of the
sequential recurrence, on the outputs and on the final state.  Config 3 itself
(T = 4096 at the 35B-class dims) is checked against 4096 sequential oracle
calls (the reference's deltanet_forward, ~10-60 s of host CPU), and in
addition against the GPU decode step run token by token.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from winmoe_b200 import GDNConfig, HEAD_MAP_INTERLEAVED, layer as L, synth
from winmoe_b200.config import DIMS_35B

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_run(cfg, t, xs, S0=None, cb0=None, pos0=0, head_map=0):
    orc = O.best() if head_map == 0 else O.port()
    S = np.zeros((cfg.num_v_heads, 128, 128), np.float32) if S0 is None else S0.copy()
    cb = np.zeros((4, cfg.qkv_dim), np.float32) if cb0 is None else cb0.copy()
    pos = np.array([pos0], np.int32)
    outs = []
    for x in xs:
        if head_map:
            outs.append(orc.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=O.ACT_FP32, head_map=head_map))
        else:
            outs.append(orc.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=O.ACT_FP32))
    return np.stack(outs), S, cb, int(pos[0])


def upload(cfg, t, **kw):
    return L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                    device=DEV, **kw)


@pytest.mark.parametrize("T", [1, 3, 63, 64, 65, 130, 256, 258, 515])
def test_prefill_small_dims(T):
    """Single and multi-tile prompts: the input projection works in 256-token tiles
    whose rows 0..2 the edge kernel finishes; T = 258 puts the next conv window
    across two tiles, T = 515 leaves a last tile of edge rows only."""
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, layer=1)
    w = upload(cfg, t)
    x = torch.from_numpy(synth.hidden_states(T, cfg.hidden, seed=T)).to(torch.bfloat16)
    want, S_ref, cb_ref, pos_ref = oracle_run(cfg, t, x.float().numpy())
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    y = L.prefill(w, st, x.to(DEV)).cpu().numpy()
    assert rel_l2(y, want) <= TOL, rel_l2(y, want)
    assert rel_l2(st.S[0].cpu().numpy(), S_ref) <= TOL
    # the window holds raw projections: one fp16 rounding of the weights away from the oracle's
    assert rel_l2(st.conv_buf[0].cpu().numpy(), cb_ref) <= 2e-3
    assert int(st.conv_pos.cpu()[0]) == pos_ref == T


@pytest.mark.parametrize("T", [100, 300])
def test_prefill_from_a_running_state(T):
    """Non-zero state and conv window with conv_pos = 5 (the window's slots rotate);
    T = 300 spans two tiles of the input projection."""
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, layer=2)
    w = upload(cfg, t)
    warm = synth.hidden_states(5, cfg.hidden, seed=50)
    _, S0, cb0, p0 = oracle_run(cfg, t, warm)
    x = torch.from_numpy(synth.hidden_states(T, cfg.hidden, seed=51)).to(torch.bfloat16)
    want, S_ref, cb_ref, pos_ref = oracle_run(cfg, t, x.float().numpy(), S0=S0, cb0=cb0, pos0=p0)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    st.S.copy_(torch.from_numpy(S0)[None])
    st.conv_buf.copy_(torch.from_numpy(cb0)[None])
    st.conv_pos.fill_(p0)
    y = L.prefill(w, st, x.to(DEV)).cpu().numpy()
    assert rel_l2(y, want) <= TOL
    assert rel_l2(st.S[0].cpu().numpy(), S_ref) <= TOL
    assert rel_l2(st.conv_buf[0].cpu().numpy(), cb_ref) <= 2e-3
    assert int(st.conv_pos.cpu()[0]) == pos_ref


def test_prefill_35b_dims_then_decode():
    """Config 3 dims, T = 192, then the state is handed to the decode step."""
    cfg = DIMS_35B
    t = synth.layer_tensors(cfg)
    w = upload(cfg, t)
    xs = synth.hidden_states(196, cfg.hidden, seed=0)
    x = torch.from_numpy(xs).to(torch.bfloat16)
    xin = x.float().numpy()
    want, S_ref, _, _ = oracle_run(cfg, t, xin)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    y = L.prefill(w, st, x[:192].to(DEV)).cpu().numpy()
    assert rel_l2(y, want[:192]) <= TOL, rel_l2(y, want[:192])
    for i in range(192, 196):
        yd = L.decode_step(w, st, x[i:i + 1].to(DEV)).cpu().numpy()[0]
        assert rel_l2(yd, want[i]) <= TOL
    assert rel_l2(st.S[0].cpu().numpy(), S_ref) <= TOL


def test_prefill_interleaved_head_map():
    cfg = GDNConfig(512, 2, 8, 128)
    t = synth.layer_tensors(cfg, layer=3)
    w = upload(cfg, t, head_map=HEAD_MAP_INTERLEAVED)
    x = torch.from_numpy(synth.hidden_states(70, cfg.hidden, seed=3)).to(torch.bfloat16)
    want, S_ref, _, _ = oracle_run(cfg, t, x.float().numpy(), head_map=1)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    y = L.prefill(w, st, x.to(DEV)).cpu().numpy()
    assert rel_l2(y, want) <= TOL
    assert rel_l2(st.S[0].cpu().numpy(), S_ref) <= TOL


def test_prefill_4096_matches_oracle():
    """Config 3: T = 4096 bf16 prefill from a zero state against 4096 sequential
    deltanet_forward calls of the reference (fp32-activation mode) on the same
    seeded inputs: every output row block of 64 tokens, all outputs together,
    the final state S, the conv window and conv_pos."""
    cfg = DIMS_35B
    t = synth.layer_tensors(cfg)
    w = upload(cfg, t)
    T = 4096
    x = torch.from_numpy(synth.hidden_states(T, cfg.hidden, seed=0)).to(torch.bfloat16)
    want, S_ref, cb_ref, pos_ref = oracle_run(cfg, t, x.float().numpy())
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    y = L.prefill(w, st, x.to(DEV)).cpu().numpy()
    assert rel_l2(y, want) <= TOL, rel_l2(y, want)
    worst = max(rel_l2(y[i:i + 64], want[i:i + 64]) for i in range(0, T, 64))
    assert worst <= TOL, worst
    assert rel_l2(st.S[0].cpu().numpy(), S_ref) <= TOL, rel_l2(st.S[0].cpu().numpy(), S_ref)
    assert rel_l2(st.conv_buf[0].cpu().numpy(), cb_ref) <= 2e-3
    assert int(st.conv_pos.cpu()[0]) == pos_ref == T


def test_prefill_4096_matches_decode_steps():
    """Config 3 size: T = 4096 prefill vs the decode kernel run token by token."""
    cfg = DIMS_35B
    t = synth.layer_tensors(cfg)
    w = upload(cfg, t)
    T = 4096
    x = torch.randn((T, cfg.hidden), generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).to(DEV)
    st_p = L.DeltaNetState.zeros(cfg, 1, DEV)
    y = L.prefill(w, st_p, x)
    st_d = L.DeltaNetState.zeros(cfg, 1, DEV)
    yd = torch.empty_like(y)
    for i in range(T):
        L.decode_step(w, st_d, x[i:i + 1], out=yd[i:i + 1])
    err = ((y - yd).norm() / yd.norm()).item()
    assert err <= TOL, err
    err_s = ((st_p.S - st_d.S).norm() / st_d.S.norm()).item()
    assert err_s <= TOL, err_s
    assert torch.equal(st_p.conv_pos, st_d.conv_pos)


@pytest.mark.parametrize("T", [5, 70, 300])
def test_prefill_q4_k_layer(T):
    """A layer with Q4_K projections: T >= 8 runs them on the tensor cores (fp16
    activations, exact hi + lo weights), T < 8 on the CUDA-core GEMV."""
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, layer=3, weight_type=12)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 weight_type=12, device=DEV)
    x = torch.from_numpy(synth.hidden_states(T, cfg.hidden, seed=T + 7)).to(torch.bfloat16)
    want, S_ref, _, pos_ref = oracle_run(cfg, t, x.float().numpy())
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    y = L.prefill(w, st, x.to(DEV)).cpu().numpy()
    assert rel_l2(y, want) <= TOL, rel_l2(y, want)
    assert rel_l2(st.S[0].cpu().numpy(), S_ref) <= TOL
    assert int(st.conv_pos.cpu()[0]) == pos_ref == T
