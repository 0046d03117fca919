"""gdn_layer_forward -- deltanet_forward's own argument list (raw GGUF blocks
plus GGML type ids, dims from gdn_dn_init_dims) -- through the C ABI.

It prepares the weight set once and then runs the same kernels as
gdn_decode_step / gdn_prefill, so its results must equal the DeltaNetWeights
path bit for bit; with host- or device-resident weights alike; and one decode
token is checked against the reference's deltanet_forward (1e-3, the decode
bound)."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as O
from winmoe_b200 import GDNConfig, layer as L, synth
from winmoe_b200._lib import check, gdn_dn_state, lib
from winmoe_b200.config import DIMS_35B

pytestmark = pytest.mark.gpu
DEV = "cuda"


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(a):
    if isinstance(a, torch.Tensor):
        return C.c_void_p(a.data_ptr())
    return C.c_void_p(a.ctypes.data) if a is not None else None


class Args:
    """The reference's tensors of one layer, on the host (numpy) or the device."""

    def __init__(self, t, device: bool):
        parts = t.split_in_proj()
        keep = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV) if device else np.ascontiguousarray(a)
        self.w = [keep(parts["w_qkv"]), keep(parts["w_gate"]), keep(parts["w_alpha"]), keep(parts["w_beta"]),
                  keep(t.out_proj)]
        self.p = [keep(t.conv1d_w), keep(t.ssm_a), keep(t.dt_bias), keep(t.head_norm)]
        self.wt = t.weight_type

    def call(self, out, x, st, hidden, batch, T, no_gates=False):
        w = list(self.w)
        if no_gates:
            w[2] = w[3] = None
        state = gdn_dn_state(st.S.data_ptr(), st.conv_buf.data_ptr(), st.conv_pos.data_ptr())
        args = [ptr(out), ptr(x), C.byref(state)]
        for a in w:
            args += [ptr(a), self.wt]
        args += [ptr(a) for a in self.p]
        return lib().gdn_layer_forward(*args, hidden, batch, T, stream())


def weights(cfg, t, zero_gates=False):
    in_proj = t.in_proj.copy()
    if zero_gates:  # the rows of ssm_beta and ssm_alpha as all-zero blocks
        in_proj[cfg.qkv_dim + cfg.inner:] = 0
    return L.DeltaNetWeights.upload(cfg, in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                    weight_type=t.weight_type, device=DEV)


def init_dims(cfg):
    check(lib().gdn_dn_init_dims(cfg.inner, cfg.num_k_heads, cfg.head_dim))


@pytest.mark.parametrize("on_device", [False, True])
def test_decode_token_matches_decode_step(on_device):
    cfg = DIMS_35B
    t = synth.layer_tensors(cfg, layer=1)
    init_dims(cfg)
    a = Args(t, on_device)
    B = 3
    st = L.DeltaNetState.zeros(cfg, B, DEV)
    for b in range(B):
        st.S[b] = torch.from_numpy(synth.prefilled_state(cfg, b))
    st_ref = st.clone()
    w = weights(cfg, t)
    gen = torch.Generator().manual_seed(5)
    for _ in range(2):
        x = torch.randn((B, cfg.hidden), generator=gen).to(DEV)
        y = torch.empty((B, cfg.hidden), device=DEV)
        check(a.call(y, x, st, cfg.hidden, B, 1))
        y_ref = L.decode_step(w, st_ref, x)
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref)
        assert torch.equal(st.S, st_ref.S) and torch.equal(st.conv_buf, st_ref.conv_buf)
        assert torch.equal(st.conv_pos, st_ref.conv_pos)
    check(lib().gdn_layer_release_all())


def test_prompts_match_prefill_per_sequence():
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, layer=2)
    init_dims(cfg)
    a = Args(t, False)
    B, T = 2, 130
    x = torch.from_numpy(synth.hidden_states(B * T, cfg.hidden, seed=8)).reshape(B, T, cfg.hidden).to(DEV)
    st = L.DeltaNetState.zeros(cfg, B, DEV)
    y = torch.empty((B, T, cfg.hidden), device=DEV)
    check(a.call(y, x, st, cfg.hidden, B, T))
    w = weights(cfg, t)
    for b in range(B):
        s1 = L.DeltaNetState.zeros(cfg, 1, DEV)
        y1 = L.prefill(w, s1, x[b])
        torch.cuda.synchronize()
        assert torch.equal(y[b], y1)
        assert torch.equal(st.S[b], s1.S[0]) and torch.equal(st.conv_buf[b], s1.conv_buf[0])
        assert int(st.conv_pos[b]) == T
    check(lib().gdn_layer_release_all())


def test_null_gate_projections_are_zero():
    """w_alpha = w_beta = NULL: the reference zeroes those projections; the
    same layer with all-zero gate rows must give the same bits."""
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, layer=3)
    init_dims(cfg)
    a = Args(t, True)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    x = torch.from_numpy(synth.hidden_states(1, cfg.hidden, seed=3)).to(DEV)
    y = torch.empty((1, cfg.hidden), device=DEV)
    check(a.call(y, x, st, cfg.hidden, 1, 1, no_gates=True))
    st_ref = L.DeltaNetState.zeros(cfg, 1, DEV)
    y_ref = L.decode_step(weights(cfg, t, zero_gates=True), st_ref, x)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref) and torch.equal(st.S, st_ref.S)
    check(lib().gdn_layer_release_all())


def test_decode_matches_the_reference():
    cfg = DIMS_35B
    t = synth.layer_tensors(cfg)
    init_dims(cfg)
    a = Args(t, False)
    xs = synth.hidden_states(4, cfg.hidden, seed=21)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    orc = O.best()
    S = np.zeros((cfg.num_v_heads, 128, 128), np.float32)
    cb = np.zeros((4, cfg.qkv_dim), np.float32)
    pos = np.zeros(1, np.int32)
    for x in xs:
        y = torch.empty((1, cfg.hidden), device=DEV)
        check(a.call(y, torch.from_numpy(x).reshape(1, -1).to(DEV), st, cfg.hidden, 1, 1))
        want = orc.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=O.ACT_FP32)
        got = y.cpu().numpy()[0]
        assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 1e-3
    assert np.linalg.norm(st.S[0].cpu().numpy() - S) / np.linalg.norm(S) <= 1e-3
    check(lib().gdn_layer_release_all())


def test_rejects_mixed_types_and_bad_dims():
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg)
    a = Args(t, False)
    st = L.DeltaNetState.zeros(cfg, 1, DEV)
    x = torch.zeros((1, cfg.hidden), device=DEV)
    y = torch.empty_like(x)
    init_dims(cfg)
    # w_qkv says Q4_K while the others say Q8_0: rejected before any work
    state = gdn_dn_state(st.S.data_ptr(), st.conv_buf.data_ptr(), st.conv_pos.data_ptr())
    args = [ptr(y), ptr(x), C.byref(state), ptr(a.w[0]), 12] + sum([[ptr(w), 8] for w in a.w[1:]], [])
    args += [ptr(p) for p in a.p]
    assert lib().gdn_layer_forward(*args, cfg.hidden, 1, 1, stream()) == -3
    assert lib().gdn_dn_init_dims(4096, 16, 64) == -2
