"""The expert FFN's GGUF projections and its fused and batched routes on the
GPU (engine/runtime/gpu_offload.cu:271-331, 341-457, 718-809) against the CPU
oracle.

Bit-exact: Q5_K dequantised weights.  Tolerances: the streamed Q5_K GEMV with
fp32 activations vs the oracle's fp32-activation rows (q5k_matvec_kernel),
rel-L2 <= 1e-5 (summation order and the activations' int8-level split, below
5e-7 of a block's max |x|, differ); the whole expert FFN (gate / up Q4_K or
Q5_K, SwiGLU, down) vs the oracle's, rel-L2 <= 1e-4 (the SwiGLU's expf on two
sides of a 1e-5 projection difference)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from winmoe_b200 import layer as L, synth
from winmoe_b200._lib import GDNError, lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
Q4K, Q5K = 12, 13


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).to(DEV)


@pytest.mark.parametrize("rows,cols", [(64, 512), (2048, 512), (3, 256)])
def test_q5_k_dequant_bit_exact(rows, cols):
    blocks = synth.q5_k_blocks(rows, cols, seed=600 + rows)
    got = L.dequant_q5_k(dev(blocks), rows, cols).cpu().numpy()
    want = O.port().q5_k_dequant(blocks, rows * cols).reshape(rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13])
@pytest.mark.parametrize("n,k", [(2048, 512), (512, 2048), (300, 4096), (64, 256)])
def test_q5_k_gemv_fp32(m, n, k):
    blocks = synth.q5_k_blocks(n, k, seed=610 + n)
    x = synth.hidden_states(m, k, seed=611)
    y = L.gemm_q5_k(dev(blocks), n, k, torch.from_numpy(x).to(DEV)).cpu().numpy()
    P = O.port()
    for i in range(m):
        want = P.quant_matvec(blocks, x[i], n, k, Q5K, O.ACT_FP32)
        assert rel_l2(y[i], want) <= 1e-5, i


def _expert(hidden, inter, gate_type, down_type, seed):
    gen = {Q4K: synth.q4_k_blocks, Q5K: synth.q5_k_blocks}
    return (gen[gate_type](inter, hidden, seed), gen[gate_type](inter, hidden, seed + 1),
            gen[down_type](hidden, inter, seed + 2))


@pytest.mark.parametrize("gate_type,down_type", [(Q4K, Q5K), (Q4K, Q4K), (Q5K, Q5K)])
@pytest.mark.parametrize("m", [1, 3])
def test_expert_ffn_matches_oracle(gate_type, down_type, m):
    hidden, inter = 2048, 512  # 35B-class MoE expert dims
    wg, wu, wd = _expert(hidden, inter, gate_type, down_type, seed=620)
    x = synth.hidden_states(m, hidden, seed=623)
    got = L.expert_ffn(dev(wg), dev(wu), dev(wd), gate_type, down_type, hidden, inter,
                       torch.from_numpy(x).to(DEV)).cpu().numpy()
    P = O.port()
    for i in range(m):
        want = P.expert_ffn(x[i], wg, wu, wd, gate_type, down_type, hidden, inter)
        assert rel_l2(got[i], want) <= 1e-4, i


def test_expert_batch_accumulates_weighted_experts():
    """gpu_expert_batch_add semantics: moe_out += w_e * expert_e(x) over experts."""
    hidden, inter = 2048, 512
    x = synth.hidden_states(1, hidden, seed=630)
    xd = torch.from_numpy(x).to(DEV)
    experts = [_expert(hidden, inter, Q4K, Q5K, seed=640 + 3 * e) for e in range(3)]
    weights = [0.5, 0.3, 0.2]
    out = torch.zeros((1, hidden), dtype=torch.float32, device=DEV)
    ws = torch.empty(lib().gdn_expert_ffn_workspace_size(1, hidden, inter), dtype=torch.uint8, device=DEV)
    want = np.zeros(hidden, np.float32)
    P = O.port()
    for (wg, wu, wd), w in zip(experts, weights):
        L.expert_ffn(dev(wg), dev(wu), dev(wd), Q4K, Q5K, hidden, inter, xd, out=out, weight=w, accumulate=True,
                     workspace=ws)
        P.expert_ffn(x[0], wg, wu, wd, Q4K, Q5K, hidden, inter, weight=w, out=want)
    assert rel_l2(out.cpu().numpy()[0], want) <= 1e-4


@pytest.mark.parametrize("ne,m,accumulate", [(1, 1, False), (2, 3, True), (8, 1, True), (8, 4, False),
                                               (5, 2, True)])
def test_experts_ffn_batched_matches_oracle(ne, m, accumulate):
    """gpu_expert_batch_start / _add x ne / _finish as one call: two launches
    whatever ne; out (+)= sum_e w_e * expert_e(x), in expert order."""
    hidden, inter = 2048, 512
    experts = [_expert(hidden, inter, Q4K, Q5K, seed=700 + 3 * e) for e in range(ne)]
    weights = [0.9 / (e + 1) for e in range(ne)]
    x = synth.hidden_states(m, hidden, seed=701)
    base = synth.hidden_states(m, hidden, seed=702) if accumulate else np.zeros((m, hidden), np.float32)
    out = torch.from_numpy(base.copy()).to(DEV)
    L.experts_ffn([dev(e[0]) for e in experts], [dev(e[1]) for e in experts], [dev(e[2]) for e in experts], Q4K,
                  Q5K, hidden, inter, torch.from_numpy(x).to(DEV), weights=weights, out=out, accumulate=accumulate)
    got = out.cpu().numpy()
    P = O.port()
    for i in range(m):
        want = base[i].copy()
        for (wg, wu, wd), w in zip(experts, weights):
            P.expert_ffn(x[i], wg, wu, wd, Q4K, Q5K, hidden, inter, weight=w, out=want)
        assert rel_l2(got[i], want) <= 1e-4, i
    # and the same sum as ne single-expert accumulating calls
    seq = torch.from_numpy(base.copy()).to(DEV)
    for (wg, wu, wd), w in zip(experts, weights):
        L.expert_ffn(dev(wg), dev(wu), dev(wd), Q4K, Q5K, hidden, inter, torch.from_numpy(x).to(DEV), out=seq,
                     weight=w, accumulate=True)
    assert rel_l2(got, seq.cpu().numpy()) <= 1e-6


@pytest.mark.parametrize("gate_type,down_type", [(Q5K, Q4K), (Q4K, Q4K)])
@pytest.mark.parametrize("m", [1, 4])
def test_experts_ffn_batched_other_types(gate_type, down_type, m):
    """The batched block with Q5_K gate / up segments and Q4_K down k-segments, on
    the dp4a (m = 1) and fp16-MMA (m = 4) GEMVs."""
    hidden, inter, ne = 2048, 512, 3
    experts = [_expert(hidden, inter, gate_type, down_type, seed=760 + 3 * e) for e in range(ne)]
    weights = [0.5, -0.25, 0.125]
    x = synth.hidden_states(m, hidden, seed=761)
    got = L.experts_ffn([dev(e[0]) for e in experts], [dev(e[1]) for e in experts], [dev(e[2]) for e in experts],
                        gate_type, down_type, hidden, inter, torch.from_numpy(x).to(DEV), weights=weights).cpu().numpy()
    P = O.port()
    for i in range(m):
        want = np.zeros(hidden, np.float32)
        for (wg, wu, wd), w in zip(experts, weights):
            P.expert_ffn(x[i], wg, wu, wd, gate_type, down_type, hidden, inter, weight=w, out=want)
        assert rel_l2(got[i], want) <= 1e-4, i


def test_experts_ffn_unweighted_and_empty():
    hidden, inter = 512, 256
    experts = [_expert(hidden, inter, Q5K, Q5K, seed=720 + 3 * e) for e in range(3)]
    x = synth.hidden_states(2, hidden, seed=721)
    args = ([dev(e[0]) for e in experts], [dev(e[1]) for e in experts], [dev(e[2]) for e in experts], Q5K, Q5K,
            hidden, inter, torch.from_numpy(x).to(DEV))
    got = L.experts_ffn(*args).cpu().numpy()  # weights None: all 1
    P = O.port()
    for i in range(2):
        want = np.zeros(hidden, np.float32)
        for wg, wu, wd in experts:
            P.expert_ffn(x[i], wg, wu, wd, Q5K, Q5K, hidden, inter, weight=1.0, out=want)
        assert rel_l2(got[i], want) <= 1e-4, i
    out = torch.full((2, hidden), 3.0, device=DEV)
    L.experts_ffn([], [], [], Q5K, Q5K, hidden, inter, torch.from_numpy(x).to(DEV), out=out, accumulate=True)
    assert bool((out == 3.0).all())  # no experts: nothing launched, out untouched


def test_experts_ffn_rejects_bad_arguments():
    hidden, inter = 512, 256
    wg, wu, wd = (dev(a) for a in _expert(hidden, inter, Q4K, Q5K, seed=730))
    x = torch.zeros((1, hidden), device=DEV)
    with pytest.raises(GDNError):  # more experts than one call takes
        L.experts_ffn([wg] * 9, [wu] * 9, [wd] * 9, Q4K, Q5K, hidden, inter, x)
    with pytest.raises(GDNError):  # a misaligned expert among aligned ones
        L.experts_ffn([wg, wg[1:]], [wu, wu], [wd, wd], Q4K, Q5K, hidden, inter, x)
    with pytest.raises(GDNError):
        L.experts_ffn([wg], [wu], [wd, wd], Q4K, Q5K, hidden, inter, x)


def test_expert_ffn_rejects_bad_arguments():
    hidden, inter = 512, 256
    wg, wu, wd = _expert(hidden, inter, Q4K, Q5K, seed=650)
    x = torch.zeros((1, hidden), device=DEV)
    with pytest.raises(GDNError):
        L.expert_ffn(dev(wg), dev(wu), dev(wd), 8, Q5K, hidden, inter, x)  # Q8_0 is not an expert type
    with pytest.raises(GDNError):
        L.expert_ffn(dev(wg), dev(wu), dev(wd), Q4K, Q5K, hidden, 100, x)  # inter not a multiple of 256
