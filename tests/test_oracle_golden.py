"""The CPU oracle (plain-C restatement) against golden fixtures produced by the
reference's own CPU code (tests/golden/make_golden.py).  Bit-exact throughout:
the restatement keeps the reference's operation order.  Runs without the
reference tree and without a GPU."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from winmoe_b200 import synth
from winmoe_b200.config import DIMS_35B, GDNConfig

G = np.load(Path(__file__).resolve().parent / "golden" / "reference_cpu.npz")
SMALL = GDNConfig(hidden=256, num_k_heads=1, num_v_heads=2, head_dim=128)


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(bytes.fromhex(h.hexdigest()), np.uint8)


def same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.fixture(scope="module")
def P():
    return O.port()


def test_q8_0(P):
    blocks = synth.q8_0_blocks(96, 256, seed=11)
    x = synth.hidden_states(1, 256, seed=12)[0]
    assert np.array_equal(sha(blocks, x), G["q8_blocks_sha"]), "synthetic generator changed"
    assert same_bits(P.q8_0_dequant(blocks, 96 * 256), G["q8_dequant"])
    assert same_bits(P.quant_matvec(blocks, x, 96, 256, 8, O.ACT_EXACT), G["q8_matvec_exact"])
    bl = synth.q8_0_blocks(160, 512, seed=13)
    xl = synth.hidden_states(1, 512, seed=14)[0]
    assert np.array_equal(sha(bl, xl), G["q8l_sha"])
    assert same_bits(P.quant_matvec(bl, xl, 160, 512, 8, O.ACT_EXACT), G["q8l_matvec_exact"])
    assert same_bits(P.quant_matvec(bl, xl, 160, 512, 8, O.ACT_FP32), G["q8l_matvec_fp32"])


def test_q8_k_quantisation(P):
    xq = synth.hidden_states(1, 1024, seed=15)[0] * 3.0
    xq[300:556] = 0.0
    assert np.array_equal(sha(xq), G["q8k_x_sha"])
    assert np.array_equal(P.quantize_q8_K(xq), G["q8k_bytes"])


def test_q4_k(P):
    b4 = synth.q4_k_blocks(64, 512, seed=16)
    x4 = synth.hidden_states(1, 512, seed=17)[0]
    assert np.array_equal(sha(b4, x4), G["q4_sha"])
    assert same_bits(P.quant_matvec(b4, x4, 64, 512, 12, O.ACT_EXACT), G["q4_matvec_exact"])
    assert same_bits(P.quant_matvec(b4, x4, 64, 512, 12, O.ACT_FP32), G["q4_matvec_fp32"])
    import ctypes as C
    for r in range(64):
        q12 = np.ascontiguousarray(b4.reshape(64, 2, 144)[r, 0, 4:16])
        sc, mn = np.zeros(8, np.uint8), np.zeros(8, np.uint8)
        P.h.orc_q4_k_scales(q12.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p),
                            mn.ctypes.data_as(C.c_void_p))
        assert np.array_equal(np.concatenate([sc, mn]), G["q4_scales"][r])


def test_q4_k_dequant_consistent_with_reference_int_kernel(P):
    """The GGML nibble layout of the float dequant agrees with the reference's
    integer q4k_dot_q8k (golden): sum(w*x) matches up to int8 activation rounding."""
    b4 = synth.q4_k_blocks(64, 512, seed=16)
    x4 = synth.hidden_states(1, 512, seed=17)[0]
    w = P.q4_k_dequant(b4, 64 * 512).reshape(64, 512).astype(np.float64)
    y = w @ x4.astype(np.float64)
    ref = G["q4_matvec_exact"].astype(np.float64)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 2e-2
    yf = G["q4_matvec_fp32"].astype(np.float64)
    assert np.linalg.norm(y - yf) / np.linalg.norm(yf) < 1e-6


def test_q4_k_known_answer_is_the_float_fallback_layout(P):
    """test_q4k.c:42-43 expects 240.0 from q4k_dot_block; the golden file holds the
    reference build's own answer.  In the GGML layout the same block sums the
    32 low nibbles of chunk 0 with scale 1: 15*32 = 480, which is why the
    reference's float fallback is not the layout the kernels use."""
    assert float(G["q4k_kat_dot_block"][0]) == 240.0
    kat = np.zeros(144, np.uint8)
    kat[0:2] = [0x00, 0x3C]
    kat[4] = 1
    kat[16:] = 0x0F
    w = P.q4_k_dequant(kat, 256)
    assert float(w.astype(np.float64).sum()) == 480.0


def test_rmsnorm(P):
    xr = synth.hidden_states(1, 2048, seed=18)[0]
    wr = (1.0 + 0.1 * synth.hidden_states(1, 2048, seed=19)[0]).astype(np.float32)
    assert np.array_equal(sha(xr, wr), G["rms_sha"])
    assert same_bits(P.rmsnorm(xr, wr), G["rmsnorm"])


def _run(P, cfg, steps, mode, layer=0, s0_std=0.0):
    t = synth.layer_tensors(cfg, layer=layer)
    xs = synth.hidden_states(steps, cfg.hidden, seed=100 + layer)
    S = (synth.prefilled_state(cfg, 0, std=s0_std) if s0_std else
         np.zeros((cfg.num_v_heads, cfg.head_dim, cfg.head_dim), np.float32))
    cb = np.zeros((4, cfg.qkv_dim), np.float32)
    pos = np.zeros(1, np.int32)
    outs = np.stack([P.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=mode) for x in xs])
    h = sha(t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm, xs)
    return outs, S, cb, pos, h


@pytest.mark.parametrize("mode,name", [(O.ACT_EXACT, "exact"), (O.ACT_FP32, "fp32")])
def test_layer_small(P, mode, name):
    outs, S, cb, pos, h = _run(P, SMALL, 6, mode)
    assert np.array_equal(h, G["small_inputs_sha"])
    assert same_bits(outs, G[f"small_{name}_out"])
    assert same_bits(S, G[f"small_{name}_S"])
    assert same_bits(cb, G[f"small_{name}_conv"])
    assert int(pos[0]) == int(G[f"small_{name}_pos"][0]) == 6


def test_layer_small_prefilled(P):
    outs, S, _, _, h = _run(P, SMALL, 5, O.ACT_FP32, layer=1, s0_std=0.05)
    assert np.array_equal(h, G["small_prefilled_sha"])
    assert same_bits(outs, G["small_prefilled_out"])
    assert same_bits(S, G["small_prefilled_S"])


def test_layer_benchmark_dims(P):
    outs, S, cb, _, h = _run(P, DIMS_35B, 4, O.ACT_FP32)
    assert np.array_equal(h, G["d35_inputs_sha"])
    assert same_bits(outs, G["d35_out"])
    assert np.array_equal(sha(S), G["d35_S_sha"])
    assert np.array_equal(sha(cb), G["d35_conv_sha"])
