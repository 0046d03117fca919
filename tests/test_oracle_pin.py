"""The plain-C oracle against the reference's own CPU code compiled in place
(oracle/_ref), on fresh seeded inputs: bit-exact.  Skipped where the reference
build is absent or the host lacks AVX-512/VNNI (e.g. a GPU box without them;
the golden fixtures still pin the oracle there)."""
import numpy as np
import pytest

from oracle import oracle as O
from winmoe_b200 import synth
from winmoe_b200.config import GDNConfig

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="reference build unavailable on this host")


def same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("rows,cols,seed", [(128, 256, 1), (130, 2048, 2), (64, 4096, 3), (300, 512, 4)])
def test_q8_0_matvec_both_modes(rows, cols, seed):
    b = synth.q8_0_blocks(rows, cols, seed)
    x = synth.hidden_states(1, cols, seed + 50)[0]
    for mode in (O.ACT_EXACT, O.ACT_FP32):
        assert same_bits(O.port().quant_matvec(b, x, rows, cols, 8, mode),
                         O.ref().quant_matvec(b, x, rows, cols, 8, mode))
    assert same_bits(O.port().q8_0_dequant(b, rows * cols), O.ref().q8_0_dequant(b, rows * cols))


@pytest.mark.parametrize("rows,cols,seed", [(128, 256, 5), (64, 2048, 6), (129, 4096, 7)])
def test_q4_k_matvec_both_modes(rows, cols, seed):
    b = synth.q4_k_blocks(rows, cols, seed)
    x = synth.hidden_states(1, cols, seed + 50)[0] * 4.0
    for mode in (O.ACT_EXACT, O.ACT_FP32):
        assert same_bits(O.port().quant_matvec(b, x, rows, cols, 12, mode),
                         O.ref().quant_matvec(b, x, rows, cols, 12, mode))


@pytest.mark.parametrize("rows,cols,seed", [(128, 256, 8), (64, 2048, 9), (129, 512, 10)])
def test_q5_k_matvec_both_modes(rows, cols, seed):
    """Q5_K (the expert FFN's down projections): the restatement against the
    reference's q5k_matvec (Q8_K activations) and the shim's fp32-activation
    rows of q5k_matvec_kernel, bit for bit."""
    b = synth.q5_k_blocks(rows, cols, seed)
    x = synth.hidden_states(1, cols, seed + 50)[0] * 4.0
    for mode in (O.ACT_EXACT, O.ACT_FP32):
        assert same_bits(O.port().quant_matvec(b, x, rows, cols, 13, mode),
                         O.ref().quant_matvec(b, x, rows, cols, 13, mode))


@pytest.mark.parametrize("mode", [O.ACT_EXACT, O.ACT_FP32])
def test_expert_ffn_is_the_reference_projections(mode):
    """The oracle's expert FFN = the reference build's gate / up / down
    projections around swiglu_kernel's (g * sigmoid(g)) * u, bit for bit."""
    hidden, inter = 512, 256
    wg, wu = synth.q4_k_blocks(inter, hidden, 11), synth.q4_k_blocks(inter, hidden, 12)
    wd = synth.q5_k_blocks(hidden, inter, 13)
    x = synth.hidden_states(1, hidden, 14)[0]
    R = O.ref()
    g = R.quant_matvec(wg, x, inter, hidden, 12, mode)
    u = R.quant_matvec(wu, x, inter, hidden, 12, mode)
    a = ((g * (np.float32(1) / (np.float32(1) + np.exp(-g).astype(np.float32)))) * u).astype(np.float32)
    want = R.quant_matvec(wd, a, hidden, inter, 13, mode)
    got = O.port().expert_ffn(x, wg, wu, wd, 12, 13, hidden, inter, act_mode=mode)
    # the SwiGLU here uses numpy's exp, which may differ from expf in the last
    # bit: the whole is compared at 1e-6 (the projections themselves are pinned
    # bit for bit by test_q4_k_matvec_both_modes / test_q5_k_matvec_both_modes)
    assert np.linalg.norm(got - want) <= 1e-6 * np.linalg.norm(want)
    acc = np.full(hidden, 0.5, np.float32)
    O.port().expert_ffn(x, wg, wu, wd, 12, 13, hidden, inter, weight=0.25, out=acc, act_mode=mode)
    assert np.allclose(acc, 0.5 + 0.25 * got, rtol=1e-6, atol=1e-6)


def test_q8_k_edge_values():
    x = synth.hidden_states(1, 2048, 9)[0]
    x[0:256] = 0.0                      # zero block
    x[256:512] = 1e-12                  # amax below 1e-10
    x[512] = 1e30                       # huge outlier
    x[1024:1280] = np.linspace(-2.5, 2.5, 256, dtype=np.float32)  # exact .5 ties after scaling
    assert np.array_equal(O.port().quantize_q8_K(x), O.ref().quantize_q8_K(x))


@pytest.mark.parametrize("cfg", [GDNConfig(256, 1, 2, 128), GDNConfig(512, 2, 8, 128), GDNConfig(1024, 4, 4, 128)])
@pytest.mark.parametrize("mode", [O.ACT_EXACT, O.ACT_FP32])
def test_layer_sequences(cfg, mode):
    t = synth.layer_tensors(cfg, layer=2)
    xs = synth.hidden_states(7, cfg.hidden, seed=5) * 3.0
    Sp = synth.prefilled_state(cfg, 3)
    Sr = Sp.copy()
    cp = np.zeros((4, cfg.qkv_dim), np.float32)
    cr = cp.copy()
    pp = np.zeros(1, np.int32)
    pr = pp.copy()
    for x in xs:
        a = O.port().deltanet_forward(cfg, x, Sp, cp, pp, t, act_mode=mode)
        b = O.ref().deltanet_forward(cfg, x, Sr, cr, pr, t, act_mode=mode)
        assert same_bits(a, b)
    assert same_bits(Sp, Sr) and same_bits(cp, cr) and int(pp[0]) == int(pr[0])


def test_interleaved_map_is_a_head_permutation():
    """winmoe_inference.c:1330 (g = h % Hk) equals deltanet_impl.h:280 (g = h / hpg)
    after permuting value heads; the oracle's interleaved mode is checked against the
    reference's grouped code run on permuted weights."""
    cfg = GDNConfig(512, 2, 8, 128)
    t = synth.layer_tensors(cfg, layer=4)
    hv, hk, hpg, d = cfg.num_v_heads, cfg.num_k_heads, cfg.heads_per_group, cfg.head_dim
    # value head h (interleaved, group h % hk) -> grouped position p with p // hpg == h % hk
    perm = [0] * hv
    for h in range(hv):
        perm[h] = (h % hk) * hpg + h // hk
    inv = np.argsort(perm)
    row_bytes = cfg.hidden // 32 * 34
    qkvz = t.in_proj.reshape(cfg.in_proj_rows, row_bytes)
    rows = np.arange(cfg.in_proj_rows)
    new = rows.copy()
    v0, z0, b0, a0 = 2 * cfg.key_dim, cfg.qkv_dim, cfg.qkv_dim + cfg.inner, cfg.qkv_dim + cfg.inner + hv
    for p in range(hv):
        h = inv[p]
        new[v0 + p * d: v0 + (p + 1) * d] = rows[v0 + h * d: v0 + (h + 1) * d]
        new[z0 + p * d: z0 + (p + 1) * d] = rows[z0 + h * d: z0 + (h + 1) * d]
        new[b0 + p] = b0 + h
        new[a0 + p] = a0 + h
    tp = synth.LayerTensors(cfg, 8, np.ascontiguousarray(qkvz[new]), None, None, None, None, t.head_norm)
    conv = t.conv1d_w.copy()
    for p in range(hv):
        h = inv[p]
        conv[v0 + p * d: v0 + (p + 1) * d] = t.conv1d_w[v0 + h * d: v0 + (h + 1) * d]
    tp.conv1d_w = conv
    tp.ssm_a = np.ascontiguousarray(t.ssm_a[inv])
    tp.dt_bias = np.ascontiguousarray(t.dt_bias[inv])
    # out_proj columns follow the permuted gated vector
    Wout = synth.q8_0_dequant_np(t.out_proj, cfg.hidden, cfg.inner)  # only used for the block permutation
    ob = t.out_proj.reshape(cfg.hidden, cfg.inner // 32, 34)
    cols = np.concatenate([np.arange(h * d // 32, (h + 1) * d // 32) for h in inv])
    tp.out_proj = np.ascontiguousarray(ob[:, cols, :].reshape(cfg.hidden, -1))
    assert Wout.shape == (cfg.hidden, cfg.inner)
    xs = synth.hidden_states(4, cfg.hidden, seed=8)
    S_i = np.zeros((hv, d, d), np.float32)
    S_g = S_i.copy()
    c_i = np.zeros((4, cfg.qkv_dim), np.float32)
    c_g = c_i.copy()
    p_i = np.zeros(1, np.int32)
    p_g = p_i.copy()
    for x in xs:
        a = O.port().deltanet_forward(cfg, x, S_i, c_i, p_i, t, act_mode=O.ACT_FP32, head_map=1)
        b = O.ref().deltanet_forward(cfg, x, S_g, c_g, p_g, tp, act_mode=O.ACT_FP32)
        # out_proj sums the permuted columns in another order: compare by rel-L2
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-6
    assert np.linalg.norm(S_i - S_g[perm]) / np.linalg.norm(S_g) < 1e-6
