"""GPU parity of the GGUF quant kernels against the CPU oracle.

Bit-exact: Q8_0 / Q4_K dequantised weights (the north-star requirement).
Tolerances: CUDA-core GEMVs with fp32 activations vs the oracle's
fp32-activation projections, rel-L2 <= 1e-5 (only the summation order
differs).  The tcgen05 GEMM, exact mode (hi + lo weight operands): vs the
fp64 product of the same activations and fp32 weights, rel-L2 <= 1e-5; fast
mode (one operand): vs the product with weights rounded once to the
activation type, rel-L2 <= 1e-5, and vs fp32 weights within that rounding.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from winmoe_b200 import layer as L, synth

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("rows,cols", [(96, 256), (12352, 2048), (2048, 4096), (7, 32)])
def test_q8_0_dequant_bit_exact(rows, cols):
    blocks = synth.q8_0_blocks(rows, cols, seed=100 + rows)
    qs, d = L.q8_0_planes(blocks, rows, cols, DEV)
    got = L.dequant_q8_0(qs, d).cpu().numpy()
    want = O.port().q8_0_dequant(blocks, rows * cols).reshape(rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    qs_np, d_np = synth.q8_0_split(blocks, rows, cols)
    assert np.array_equal(qs.cpu().numpy(), qs_np)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), d_np)


@pytest.mark.parametrize("rows,cols", [(64, 512), (12352, 2048), (2048, 4096), (3, 256)])
def test_q4_k_dequant_bit_exact(rows, cols):
    blocks = synth.q4_k_blocks(rows, cols, seed=200 + rows)
    dev = torch.from_numpy(blocks.reshape(-1)).to(DEV)
    got = L.dequant_q4_k(dev, rows, cols).cpu().numpy()
    want = O.port().q4_k_dequant(blocks, rows * cols).reshape(rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13, 32])
@pytest.mark.parametrize("n,k", [(12352, 2048), (2048, 4096), (50, 96)])
def test_q8_0_gemv_fp32(m, n, k):
    blocks = synth.q8_0_blocks(n, k, seed=300 + n)
    x = synth.hidden_states(m, k, seed=301)
    qs, d = L.q8_0_planes(blocks, n, k, DEV)
    y = L.gemm_q8_0(qs, d, torch.from_numpy(x).to(DEV)).cpu().numpy()
    P = O.port()
    for i in range(m):
        want = P.quant_matvec(blocks, x[i], n, k, 8, O.ACT_FP32)
        assert rel_l2(y[i], want) <= 1e-5, i


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13, 16, 32])
@pytest.mark.parametrize("n,k", [(12352, 2048), (2048, 4096), (64, 2048), (300, 256), (200, 768)])
def test_q4_k_gemv_fp32(m, n, k):
    blocks = synth.q4_k_blocks(n, k, seed=400 + n)
    x = synth.hidden_states(m, k, seed=401)
    dev = torch.from_numpy(blocks.reshape(-1)).to(DEV)
    y = L.gemm_q4_k(dev, n, k, torch.from_numpy(x).to(DEV)).cpu().numpy()
    P = O.port()
    for i in range(m):
        want = P.quant_matvec(blocks, x[i], n, k, 12, O.ACT_FP32)
        assert rel_l2(y[i], want) <= 1e-5, i


def _edge_activations(k):
    """Activation rows whose 32-blocks test the streamed GEMV's split of x into
    int8 levels: all-zero blocks, a lone outlier, and rows scaled near and far
    below 2^-64 (where the block scale is formed from x * 2^64)."""
    x = synth.hidden_states(4, k, seed=501).astype(np.float32)
    x[0, :64] = 0.0           # two zero blocks
    x[0, 100] = 3.0e4         # an outlier in its block
    x[1] *= np.float32(1e-30)  # every block scaled below 2^-64
    x[2, ::2] *= np.float32(1e-20)  # blocks straddling 2^-64: tiny and ordinary values mixed
    x[3, 32:64] = np.float32(-7.5)  # a constant block
    return x


@pytest.mark.parametrize("fmt", ["q8_0", "q4_k"])
def test_gemv_edge_activations(fmt):
    n, k = 2048, 2048
    x = _edge_activations(k)
    P = O.port()
    if fmt == "q8_0":
        blocks = synth.q8_0_blocks(n, k, seed=502)
        qs, d = L.q8_0_planes(blocks, n, k, DEV)
        run = lambda xi: L.gemm_q8_0(qs, d, xi)
        ty = 8
    else:
        blocks = synth.q4_k_blocks(n, k, seed=503)
        dev = torch.from_numpy(blocks.reshape(-1)).to(DEV)
        run = lambda xi: L.gemm_q4_k(dev, n, k, xi)
        ty = 12
    for i in range(x.shape[0]):  # one row per call: the batch-1 streamed path
        y = run(torch.from_numpy(x[i:i + 1]).to(DEV)).cpu().numpy()[0]
        want = P.quant_matvec(blocks, x[i], n, k, ty, O.ACT_FP32)
        assert rel_l2(y, want) <= 1e-5, i
    xn = x[3:4].copy()
    xn[0, 1000] = np.nan  # a NaN activation reaches every output, as through fp32 products
    y = run(torch.from_numpy(xn).to(DEV)).cpu().numpy()[0]
    assert np.isnan(y).all()


@pytest.mark.parametrize("fmt", ["q8_0", "q4_k", "q5_k"])
def test_gemv_edge_activations_batched(fmt):
    """The same edge rows as one 4-row call: the tensor-core batch paths (IMMA for
    Q8_0; fp16 MMA for the K-quants, whose activations are split per 256-element
    piece into a power-of-two scale and fp16 hi + lo parts)."""
    n, k = 2048, 2048
    x = _edge_activations(k)
    P = O.port()
    if fmt == "q8_0":
        blocks = synth.q8_0_blocks(n, k, seed=502)
        qs, d = L.q8_0_planes(blocks, n, k, DEV)
        run = lambda xi: L.gemm_q8_0(qs, d, xi)
        ty = 8
    else:
        gen, ty = (synth.q4_k_blocks, 12) if fmt == "q4_k" else (synth.q5_k_blocks, 13)
        blocks = gen(n, k, seed=503)
        dev = torch.from_numpy(blocks.reshape(-1)).to(DEV)
        run = lambda xi: (L.gemm_q4_k if ty == 12 else L.gemm_q5_k)(dev, n, k, xi)
    y = run(torch.from_numpy(x).to(DEV)).cpu().numpy()
    for i in range(x.shape[0]):
        want = P.quant_matvec(blocks, x[i], n, k, ty, O.ACT_FP32)
        assert rel_l2(y[i], want) <= 1e-5, i
    xn = x.copy()
    xn[3, 1000] = np.nan  # reaches every output of its row only
    xn[1, 5] = np.inf  # as an inf among fp32 products of either sign: NaN (the rows' other outputs too)
    y = run(torch.from_numpy(xn).to(DEV)).cpu().numpy()
    assert np.isnan(y[3]).all() and np.isnan(y[1]).all() and np.isfinite(y[[0, 2]]).all()


@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m", [3, 5])
def test_q4_k_gemv_half_activations(xdt, m):
    """fp16 / bf16 activations below the tensor-core GEMM's batch threshold go
    through the batched GEMV: the fp32 product of the same (rounded) activations."""
    n, k = 2048, 4096
    blocks = synth.q4_k_blocks(n, k, seed=510)
    xh = torch.from_numpy(synth.hidden_states(m, k, seed=511)).to(xdt)
    y = L.gemm_q4_k(torch.from_numpy(blocks.reshape(-1)).to(DEV), n, k, xh.to(DEV)).cpu().numpy()
    P = O.port()
    x32 = xh.float().numpy()
    for i in range(m):
        assert rel_l2(y[i], P.quant_matvec(blocks, x32[i], n, k, 12, O.ACT_FP32)) <= 1e-5, i


# One M tile (m <= 128) short of one wave takes the narrowest single-wave tile: 96 weight rows for
# most of these (ragged last tile where 96 does not divide n), 128 for n = 16384 (171 tiles of 96
# would exceed one wave); m > 128 pairs two M tiles per CTA.
GEMM_SHAPES = [(128, 256, 64), (256, 12352, 2048), (256, 2048, 4096), (200, 300, 2048), (64, 128, 128),
               (1000, 12352, 2048), (4096, 2048, 4096), (130, 12288, 2048), (16, 12352, 2048), (40, 2048, 4096),
               (100, 16384, 128), (33, 1000, 256)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
def test_q8_0_gemm_tensor_core_exact(m, n, k, xdt):
    """Exact mode: the fp32 product of the same activations up to summation order
    (fp16 x: tensor cores with hi + lo weight operands; bf16 x: CUDA cores)."""
    blocks = synth.q8_0_blocks(n, k, seed=500 + n + k)
    qs, d = L.q8_0_planes(blocks, n, k, DEV)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + n + k)).to(xdt).to(DEV)
    y = L.gemm_q8_0(qs, d, x).double()
    w32 = torch.from_numpy(synth.q8_0_dequant_np(blocks, n, k)).double().to(DEV)
    want = x.double() @ w32.T
    err = ((y - want).norm() / want.norm()).item()
    assert err <= 1e-5, err
    rows_err = ((y - want).norm(dim=1) / want.norm(dim=1)).max().item()
    assert rows_err <= 1e-4, rows_err  # every row/column tile written


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
def test_q8_0_gemm_tensor_core_fast(m, n, k, xdt):
    """One weight operand: the fp32 product of weights rounded once to the x type."""
    blocks = synth.q8_0_blocks(n, k, seed=600 + n + k)
    qs, d = L.q8_0_planes(blocks, n, k, DEV)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + n + k)).to(xdt).to(DEV)
    y = L.gemm_q8_0(qs, d, x, fast=True).double()
    w = torch.from_numpy(synth.q8_0_dequant_np(blocks, n, k)).to(xdt).to(DEV)
    want = x.double() @ w.double().T
    err = ((y - want).norm() / want.norm()).item()
    assert err <= 1e-5, err
    w32 = torch.from_numpy(synth.q8_0_dequant_np(blocks, n, k)).double().to(DEV)
    want32 = x.double() @ w32.T
    assert ((y - want32).norm() / want32.norm()).item() <= (2e-3 if xdt == torch.float16 else 8e-3)


@pytest.mark.parametrize("m,n,k", [(70, 2560, 512), (128, 2560, 512), (100, 12352, 2048)])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("fast", [True, False])
def test_q8_0_gemm_tensor_core_repeatable(m, n, k, xdt, fast):
    """One-M-tile shapes (the prefill in_proj of short prompts), 12 launches in a
    row: every launch bit-identical, and every 32-column epilogue group close to
    the fp64 product (a group read out of TMEM too early shows up here)."""
    blocks = synth.q8_0_blocks(n, k, seed=700 + n + k)
    qs, d = L.q8_0_planes(blocks, n, k, DEV)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + k)).to(xdt).to(DEV)
    w = torch.from_numpy(synth.q8_0_dequant_np(blocks, n, k)).to(DEV)
    if fast:
        w = w.to(xdt)
    want = x.double() @ w.double().T
    ys = [L.gemm_q8_0(qs, d, x, fast=fast) for _ in range(12)]
    torch.cuda.synchronize()
    for i, y in enumerate(ys):
        assert torch.equal(y, ys[0]), f"launch {i} differs from launch 0"
    diff = (ys[0].double() - want).reshape(m, n // 32, 32).norm(dim=(0, 2))
    ref = want.reshape(m, n // 32, 32).norm(dim=(0, 2))
    assert (diff / ref).max().item() <= 1e-4


def test_no_device_timeout_flag():
    from winmoe_b200._lib import lib
    torch.cuda.synchronize()
    assert lib().gdn_check_device_error(None) == 0


def test_quantize_q8_K_bit_exact():
    """quantize_row_q8_K on the device = the CPU's (d, qs and bsums), incl. an all-zero block."""
    P = O.best()
    g = np.random.default_rng(17)
    x = (g.standard_normal(4 * 2048) * g.choice([1e-3, 1.0, 300.0], size=4 * 2048)).astype(np.float32)
    x[256:512] = 0.0
    want = P.quantize_q8_K(x)
    got = L.quantize_q8_K(torch.from_numpy(x).to(DEV)).cpu().numpy()
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("n,k", [(8192, 2048), (2048, 4096), (32, 2048), (100, 2048), (256, 2080)])
@pytest.mark.parametrize("m", [1, 3, 9])
def test_q8_0_gemm_ref_exact_bit_exact(n, k, m):
    """GDN_GEMM_REF_EXACT = the reference CPU's quant_matvec(type 8), bit for bit:
    Q8_K activations for n >= 128 and k % 256 == 0, fp32 block dots otherwise."""
    P = O.best()
    blocks = synth.q8_0_blocks(n, k, seed=800 + n + k)
    qs, d = L.q8_0_planes(blocks, n, k, DEV)
    x = synth.hidden_states(m, k, seed=n + m)
    y = L.gemm_q8_0(qs, d, torch.from_numpy(x).to(DEV), ref_exact=True).cpu().numpy()
    for i in range(m):
        np.testing.assert_array_equal(y[i], P.quant_matvec(blocks, x[i], n, k, 8, O.ACT_EXACT))


@pytest.mark.parametrize("m,n,k", [(8, 12352, 2048), (32, 12352, 2048), (32, 2048, 4096), (130, 2048, 4096),
                                   (40, 100, 256), (64, 300, 768)])
def test_q4_k_gemm_tensor_core_exact(m, n, k):
    """fp16 x: from 32 rows Q4_K superblocks dequantised into hi + lo fp16
    tcgen05 operands (below, the fp16-MMA GEMV) = the fp64 product of the same
    activations and the bit-exact fp32 weights up to summation order (incl.
    ragged n, one superblock, split K); two launches bit-identical."""
    blocks = synth.q4_k_blocks(n, k, seed=900 + n + k)
    dev = torch.from_numpy(blocks.reshape(-1)).to(DEV)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + n)).half().to(DEV)
    y = L.gemm_q4_k(dev, n, k, x)
    y2 = L.gemm_q4_k(dev, n, k, x)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    w = torch.from_numpy(O.port().q4_k_dequant(blocks, n * k).reshape(n, k)).double().to(DEV)
    want = x.double() @ w.T
    got = y.double()
    err = ((got - want).norm() / want.norm()).item()
    assert err <= 1e-5, err
    rows_err = ((got - want).norm(dim=1) / want.norm(dim=1)).max().item()
    assert rows_err <= 1e-4, rows_err
