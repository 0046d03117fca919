"""gdn_decode_step_noalloc (fixed static scratch, no allocation) against
gdn_decode_step (caller workspace), both called through the C ABI.

Both run the same kernels in the same order on identically carved scratch, so
outputs, S, the conv window and conv_pos must be bit-identical, on two decode
tokens in a row.  A larger batch followed by a smaller one through the shared
scratch shows any byte a call reads without writing it first (stale data of
the previous call).  The file name sorts last so it also runs after every
other GPU test; it passes on its own in a fresh process too (the first call
sets up the scratch).
"""
import ctypes as C

import pytest
import torch

from winmoe_b200 import GDNConfig, layer as L, synth
from winmoe_b200._lib import check, gdn_dims, lib
from winmoe_b200.config import DIMS_35B

pytestmark = pytest.mark.gpu
DEV = "cuda"
DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
SCRATCH_BYTES = 8 << 20  # GDN_NOALLOC_SCRATCH_BYTES


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def setup(cfg, batch):
    t = synth.layer_tensors(cfg, layer=2)
    w = L.DeltaNetWeights.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                                 device=DEV)
    st = L.DeltaNetState.zeros(cfg, batch, DEV)
    for b in range(batch):
        st.S[b] = torch.from_numpy(synth.prefilled_state(cfg, b))
    return w, st


def step_workspace(w, st, x, out):
    """The existing entry point with a caller workspace."""
    cfg = w.cfg
    dims = gdn_dims(cfg.hidden, cfg.num_k_heads, cfg.num_v_heads, cfg.head_dim)
    ws = torch.empty(lib().gdn_decode_workspace_size(C.byref(dims), x.shape[0]), dtype=torch.uint8, device=DEV)
    check(lib().gdn_decode_step(C.byref(w.struct()), x.shape[0], x.data_ptr(), DTYPES[x.dtype], out.data_ptr(),
                                st.S.data_ptr(), st.conv_buf.data_ptr(), st.conv_pos.data_ptr(), ws.data_ptr(),
                                ws.numel(), stream()))


def step_noalloc(w, st, x, out):
    return lib().gdn_decode_step_noalloc(C.byref(w.struct()), x.shape[0], x.data_ptr(), DTYPES[x.dtype],
                                         out.data_ptr(), st.S.data_ptr(), st.conv_buf.data_ptr(),
                                         st.conv_pos.data_ptr(), stream())


def two_steps_identical(cfg, batch, dtype, seed):
    w, st_ref = setup(cfg, batch)
    st_new = st_ref.clone()
    gen = torch.Generator().manual_seed(seed)
    for _ in range(2):
        x = torch.randn((batch, cfg.hidden), generator=gen).to(dtype).to(DEV)
        y_ref = torch.empty((batch, cfg.hidden), dtype=torch.float32, device=DEV)
        y_new = torch.full_like(y_ref, float("nan"))
        step_workspace(w, st_ref, x, y_ref)
        check(step_noalloc(w, st_new, x, y_new))
        torch.cuda.synchronize()
        assert torch.equal(y_new, y_ref)
        assert torch.equal(st_new.S, st_ref.S)
        assert torch.equal(st_new.conv_buf, st_ref.conv_buf)
        assert torch.equal(st_new.conv_pos, st_ref.conv_pos)
    assert lib().gdn_check_device_error(stream()) == 0


@pytest.mark.parametrize("cfg,batch,dtype", [
    (DIMS_35B, 1, torch.float32),                    # the reference engine's single-sequence decode
    (DIMS_35B, 8, torch.bfloat16),                   # CUDA-core projections
    (DIMS_35B, 32, torch.bfloat16),                  # tensor-core projections and split-K out_proj
    (DIMS_35B, 46, torch.float16),                   # the largest 35B 16-bit batch the scratch holds
    (DIMS_35B, 63, torch.float32),                   # the largest 35B fp32 batch (CUDA-core projections)
    (GDNConfig(512, 2, 4, 128), 64, torch.bfloat16),  # tensor-core projections and split-K out_proj
])
def test_noalloc_matches_workspace_entry(cfg, batch, dtype):
    two_steps_identical(cfg, batch, dtype, seed=batch)


def test_noalloc_larger_then_smaller_batch():
    """The scratch keeps the previous call's bytes: a smaller batch after a larger
    one must still match the workspace entry point bit for bit."""
    two_steps_identical(DIMS_35B, 40, torch.bfloat16, seed=1)
    two_steps_identical(DIMS_35B, 3, torch.float32, seed=2)
    two_steps_identical(GDNConfig(512, 2, 4, 128), 96, torch.bfloat16, seed=3)
    two_steps_identical(GDNConfig(512, 2, 4, 128), 5, torch.float32, seed=4)


@pytest.mark.parametrize("batch,dtype", [(64, torch.float32), (47, torch.bfloat16)])
def test_noalloc_rejects_batches_above_the_scratch(batch, dtype):
    # fp32 x: from 64 sequences the 35B out_proj splits K; 16-bit x: from 5, and
    # from 47 its partials no longer fit
    cfg = DIMS_35B
    dims = gdn_dims(cfg.hidden, cfg.num_k_heads, cfg.num_v_heads, cfg.head_dim)
    assert lib().gdn_decode_workspace_size(C.byref(dims), batch) > SCRATCH_BYTES
    w, st = setup(cfg, batch)
    x = torch.zeros((batch, cfg.hidden), dtype=dtype, device=DEV)
    y = torch.zeros_like(x)
    S0 = st.S.clone()
    rc = step_noalloc(w, st, x, y)
    assert rc == -2  # GDN_ERR_SHAPE
    assert "scratch" in lib().gdn_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(st.S, S0) and int(st.conv_pos.sum()) == 0  # nothing ran
