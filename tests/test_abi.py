"""The C ABI without a GPU: the library loads, exports every entry point that
include/*.h declares, and rejects bad arguments with a status and a message
before touching CUDA."""
import ctypes as C
import re
from pathlib import Path

import pytest

from winmoe_b200 import _lib
from winmoe_b200._lib import lib

ROOT = Path(__file__).resolve().parent.parent
DECL = re.compile(r"^(?:GDN_API|GDN_LEGACY_API)\s+[\w\s\*]+?\b(\w+)\s*\(", re.M)


def declared():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += DECL.findall(h.read_text())
    return names


def test_headers_declare_the_expected_entry_points():
    names = set(declared())
    assert {"gdn_decode_step", "gdn_q8_0_gemm", "gdn_q4_k_gemm", "gpu_init", "gpu_launch_qkv_gate"} <= names
    assert len(names) == len(declared())  # no duplicates


@pytest.mark.parametrize("name", declared())
def test_symbol_exported(name):
    assert hasattr(lib(), name), name


def test_bindings_cover_every_declaration():
    assert set(declared()) == set(_lib.SIGNATURES)


def test_abi_version():
    assert lib().gdn_abi_version() >= 100


def test_shape_errors_need_no_gpu():
    h = lib()
    buf = C.create_string_buffer(64)
    vp = C.cast(buf, C.c_void_p)
    assert h.gdn_q8_0_repack(vp, vp, vp, 1, 33, None) == -2
    assert "cols" in _lib.last_error()
    assert h.gdn_q8_0_gemm(vp, vp, 4, 0, vp, 0, 1, vp, 0, None) == -2
    assert h.gdn_q8_0_gemm(None, vp, 4, 32, vp, 0, 1, vp, 0, None) == -6
    assert h.gdn_q8_0_gemm(vp, vp, 4, 32, vp, 9, 1, vp, 0, None) == -3
    assert h.gdn_q4_k_gemm(vp, 4, 100, vp, 0, 1, vp, None) == -2
    assert h.gdn_q4_k_dequant(vp, vp, 1, 255, None) == -2


def test_layer_validation_errors():
    h = lib()
    dims = _lib.gdn_dims(2048, 16, 32, 64)
    layer = _lib.gdn_layer(dims, 8, 0)
    x = C.create_string_buffer(256)
    vp = C.cast(x, C.c_void_p)
    assert h.gdn_decode_step(None, 1, vp, 0, vp, vp, vp, vp, vp, 0, None) == -6
    assert h.gdn_decode_step(C.byref(layer), 1, vp, 0, vp, vp, vp, vp, vp, 0, None) == -2
    assert "head_dim" in _lib.last_error()
    layer.dims = _lib.gdn_dims(2048, 16, 30, 128)
    assert h.gdn_decode_step(C.byref(layer), 1, vp, 0, vp, vp, vp, vp, vp, 0, None) == -2
    layer.dims = _lib.gdn_dims(2048, 16, 32, 128)
    layer.weight_type = 3
    assert h.gdn_decode_step(C.byref(layer), 1, vp, 0, vp, vp, vp, vp, vp, 0, None) == -3
    layer.weight_type = 8
    assert h.gdn_decode_step(C.byref(layer), 1, vp, 0, vp, vp, vp, vp, vp, 0, None) == -6  # NULL planes


def test_workspace_size_grows_with_batch():
    h = lib()
    dims = _lib.gdn_dims(2048, 16, 32, 128)
    w1 = h.gdn_decode_workspace_size(C.byref(dims), 1)
    w256 = h.gdn_decode_workspace_size(C.byref(dims), 256)
    assert 0 < w1 < w256
    assert w256 % 256 == 0
    assert h.gdn_decode_workspace_size(C.byref(dims), 0) == 0
    # the proj buffer alone: 256 x (QKV + inner + 2 Hv) floats
    assert w256 >= 256 * (8192 + 4096 + 64) * 4


def test_legacy_api_before_init():
    h = lib()
    assert h.gpu_is_initialized() == 0
    x = (C.c_float * 8)()
    assert h.gpu_launch_qkv_gate(0, 0, C.cast(x, C.c_void_p), 8, 8, 8) == -1
    assert "gpu_init" in _lib.last_error()
    assert h.gpu_wait_qkv_gate(0) == -1
    assert h.gpu_upload_deltanet_weights(0, None, 1, 1, None, 1, 1, None, 1, 1) == -1
    assert h.gpu_upload_gqa_weights(0, None, 1, 1, None, 1, 1, None, 1, 1, None, 1, 1) == -1
    assert h.gpu_gqa_projections(0, C.cast(x, C.c_void_p), 8, C.cast(x, C.c_void_p), 8, C.cast(x, C.c_void_p), 8,
                                 C.cast(x, C.c_void_p), 8) == -1
    assert h.gpu_gqa_output(0, C.cast(x, C.c_void_p), 8, C.cast(x, C.c_void_p), 8) == -1
    assert not h.gpu_get_qkv_out(5)
    assert h.gpu_vram_used_mb() == 0.0
