"""ctypes binding of winmoe_b200/libwinmoe_gdn.so (include/winmoe_gdn.h).

The library is the only compute path: if it is missing or fails to load,
every entry point raises -- there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libwinmoe_gdn.so"

GDN_OK = 0
STATUS_NAMES = {
    0: "GDN_OK", -1: "GDN_ERR_CUDA", -2: "GDN_ERR_SHAPE", -3: "GDN_ERR_TYPE",
    -4: "GDN_ERR_TIMEOUT", -5: "GDN_ERR_STATE", -6: "GDN_ERR_ARG", -7: "GDN_ERR_NOMEM",
}
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
GGML_F32, GGML_Q8_0, GGML_Q4_K = 0, 8, 12
HEAD_MAP_GROUPED, HEAD_MAP_INTERLEAVED = 0, 1
GEMM_EXACT, GEMM_FAST, GEMM_REF_EXACT = 0, 1, 2


class GDNError(RuntimeError):
    """A gdn_* call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class gdn_dims(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("num_k_heads", C.c_int32),
                ("num_v_heads", C.c_int32), ("head_dim", C.c_int32)]


class gdn_layer(C.Structure):
    _fields_ = [
        ("dims", gdn_dims), ("weight_type", C.c_int32), ("head_map", C.c_int32),
        ("in_qs", C.c_void_p), ("in_d", C.c_void_p), ("out_qs", C.c_void_p), ("out_d", C.c_void_p),
        ("in_blocks", C.c_void_p), ("out_blocks", C.c_void_p),
        ("conv1d_w", C.c_void_p), ("ssm_a", C.c_void_p), ("dt_bias", C.c_void_p), ("head_norm", C.c_void_p),
    ]


class gdn_dn_state(C.Structure):
    _fields_ = [("S", C.c_void_p), ("conv_buf", C.c_void_p), ("conv_pos", C.c_void_p)]


_vp, _i64, _int, _sz = C.c_void_p, C.c_int64, C.c_int, C.c_size_t

# name -> (restype, argtypes) for every entry point of include/*.h
SIGNATURES = {
    "gdn_last_error": (C.c_char_p, []),
    "gdn_abi_version": (_int, []),
    "gdn_check_device_error": (_int, [_vp]),
    "gdn_q8_0_repack": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "gdn_q8_0_dequant": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "gdn_q8_0_gemm": (_int, [_vp, _vp, _i64, _i64, _vp, _int, _i64, _vp, _int, _vp]),
    "gdn_q4_k_dequant": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "gdn_q4_k_gemm": (_int, [_vp, _i64, _i64, _vp, _int, _i64, _vp, _vp]),
    "gdn_q5_k_dequant": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "gdn_q5_k_gemm": (_int, [_vp, _i64, _i64, _vp, _int, _i64, _vp, _vp]),
    "gdn_expert_ffn_workspace_size": (_sz, [_i64, _i64, _i64]),
    "gdn_expert_ffn": (_int, [_vp, _vp, _vp, _int, _int, _i64, _i64, _vp, _int, _i64, _vp, C.c_float, _int, _vp,
                              _sz, _vp]),
    "gdn_experts_ffn_workspace_size": (_sz, [_int, _i64, _i64, _i64]),
    "gdn_experts_ffn": (_int, [_int, _vp, _vp, _vp, _int, _int, _i64, _i64, _vp, _int, _i64, _vp, _vp, _int, _vp,
                               _sz, _vp]),
    "gdn_decode_workspace_size": (_sz, [C.POINTER(gdn_dims), _i64]),
    "gdn_decode_step": (_int, [C.POINTER(gdn_layer), _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gdn_decode_step_ex": (_int, [C.POINTER(gdn_layer), _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, _sz, _int, _vp]),
    "gdn_decode_step_noalloc": (_int, [C.POINTER(gdn_layer), _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp]),
    "gdn_quantize_q8_K": (_int, [_vp, _vp, _i64, _vp]),
    "gdn_prefill_workspace_size": (_sz, [C.POINTER(gdn_dims), _i64]),
    "gdn_prefill_gated": (_int, [C.POINTER(gdn_layer), _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gdn_out_proj_gathered": (_int, [_vp, _vp, _i64, _i64, _vp, _int, _i64, _i64, _i64, _vp, _vp]),
    "gdn_add_rmsnorm": (_int, [_vp, _vp, _vp, _vp, _int, _i64, _i64, _vp]),
    "gdn_add_rmsnorm_bcast": (_int, [_vp, _vp, _vp, C.POINTER(_vp), _int, _int, _i64, _i64, _i64, _vp]),
    "gdn_prefill_scatter": (_int, [C.POINTER(gdn_layer), _i64, _vp, _int, C.POINTER(_vp), _int, _i64, _i64, _vp, _vp,
                                   _vp, _vp, _sz, _vp]),
    "gdn_out_proj_blocks": (_int, [_vp, _vp, _i64, _i64, C.POINTER(_vp), _int, _i64, _i64, _i64, _vp, _vp]),
    "gdn_ipc_alloc": (_int, [_sz, C.POINTER(_vp), _vp]),
    "gdn_ipc_open": (_int, [_vp, C.POINTER(_vp)]),
    "gdn_ipc_close": (_int, [_vp]),
    "gdn_ipc_free": (_int, [_vp]),
    "gdn_prefill": (_int, [C.POINTER(gdn_layer), _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gdn_dn_init_dims": (_int, [_int, _int, _int]),
    "gdn_layer_forward": (_int, [_vp, _vp, C.POINTER(gdn_dn_state)] + [_vp, _int] * 5 + [_vp] * 4
                          + [_int, _i64, _i64, _vp]),
    "gdn_layer_release": (_int, [_vp]),
    "gdn_layer_release_all": (_int, []),
    "gdn_offload_experts_linked": (_int, []),
    "gdn_profile_enable": (_int, [_int]),
    "gdn_decode_phase_ms": (_int, [C.POINTER(C.c_float), _int]),
    "gpu_init": (_int, []),
    "gpu_shutdown": (None, []),
    "gpu_is_initialized": (_int, []),
    "gpu_vram_used_mb": (C.c_float, []),
    "gpu_upload_deltanet_weights": (_int, [_int, _vp, _int, _int, _vp, _int, _int, _vp, _int, _int]),
    "gpu_deltanet_projections": (_int, [_int, _vp, _int, _vp, _int, _vp, _int]),
    "gpu_ssm_out_projection": (_int, [_int, _vp, _int, _vp, _int]),
    "gpu_upload_gqa_weights": (_int, [_int, _vp, _int, _int, _vp, _int, _int, _vp, _int, _int, _vp, _int, _int]),
    "gpu_gqa_projections": (_int, [_int, _vp, _int, _vp, _int, _vp, _int, _vp, _int]),
    "gpu_gqa_output": (_int, [_int, _vp, _int, _vp, _int]),
    "gpu_launch_qkv_gate": (_int, [_int, _int, _vp, _int, _int, _int]),
    "gpu_wait_qkv_gate": (_int, [_int]),
    "gpu_launch_ssm_out": (_int, [_int, _int, _vp, _int, _int]),
    "gpu_wait_ssm_out": (_int, [_int]),
    "gpu_get_qkv_out": (C.POINTER(C.c_float), [_int]),
    "gpu_get_gate_out": (C.POINTER(C.c_float), [_int]),
    "gpu_get_ssm_out_buf": (C.POINTER(C.c_float), [_int]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Loads the library once; raises if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = Path(os.environ.get("WINMOE_GDN_LIB", LIB_PATH))
            if not path.exists():
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m winmoe_b200.build` "
                    "(the CUDA library is the only compute path)")
            h = C.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                f = getattr(h, name)
                f.restype = res
                f.argtypes = args
            _lib = h
    return _lib


def last_error() -> str:
    msg = lib().gdn_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status != GDN_OK:
        raise GDNError(status, last_error())
