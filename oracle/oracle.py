"""TEST INFRASTRUCTURE ONLY -- the CPU oracle's Python side.

Only tests/, __graft_entry__.smoke() and the cpu_baseline / --impl reference
legs of bench.py may import this module, and only as the checker or the timed
CPU baseline; the product (winmoe_b200/) never does.

Two libraries, both built by oracle/Makefile:
  port  oracle/libgdn_oracle.so   -- the plain-C restatement (gdn_oracle.c)
  ref   oracle/_ref/libref_gdn.so -- the reference's own CPU code, compiled in
        place from the reference tree (ref_exact.c: unmodified dispatch,
        int8 Q8_K activations; ref_fp32act.c: fp32-activation projections).
The ref library needs AVX-512F/BW/VL/DQ + AVX512-VNNI; ref_available() checks
the host before loading it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_PATH = HERE / "libgdn_oracle.so"
REF_PATH = HERE / "_ref" / "libref_gdn.so"
REF_ISA = ("avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512_vnni", "fma", "f16c", "avx2")

ACT_EXACT, ACT_FP32 = 0, 1

_vp, _i, _l = C.c_void_p, C.c_int, C.c_long


def ref_dir() -> Path | None:
    """The reference tree whose headers the ref library compiles in place:
    $REF_DIR, else a `reference` directory beside this repository; None when
    neither holds engine/runtime/deltanet_impl.h."""
    env = os.environ.get("REF_DIR")
    cand = Path(env) if env else HERE.parent.parent / "reference"
    return cand if (cand / "engine" / "runtime" / "deltanet_impl.h").is_file() else None


def build(ref: bool | None = None) -> None:
    """Runs oracle/Makefile (port always; ref when the reference tree exists)."""
    target = [] if ref is None else (["port", "ref"] if ref else ["port"])
    rd = ref_dir()
    args = [f"REF_DIR={rd}"] if rd is not None else []
    r = subprocess.run(["make", "-s", "-C", str(HERE), *args, *target], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")


def host_isa_ok() -> bool:
    try:
        flags = Path("/proc/cpuinfo").read_text().split("flags", 2)[1].split("\n", 1)[0].split()
    except (OSError, IndexError):
        return False
    return all(f in flags for f in REF_ISA)


def ref_available() -> bool:
    return REF_PATH.exists() and host_isa_ok()


def _f(a: np.ndarray):
    return a.ctypes.data_as(_vp)


class Port:
    """ctypes view of libgdn_oracle.so (names orc_*, see gdn_oracle.c)."""

    def __init__(self, path: Path = PORT_PATH):
        if not path.exists():
            build(ref=False)
        self.h = C.CDLL(str(path))
        h = self.h
        h.orc_fp16_to_fp32.restype = C.c_float
        h.orc_fp16_to_fp32.argtypes = [C.c_uint16]
        for n in ("orc_q8_0_dequant", "orc_q4_k_dequant", "orc_q5_k_dequant", "orc_quantize_row_q8_K"):
            getattr(h, n).argtypes = [_vp, _vp, _l]
        h.orc_q8_0_matvec.argtypes = [_vp, _vp, _vp, _i, _i, _i]
        h.orc_q4_k_matvec.argtypes = [_vp, _vp, _vp, _i, _i, _i]
        h.orc_q5_k_matvec.argtypes = [_vp, _vp, _vp, _i, _i, _i]
        h.orc_expert_ffn.argtypes = [_vp] * 5 + [_i] * 4 + [C.c_float, _i, _i]
        h.orc_quant_matvec.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i]
        h.orc_q4_k_scales.argtypes = [_vp, _vp, _vp]
        h.orc_rmsnorm.argtypes = [_vp, _vp, _vp, _i]
        h.orc_gdn_core.argtypes = [_i, _i, _i, _i, _i] + [_vp] * 15
        h.orc_deltanet_forward.argtypes = [_i] * 6 + [_vp] * 5 + [_vp, _i] * 5 + [_vp] * 4

    def q8_0_dequant(self, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.h.orc_q8_0_dequant(_f(out), _f(np.ascontiguousarray(blocks)), n)
        return out

    def q4_k_dequant(self, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.h.orc_q4_k_dequant(_f(out), _f(np.ascontiguousarray(blocks)), n)
        return out

    def q5_k_dequant(self, blocks: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.h.orc_q5_k_dequant(_f(out), _f(np.ascontiguousarray(blocks)), n)
        return out

    def quantize_q8_K(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * 292, np.uint8)
        self.h.orc_quantize_row_q8_K(_f(out), _f(x), x.size)
        return out

    def expert_ffn(self, x, w_gate, w_up, w_down, gate_type: int, down_type: int, hidden: int, inter: int,
                   weight: float = 1.0, out: np.ndarray | None = None, act_mode: int = ACT_FP32) -> np.ndarray:
        """One expert's gate / up / SwiGLU / down for one token (gpu_expert_ffn_fused);
        with `out` given, out += weight * y, else a new y."""
        acc = out is not None
        if out is None:
            out = np.empty(hidden, np.float32)
        self.h.orc_expert_ffn(_f(out), _f(np.ascontiguousarray(x, np.float32)), _f(np.ascontiguousarray(w_gate)),
                              _f(np.ascontiguousarray(w_up)), _f(np.ascontiguousarray(w_down)), gate_type,
                              down_type, hidden, inter, weight, int(acc), act_mode)
        return out

    def quant_matvec(self, W: np.ndarray, x: np.ndarray, out_dim: int, in_dim: int, wtype: int,
                     act_mode: int) -> np.ndarray:
        out = np.empty(out_dim, np.float32)
        self.h.orc_quant_matvec(_f(out), _f(np.ascontiguousarray(W)), _f(np.ascontiguousarray(x, np.float32)),
                                out_dim, in_dim, wtype, act_mode)
        return out

    def rmsnorm(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.h.orc_rmsnorm(_f(out), _f(x), _f(np.ascontiguousarray(w, np.float32)), x.size)
        return out

    def deltanet_forward(self, cfg, x, S, conv_buf, conv_pos, tensors, act_mode=ACT_FP32, head_map=0) -> np.ndarray:
        """One token; S [Hv,d,d], conv_buf [4,QKV] float32 and conv_pos (1-elem int32) updated in place."""
        parts = tensors.split_in_proj()
        out = np.empty(cfg.hidden, np.float32)
        wt = tensors.weight_type
        self.h.orc_deltanet_forward(
            cfg.hidden, cfg.inner, cfg.num_k_heads, cfg.head_dim, act_mode, head_map,
            _f(out), _f(np.ascontiguousarray(x, np.float32)), _f(S), _f(conv_buf), _f(conv_pos),
            _f(parts["w_qkv"]), wt, _f(parts["w_gate"]), wt, _f(parts["w_alpha"]), wt, _f(parts["w_beta"]), wt,
            _f(tensors.out_proj), wt, _f(tensors.conv1d_w), _f(tensors.ssm_a), _f(tensors.dt_bias),
            _f(tensors.head_norm))
        return out

    def gdn_core(self, cfg, qkv, z, alpha_raw, beta_raw, S, conv_buf, conv_pos, tensors, head_map=0):
        """The layer between projections and out_proj; returns (gated, decay, beta, head_out)."""
        qkv = np.ascontiguousarray(qkv, np.float32).copy()
        gated = np.empty(cfg.inner, np.float32)
        decay = np.empty(cfg.num_v_heads, np.float32)
        beta = np.empty(cfg.num_v_heads, np.float32)
        ho = np.empty(cfg.inner, np.float32)
        self.h.orc_gdn_core(cfg.hidden, cfg.inner, cfg.num_k_heads, cfg.head_dim, head_map, _f(qkv),
                            _f(np.ascontiguousarray(z, np.float32)), _f(np.ascontiguousarray(alpha_raw, np.float32)),
                            _f(np.ascontiguousarray(beta_raw, np.float32)), _f(S), _f(conv_buf), _f(conv_pos),
                            _f(tensors.conv1d_w), _f(tensors.ssm_a), _f(tensors.dt_bias), _f(tensors.head_norm),
                            _f(gated), _f(decay), _f(beta), _f(ho))
        return gated, decay, beta, ho, qkv


class Ref:
    """ctypes view of oracle/_ref/libref_gdn.so (the reference's CPU code)."""

    def __init__(self, path: Path = REF_PATH):
        if not host_isa_ok():
            raise RuntimeError("host CPU lacks the AVX-512 / VNNI features the reference build needs")
        self.h = C.CDLL(str(path))
        h = self.h
        for p in ("refx", "reff"):
            getattr(h, f"{p}_init_dims").argtypes = [_i, _i, _i]
            getattr(h, f"{p}_init_dims").restype = _i
            getattr(h, f"{p}_deltanet_forward").argtypes = [_vp] * 5 + [_vp, _i] * 5 + [_vp] * 4 + [_i]
            getattr(h, f"{p}_quant_matvec").argtypes = [_vp, _vp, _vp, _i, _i, _i]
        h.refx_q8_dequant_row.argtypes = [_vp, _vp, _i]
        h.refx_quantize_row_q8_K.argtypes = [_vp, _vp, _i]
        h.refx_decode_q4k_scales.argtypes = [_vp, _vp, _vp]
        h.refx_q4k_matvec.argtypes = [_vp, _vp, _vp, _i, _i]
        h.refx_q4k_dot_block.argtypes = [_vp, _vp]
        h.refx_q4k_dot_block.restype = C.c_float
        h.refx_fp16_to_fp32.argtypes = [C.c_uint16]
        h.refx_fp16_to_fp32.restype = C.c_float
        h.refx_rmsnorm.argtypes = [_vp, _vp, _vp, _i]
        self._dims = None

    def init_dims(self, cfg) -> None:
        if self._dims != cfg:
            self.h.refx_init_dims(cfg.inner, cfg.num_k_heads, cfg.head_dim)
            self.h.reff_init_dims(cfg.inner, cfg.num_k_heads, cfg.head_dim)
            self._dims = cfg

    def deltanet_forward(self, cfg, x, S, conv_buf, conv_pos, tensors, act_mode=ACT_FP32) -> np.ndarray:
        self.init_dims(cfg)
        parts = tensors.split_in_proj()
        out = np.empty(cfg.hidden, np.float32)
        wt = tensors.weight_type
        fn = self.h.reff_deltanet_forward if act_mode == ACT_FP32 else self.h.refx_deltanet_forward
        fn(_f(out), _f(np.ascontiguousarray(x, np.float32)), _f(S), _f(conv_buf), _f(conv_pos),
           _f(parts["w_qkv"]), wt, _f(parts["w_gate"]), wt, _f(parts["w_alpha"]), wt, _f(parts["w_beta"]), wt,
           _f(tensors.out_proj), wt, _f(tensors.conv1d_w), _f(tensors.ssm_a), _f(tensors.dt_bias),
           _f(tensors.head_norm), cfg.hidden)
        return out

    def quant_matvec(self, W, x, out_dim, in_dim, wtype, act_mode) -> np.ndarray:
        out = np.empty(out_dim, np.float32)
        fn = self.h.reff_quant_matvec if act_mode == ACT_FP32 else self.h.refx_quant_matvec
        fn(_f(out), _f(np.ascontiguousarray(W)), _f(np.ascontiguousarray(x, np.float32)), out_dim, in_dim, wtype)
        return out

    def q8_0_dequant(self, blocks, n) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.h.refx_q8_dequant_row(_f(out), _f(np.ascontiguousarray(blocks)), n)
        return out

    def quantize_q8_K(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 256 * 292, np.uint8)
        self.h.refx_quantize_row_q8_K(_f(out), _f(x), x.size)
        return out

    def q4k_scales(self, q12: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        sc = np.zeros(8, np.uint8)
        mn = np.zeros(8, np.uint8)
        self.h.refx_decode_q4k_scales(_f(np.ascontiguousarray(q12, np.uint8)), _f(sc), _f(mn))
        return sc, mn

    def q4k_dot_block(self, block: np.ndarray, y: np.ndarray) -> float:
        return float(self.h.refx_q4k_dot_block(_f(np.ascontiguousarray(block, np.uint8)),
                                               _f(np.ascontiguousarray(y, np.float32))))

    def rmsnorm(self, x, w) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.h.refx_rmsnorm(_f(out), _f(x), _f(np.ascontiguousarray(w, np.float32)), x.size)
        return out

    def gguf_probe(self, path) -> dict:
        """The reference parser's view of a GGUF file (parse_gguf, gguf_parser.h:149-250)."""
        meta = (C.c_longlong * 8)()
        rc = self.h.refx_gguf_probe(str(path).encode(), meta)
        if rc != 0:
            raise OSError(f"parse_gguf returned {rc}")
        keys = ("n_tensors", "hidden", "ssm_inner", "ssm_groups", "ssm_state", "ssm_conv", "layers", "data_start")
        return dict(zip(keys, list(meta)))

    def gguf_tensor(self, path, name: str) -> dict:
        """find_tensor (gguf_parser.h:350-358): type, dims, offset of `name`."""
        info = (C.c_longlong * 7)()
        rc = self.h.refx_gguf_tensor(str(path).encode(), name.encode(), info)
        if rc != 0:
            raise KeyError(f"{name}: reference parser rc {rc}")
        return {"type": info[0], "dims": tuple(info[2:2 + info[1]]), "offset": info[6]}


_port: Port | None = None
_ref: Ref | None = None



def port() -> Port:
    global _port
    if _port is None:
        _port = Port()
    return _port


def ref() -> Ref:
    global _ref
    if _ref is None:
        _ref = Ref()
    return _ref


def best():
    """The reference build when this host can run it, else the port (tests and baselines)."""
    return ref() if ref_available() else port()


def omp_threads() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
