"""GGUF tensor bridge: DeltaNet layers of a GGUF model file into the library.

The reference engine parses GGUF with engine/runtime/gguf_parser.h (header,
key/value pairs, tensor infos, data aligned to 32 bytes; parse_gguf :149-250)
and loads a DeltaNet layer by tensor name (engine/runtime/winmoe_inference.c
:311-392):
    blk.N.attn_qkv.weight   blk.N.attn_gate.weight   blk.N.ssm_out.weight
    blk.N.ssm_alpha.weight  blk.N.ssm_beta.weight    blk.N.ssm_a
    blk.N.ssm_dt.bias       blk.N.ssm_norm.weight    blk.N.ssm_conv1d.weight
and the dims from the keys *.embedding_length, *.ssm.inner_size,
*.ssm.group_count, *.ssm.state_size (matched by substring, as the parser
does).  `GGUFFile` reads the same structure through a read-only memory map
and hands the raw GGUF bytes of those tensors to `DeltaNetWeights` (Q8_0 /
Q4_K blocks stay as stored; the library repacks Q8_0 on the device), so a
layer of a real model file runs without changing the engine's parser.
`write_gguf` writes the format (used by the tests and to package layers).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .config import CONV_WIDTH, GDNConfig
from .synth import LayerTensors

MAGIC = b"GGUF"
ALIGNMENT = 32  # the reference parser's fixed data alignment (gguf_parser.h:241-242)

# GGUF value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}

# GGML tensor types used on this path and their (block bytes, weights per block)
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K = 0, 1, 8, 12
_BLOCK = {GGML_F32: (4, 1), GGML_F16: (2, 1), GGML_Q8_0: (34, 32), GGML_Q4_K: (144, 256)}


@dataclass
class TensorInfo:
    name: str
    ggml_type: int
    dims: tuple[int, ...]  # GGUF order: dims[0] is the innermost (row length)
    offset: int            # relative to the data section

    @property
    def nbytes(self) -> int:
        if self.ggml_type not in _BLOCK:
            raise ValueError(f"{self.name}: GGML type {self.ggml_type} is not on the DeltaNet path")
        bb, bw = _BLOCK[self.ggml_type]
        n = int(np.prod(self.dims, dtype=np.int64))
        if n % bw:
            raise ValueError(f"{self.name}: {n} weights are not whole blocks of {bw}")
        return n // bw * bb


class _Reader:
    def __init__(self, buf: memoryview):
        self.buf, self.pos = buf, 0

    def take(self, fmt: str):
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.take("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == STRING:
            return self.string()
        if vtype == ARRAY:
            etype, n = self.take("<I"), self.take("<Q")
            return [self.value(etype) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {vtype}")


class GGUFFile:
    """A GGUF file (v2/v3) opened read-only: key/values, tensor infos, raw tensor bytes."""

    def __init__(self, path):
        self.path = Path(path)
        self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        r = _Reader(memoryview(self._mm))
        if bytes(self._mm[:4]) != MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        r.pos = 4
        self.version = r.take("<I")
        n_tensors, n_kv = r.take("<Q"), r.take("<Q")
        self.kv: dict[str, object] = {}
        for _ in range(n_kv):
            key = r.string()
            self.kv[key] = r.value(r.take("<I"))
        self.tensors: dict[str, TensorInfo] = {}
        for _ in range(n_tensors):
            name = r.string()
            nd = r.take("<I")
            dims = tuple(r.take("<Q") for _ in range(nd))
            self.tensors[name] = TensorInfo(name, r.take("<I"), dims, r.take("<Q"))
        align = int(self.kv.get("general.alignment", ALIGNMENT))
        self.data_start = (r.pos + align - 1) // align * align

    def key(self, suffix: str, default=None):
        """The value of the first key containing `suffix` (the reference parser's strstr match)."""
        for k, v in self.kv.items():
            if suffix in k:
                return v
        return default

    def raw(self, name: str) -> tuple[TensorInfo, np.ndarray]:
        """Tensor info and its bytes as stored (a view of the memory map)."""
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"{self.path.name}: no tensor {name}")
        a = self.data_start + t.offset
        return t, self._mm[a:a + t.nbytes]

    def config(self) -> GDNConfig:
        """dn_init_dims from the file's keys (deltanet_impl.h:32-44)."""
        return GDNConfig.from_gguf(int(self.key("embedding_length", 0)), int(self.key("ssm.inner_size", 0)),
                                   int(self.key("ssm.group_count", 0)), int(self.key("ssm.state_size", 0)))

    def deltanet_layers(self) -> list[int]:
        """Indices of the DeltaNet layers (the reference's test: blk.N.ssm_a exists)."""
        return sorted(int(n.split(".")[1]) for n in self.tensors if n.endswith(".ssm_a") and n.startswith("blk."))

    def deltanet_layer(self, layer: int) -> tuple[GDNConfig, LayerTensors]:
        """The nine tensors of DeltaNet layer `layer` (winmoe_inference.c:311-392),
        in_proj stacked as qkv | gate | beta | alpha rows."""
        cfg = self.config()
        p = f"blk.{layer}."
        parts, wtype = [], None
        for name, rows in (("attn_qkv", cfg.qkv_dim), ("attn_gate", cfg.inner), ("ssm_beta", cfg.num_v_heads),
                           ("ssm_alpha", cfg.num_v_heads)):
            t, b = self.raw(p + name + ".weight")
            if t.dims != (cfg.hidden, rows):
                raise ValueError(f"{t.name}: dims {t.dims}, expected ({cfg.hidden}, {rows})")
            if wtype is None:
                wtype = t.ggml_type
            elif t.ggml_type != wtype:
                raise ValueError(f"{t.name}: type {t.ggml_type} differs from the layer's {wtype}")
            parts.append(np.asarray(b))
        if wtype not in (GGML_Q8_0, GGML_Q4_K):
            raise ValueError(f"layer {layer}: projection type {wtype} (supported: Q8_0, Q4_K)")
        to, out_b = self.raw(p + "ssm_out.weight")
        if to.dims != (cfg.inner, cfg.hidden) or to.ggml_type != wtype:
            raise ValueError(f"{to.name}: dims {to.dims} type {to.ggml_type}")
        row_bytes = cfg.hidden // _BLOCK[wtype][1] * _BLOCK[wtype][0]
        in_proj = np.concatenate(parts).reshape(cfg.in_proj_rows, row_bytes)

        def f32(name, n):
            t, b = self.raw(p + name)
            if t.ggml_type != GGML_F32 or int(np.prod(t.dims)) != n:
                raise ValueError(f"{t.name}: expected {n} fp32 values, got type {t.ggml_type} dims {t.dims}")
            return np.frombuffer(bytes(b), dtype=np.float32).copy()

        conv = f32("ssm_conv1d.weight", cfg.qkv_dim * CONV_WIDTH).reshape(cfg.qkv_dim, CONV_WIDTH)
        return cfg, LayerTensors(cfg, wtype, in_proj, np.asarray(out_b).reshape(cfg.hidden, -1), conv,
                                 f32("ssm_a", cfg.num_v_heads), f32("ssm_dt.bias", cfg.num_v_heads),
                                 f32("ssm_norm.weight", cfg.head_dim))


def _w_string(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _w_value(v) -> bytes:
    if isinstance(v, bool):
        return struct.pack("<I?", BOOL, v)
    if isinstance(v, int):
        return struct.pack("<II", U32, v) if 0 <= v < 2 ** 32 else struct.pack("<Iq", I64, v)
    if isinstance(v, float):
        return struct.pack("<If", F32, v)
    if isinstance(v, str):
        return struct.pack("<I", STRING) + _w_string(v)
    raise TypeError(f"cannot write a {type(v).__name__} value")


def write_gguf(path, kv: dict, tensors: list[tuple[str, int, tuple[int, ...], np.ndarray]]) -> None:
    """GGUF v3: kv (int -> U32, float -> F32, str, bool), tensors (name, GGML
    type, GGUF dims, raw bytes), data aligned to 32 bytes."""
    head = MAGIC + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, v in kv.items():
        head += _w_string(k) + _w_value(v)
    off, infos, blobs = 0, b"", []
    for name, gtype, dims, data in tensors:
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        t = TensorInfo(name, gtype, tuple(dims), off)
        if t.nbytes != data.size:
            raise ValueError(f"{name}: {data.size} bytes, dims {dims} type {gtype} need {t.nbytes}")
        infos += _w_string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", gtype, off)
        blobs.append((off, data))
        off = (off + data.size + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    header = head + infos
    start = (len(header) + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    with open(path, "wb") as f:
        f.write(header + b"\0" * (start - len(header)))
        for o, data in blobs:
            f.seek(start + o)
            f.write(data.tobytes())
        f.truncate(start + off)


def layer_tensor_list(layer: int, t: LayerTensors) -> list[tuple[str, int, tuple[int, ...], np.ndarray]]:
    """The nine GGUF tensors of a DeltaNet layer from LayerTensors (the reference's names and dims)."""
    c = t.cfg
    p = f"blk.{layer}."
    row_bytes = t.in_proj.shape[1]
    spans = (("attn_qkv", 0, c.qkv_dim), ("attn_gate", c.qkv_dim, c.inner),
             ("ssm_beta", c.qkv_dim + c.inner, c.num_v_heads),
             ("ssm_alpha", c.qkv_dim + c.inner + c.num_v_heads, c.num_v_heads))
    out = [(p + n + ".weight", t.weight_type, (c.hidden, rows), t.in_proj[r0:r0 + rows].reshape(-1))
           for n, r0, rows in spans]
    assert row_bytes * c.in_proj_rows == t.in_proj.size
    out.append((p + "ssm_out.weight", t.weight_type, (c.inner, c.hidden), t.out_proj.reshape(-1)))
    out.append((p + "ssm_a", GGML_F32, (c.num_v_heads,), t.ssm_a.astype(np.float32)))
    out.append((p + "ssm_dt.bias", GGML_F32, (c.num_v_heads,), t.dt_bias.astype(np.float32)))
    out.append((p + "ssm_norm.weight", GGML_F32, (c.head_dim,), t.head_norm.astype(np.float32)))
    out.append((p + "ssm_conv1d.weight", GGML_F32, (CONV_WIDTH, c.qkv_dim),
                t.conv1d_w.astype(np.float32).reshape(-1)))
    return out


def model_kv(cfg: GDNConfig, n_layers: int, arch: str = "qwen35moe") -> dict:
    """The metadata keys the reference parser reads for a DeltaNet stack."""
    return {"general.architecture": arch, f"{arch}.block_count": n_layers, f"{arch}.embedding_length": cfg.hidden,
            f"{arch}.ssm.inner_size": cfg.inner, f"{arch}.ssm.group_count": cfg.num_k_heads,
            f"{arch}.ssm.state_size": cfg.head_dim, f"{arch}.ssm.conv_kernel": CONV_WIDTH}
