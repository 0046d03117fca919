"""Seeded synthetic GGUF tensors and inputs for the benchmark configurations.

No model file is available, so every weight is drawn from a fixed seed with
numpy's PCG64, one seed per tensor (plus 16 x layer index for stacks):
  x = 0, in_proj qkvz = 1, in_proj ba = 2, out_proj = 3, conv1d = 4, A_log = 5,
  head norm = 6, state = 7 (+ sequence index).
Distributions (the benchmark configs' own, with the unspecified ones fixed here):
  Q8_0 blocks: qs ~ U{-127..127}, d = fp16(|N(0,1)| * 0.02)
  Q4_K blocks: d, dmin = fp16(|N(0,1)| * 0.02), 12 scale bytes ~ U{0..255},
               nibbles ~ U{0..15}
  Q5_K blocks: d, dmin = fp16(|N(0,1)| * 0.01), the other 172 bytes ~ U{0..255}
  A_log ~ U(0, 2.7) -> ssm_a = -exp(A_log); dt_bias = 0
  conv1d weight ~ N(0, 0.5^2); head-norm weight = 1 + 0.1 N(0,1)
  hidden states ~ N(0,1); pre-filled states ~ N(0, 0.05^2)
Block layouts are GGUF's: Q8_0 {fp16 d; int8 qs[32]} = 34 bytes
(engine/runtime/q8_dequant.h:15-18); Q4_K {fp16 d; fp16 dmin; u8 scales[12];
u8 qs[128]} = 144 bytes (engine/runtime/q4k_dequant.h:28-33).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .config import CONV_WIDTH, GDNConfig

SEED_X, SEED_QKVZ, SEED_BA, SEED_OUT, SEED_CONV, SEED_ALOG, SEED_NORM, SEED_STATE = range(8)
LAYER_SEED_STRIDE = 16


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def q8_0_blocks(rows: int, cols: int, seed: int) -> np.ndarray:
    """Random Q8_0 tensor as GGUF bytes, shape [rows, cols/32*34] uint8."""
    assert cols % 32 == 0
    g = rng(seed)
    nb = cols // 32
    d = (np.abs(g.standard_normal((rows, nb))) * 0.02).astype(np.float16)
    qs = g.integers(-127, 128, size=(rows, nb, 32), dtype=np.int8)
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = qs.view(np.uint8)
    return out.reshape(rows, nb * 34)


def q4_k_blocks(rows: int, cols: int, seed: int) -> np.ndarray:
    """Random Q4_K tensor as GGUF bytes, shape [rows, cols/256*144] uint8."""
    assert cols % 256 == 0
    g = rng(seed)
    nb = cols // 256
    d = (np.abs(g.standard_normal((rows, nb))) * 0.02).astype(np.float16)
    dmin = (np.abs(g.standard_normal((rows, nb))) * 0.02).astype(np.float16)
    scales = g.integers(0, 256, size=(rows, nb, 12), dtype=np.uint8)
    lo = g.integers(0, 16, size=(rows, nb, 128), dtype=np.uint8)
    hi = g.integers(0, 16, size=(rows, nb, 128), dtype=np.uint8)
    out = np.empty((rows, nb, 144), dtype=np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:4] = dmin.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 4:16] = scales
    out[:, :, 16:] = lo | (hi << 4)
    return out.reshape(rows, nb * 144)


def q5_k_blocks(rows: int, cols: int, seed: int) -> np.ndarray:
    """Random Q5_K tensor as GGUF bytes (d, dmin, 12 scale bytes, qh[32], qs[128]),
    shape [rows, cols/256*176] uint8."""
    assert cols % 256 == 0
    g = rng(seed)
    nb = cols // 256
    d = (np.abs(g.standard_normal((rows, nb))) * 0.01).astype(np.float16)
    dmin = (np.abs(g.standard_normal((rows, nb))) * 0.01).astype(np.float16)
    out = np.empty((rows, nb, 176), dtype=np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:4] = dmin.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 4:] = g.integers(0, 256, size=(rows, nb, 172), dtype=np.uint8)
    return out.reshape(rows, nb * 176)


def q8_0_split(blocks: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """GGUF Q8_0 bytes -> (qs int8 [rows, cols], d uint16 [rows, cols/32]) planes."""
    b = blocks.reshape(rows, cols // 32, 34)
    d = np.ascontiguousarray(b[:, :, 0:2]).view(np.uint16).reshape(rows, cols // 32)
    qs = np.ascontiguousarray(b[:, :, 2:]).view(np.int8).reshape(rows, cols)
    return qs, d


def q8_0_dequant_np(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """numpy float32 d*q (one rounding, as q8_dequant_row does)."""
    qs, d = q8_0_split(blocks, rows, cols)
    return (d.view(np.float16).astype(np.float32).repeat(32, axis=1) * qs.astype(np.float32)).astype(np.float32)


@dataclass
class LayerTensors:
    """One layer's synthetic tensors in GGUF form (host numpy)."""
    cfg: GDNConfig
    weight_type: int          # 8 = Q8_0, 12 = Q4_K
    in_proj: np.ndarray       # rows: qkv | z | beta | alpha, GGUF bytes
    out_proj: np.ndarray      # rows: hidden, cols: inner, GGUF bytes
    conv1d_w: np.ndarray      # [QKV, 4] fp32
    ssm_a: np.ndarray         # [Hv] fp32 (= -exp(A_log))
    dt_bias: np.ndarray       # [Hv] fp32
    head_norm: np.ndarray     # [d] fp32

    def row_bytes(self, cols: int) -> int:
        return cols // 32 * 34 if self.weight_type == 8 else cols // 256 * 144

    def split_in_proj(self) -> dict[str, np.ndarray]:
        """The reference's four tensors: attn_qkv, attn_gate, ssm_beta, ssm_alpha."""
        c = self.cfg
        a, b = c.qkv_dim, c.qkv_dim + c.inner
        return {
            "w_qkv": np.ascontiguousarray(self.in_proj[:a]),
            "w_gate": np.ascontiguousarray(self.in_proj[a:b]),
            "w_beta": np.ascontiguousarray(self.in_proj[b:b + c.num_v_heads]),
            "w_alpha": np.ascontiguousarray(self.in_proj[b + c.num_v_heads:]),
        }


def layer_tensors(cfg: GDNConfig, layer: int = 0, weight_type: int = 8) -> LayerTensors:
    """The seeded tensors of one DeltaNet layer (seeds + 16*layer)."""
    off = LAYER_SEED_STRIDE * layer
    gen = q8_0_blocks if weight_type == 8 else q4_k_blocks
    # in_proj = [qkvz (QKV + inner rows), seed 1 ; ba (2*Hv rows: beta then alpha), seed 2]
    qkvz = gen(cfg.qkv_dim + cfg.inner, cfg.hidden, SEED_QKVZ + off)
    ba = gen(2 * cfg.num_v_heads, cfg.hidden, SEED_BA + off)
    out = gen(cfg.hidden, cfg.inner, SEED_OUT + off)
    conv = (rng(SEED_CONV + off).standard_normal((cfg.qkv_dim, CONV_WIDTH)) * 0.5).astype(np.float32)
    a_log = rng(SEED_ALOG + off).uniform(0.0, 2.7, size=cfg.num_v_heads)
    ssm_a = (-np.exp(a_log)).astype(np.float32)
    dt_bias = np.zeros(cfg.num_v_heads, dtype=np.float32)
    norm = (1.0 + 0.1 * rng(SEED_NORM + off).standard_normal(cfg.head_dim)).astype(np.float32)
    return LayerTensors(cfg, weight_type, np.concatenate([qkvz, ba], axis=0), out, conv, ssm_a, dt_bias, norm)


def layer_tensors_device(cfg: GDNConfig, layer: int, device) -> LayerTensors:
    """Q8_0 layer tensors drawn on the device with torch's generator (same
    distributions and per-layer seeds as layer_tensors, not the same values):
    for stacks of many layers, where numpy generation would dominate the run.
    in_proj / out_proj are device uint8 GGUF bytes; the small tensors come from
    layer_tensors' numpy draws."""
    import torch
    dev = torch.device(device)
    off = LAYER_SEED_STRIDE * layer

    def q8(rows, cols, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        nb = cols // 32
        d = (torch.randn((rows, nb), generator=g, device=dev).abs() * 0.02).to(torch.float16)
        qs = torch.randint(-127, 128, (rows, nb, 32), generator=g, device=dev, dtype=torch.int8)
        out = torch.empty((rows, nb, 34), dtype=torch.uint8, device=dev)
        out[:, :, 0:2] = d.view(torch.uint8).view(rows, nb, 2)
        out[:, :, 2:] = qs.view(torch.uint8)
        return out.view(rows, nb * 34)

    qkvz = q8(cfg.qkv_dim + cfg.inner, cfg.hidden, SEED_QKVZ + off)
    ba = q8(2 * cfg.num_v_heads, cfg.hidden, SEED_BA + off)
    out = q8(cfg.hidden, cfg.inner, SEED_OUT + off)
    conv = (rng(SEED_CONV + off).standard_normal((cfg.qkv_dim, CONV_WIDTH)) * 0.5).astype(np.float32)
    a_log = rng(SEED_ALOG + off).uniform(0.0, 2.7, size=cfg.num_v_heads)
    norm = (1.0 + 0.1 * rng(SEED_NORM + off).standard_normal(cfg.head_dim)).astype(np.float32)
    return LayerTensors(cfg, 8, torch.cat([qkvz, ba]), out, conv, (-np.exp(a_log)).astype(np.float32),
                        np.zeros(cfg.num_v_heads, dtype=np.float32), norm)


def hidden_states(n_tokens: int, hidden: int, seed: int = SEED_X) -> np.ndarray:
    """x ~ N(0,1), fp32 [n_tokens, hidden]."""
    return rng(seed).standard_normal((n_tokens, hidden)).astype(np.float32)


def prefilled_state(cfg: GDNConfig, seq: int, std: float = 0.05) -> np.ndarray:
    """S of sequence `seq` ~ N(0, std^2), fp32 [Hv, d, d] (seed 7 + seq)."""
    return (rng(SEED_STATE + seq).standard_normal((cfg.num_v_heads, cfg.head_dim, cfg.head_dim)) * std).astype(
        np.float32)
