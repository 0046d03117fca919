"""Host side of the B200 Gated DeltaNet layer.

Mirrors the reference's layer interface -- DeltaNetState / dn_state_init
(engine/runtime/deltanet_impl.h:48-74) and deltanet_forward (145-377) -- over
the C ABI of libwinmoe_gdn.so.  PyTorch provides device memory and streams;
all arithmetic runs in the library's CUDA kernels.

  DeltaNetWeights   one layer's weights on the device (Q8_0 planes or Q4_K blocks)
  DeltaNetState     S [B][Hv][d][d], conv window [B][4][QKV], conv_pos [B]
  decode_step       one token for B sequences (gdn_decode_step)
  prefill           T prompt tokens of one sequence, chunked (gdn_prefill)
  deltanet_forward  the reference's own signature, one token of one sequence
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import GDNError, check, lib
from .config import CONV_WIDTH, GDNConfig


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream: torch.cuda.Stream | None, device: torch.device) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def _as_device_u8(a, device) -> torch.Tensor:
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a).view(np.uint8).reshape(-1))
    return a.reshape(-1).view(torch.uint8).to(device).contiguous()


def _as_device_f32(a, device) -> torch.Tensor | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return a.to(device=device, dtype=torch.float32).contiguous()


def q8_0_planes(blocks, rows: int, cols: int, device, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    """GGUF Q8_0 bytes (host or device) -> device planes (qs int8 [rows, cols], d fp16 bits [rows, cols/32])."""
    device = torch.device(device)
    raw = _as_device_u8(blocks, device)
    if raw.numel() != rows * cols // 32 * 34:
        raise GDNError(-2, f"Q8_0 tensor has {raw.numel()} bytes, expected {rows * cols // 32 * 34}")
    qs = torch.empty((rows, cols), dtype=torch.int8, device=device)
    d = torch.empty((rows, cols // 32), dtype=torch.int16, device=device)
    check(lib().gdn_q8_0_repack(raw.data_ptr(), qs.data_ptr(), d.data_ptr(), rows, cols, _stream(stream, device)))
    return qs, d


@dataclass
class DeltaNetWeights:
    """One DeltaNet layer on the device (the DeltaNet fields of LayerWeights,
    engine/runtime/transformer.h:63-78), with the four input projections
    stacked as qkv | z | beta | alpha rows."""

    cfg: GDNConfig
    weight_type: int
    in_qs: torch.Tensor | None
    in_d: torch.Tensor | None
    out_qs: torch.Tensor | None
    out_d: torch.Tensor | None
    in_blocks: torch.Tensor | None
    out_blocks: torch.Tensor | None
    conv1d_w: torch.Tensor | None
    ssm_a: torch.Tensor | None
    dt_bias: torch.Tensor | None
    head_norm: torch.Tensor | None
    head_map: int = _lib.HEAD_MAP_GROUPED
    _struct: _lib.gdn_layer | None = field(default=None, repr=False)

    @classmethod
    def upload(cls, cfg: GDNConfig, in_proj, out_proj, conv1d_w, ssm_a, dt_bias, head_norm,
               weight_type: int = _lib.GGML_Q8_0, head_map: int = _lib.HEAD_MAP_GROUPED,
               device="cuda") -> "DeltaNetWeights":
        """in_proj / out_proj are GGUF bytes (numpy or torch, host or device)."""
        cfg.validate()
        device = torch.device(device)
        if weight_type == _lib.GGML_Q8_0:
            in_qs, in_d = q8_0_planes(in_proj, cfg.in_proj_rows, cfg.hidden, device)
            out_qs, out_d = q8_0_planes(out_proj, cfg.hidden, cfg.inner, device)
            in_b = out_b = None
        elif weight_type == _lib.GGML_Q4_K:
            in_qs = in_d = out_qs = out_d = None
            in_b = _as_device_u8(in_proj, device)
            out_b = _as_device_u8(out_proj, device)
            if in_b.numel() != cfg.in_proj_rows * cfg.hidden // 256 * 144:
                raise GDNError(-2, "Q4_K in_proj has the wrong size")
            if out_b.numel() != cfg.hidden * cfg.inner // 256 * 144:
                raise GDNError(-2, "Q4_K out_proj has the wrong size")
        else:
            raise GDNError(-3, f"weight type {weight_type} is not supported (8 = Q8_0, 12 = Q4_K)")
        conv = _as_device_f32(conv1d_w, device)
        if conv is not None and conv.numel() != cfg.qkv_dim * CONV_WIDTH:
            raise GDNError(-2, "conv1d_w must hold QKV x 4 floats")
        return cls(cfg, weight_type, in_qs, in_d, out_qs, out_d, in_b, out_b, conv,
                   _as_device_f32(ssm_a, device), _as_device_f32(dt_bias, device),
                   _as_device_f32(head_norm, device), head_map)

    @classmethod
    def from_reference_tensors(cls, cfg: GDNConfig, w_qkv, w_gate, w_alpha, w_beta, w_out, weight_type,
                               conv1d_w, ssm_a, dt_bias, head_norm, **kw) -> "DeltaNetWeights":
        """The reference's separate GGUF tensors (blk.N.attn_qkv, attn_gate,
        ssm_alpha, ssm_beta, ssm_out; winmoe_inference.c:318-392)."""
        parts = [np.asarray(w).view(np.uint8).reshape(-1) for w in (w_qkv, w_gate, w_beta, w_alpha)]
        return cls.upload(cfg, np.concatenate(parts), w_out, conv1d_w, ssm_a, dt_bias, head_norm,
                          weight_type=weight_type, **kw)

    @classmethod
    def from_gguf(cls, gguf, layer: int, head_map: int = _lib.HEAD_MAP_GROUPED, device="cuda") -> "DeltaNetWeights":
        """DeltaNet layer `layer` of a GGUF model file (a path or winmoe_b200.gguf.GGUFFile),
        by the reference's tensor names (winmoe_inference.c:311-392)."""
        from .gguf import GGUFFile
        g = gguf if isinstance(gguf, GGUFFile) else GGUFFile(gguf)
        cfg, t = g.deltanet_layer(layer)
        return cls.upload(cfg, t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm,
                          weight_type=t.weight_type, head_map=head_map, device=device)

    @property
    def device(self) -> torch.device:
        t = self.in_qs if self.in_qs is not None else self.in_blocks
        return t.device

    def struct(self) -> _lib.gdn_layer:
        if self._struct is None:
            c = self.cfg
            self._struct = _lib.gdn_layer(
                _lib.gdn_dims(c.hidden, c.num_k_heads, c.num_v_heads, c.head_dim), self.weight_type, self.head_map,
                _ptr(self.in_qs), _ptr(self.in_d), _ptr(self.out_qs), _ptr(self.out_d),
                _ptr(self.in_blocks), _ptr(self.out_blocks), _ptr(self.conv1d_w), _ptr(self.ssm_a),
                _ptr(self.dt_bias), _ptr(self.head_norm))
        return self._struct


@dataclass
class DeltaNetState:
    """Recurrent state of B sequences (DeltaNetState, deltanet_impl.h:48-60):
    S [B][Hv][d][d] fp32 (row = key index, col = value index), the conv1d
    window [B][4][QKV] fp32 (circular) and conv_pos [B] int32."""

    S: torch.Tensor
    conv_buf: torch.Tensor
    conv_pos: torch.Tensor

    @classmethod
    def zeros(cls, cfg: GDNConfig, batch: int, device="cuda") -> "DeltaNetState":
        """dn_state_init: calloc'ed S and window, conv_pos = 0 (deltanet_impl.h:62-74)."""
        device = torch.device(device)
        return cls(torch.zeros((batch, cfg.num_v_heads, cfg.head_dim, cfg.head_dim), dtype=torch.float32, device=device),
                   torch.zeros((batch, CONV_WIDTH, cfg.qkv_dim), dtype=torch.float32, device=device),
                   torch.zeros(batch, dtype=torch.int32, device=device))

    @property
    def batch(self) -> int:
        return self.S.shape[0]

    def clone(self) -> "DeltaNetState":
        return DeltaNetState(self.S.clone(), self.conv_buf.clone(), self.conv_pos.clone())


_ws_cache: dict[tuple, torch.Tensor] = {}


def workspace(cfg: GDNConfig, batch: int, device) -> torch.Tensor:
    """Cached scratch for gdn_decode_step (allocated by torch, outside the C ABI),
    looked up by (dims, batch, device) so that a decode loop pays one dict hit."""
    key = (cfg, batch, device)
    ws = _ws_cache.get(key)
    if ws is None:
        dims = _lib.gdn_dims(cfg.hidden, cfg.num_k_heads, cfg.num_v_heads, cfg.head_dim)
        need = lib().gdn_decode_workspace_size(C.byref(dims), batch)
        ws = torch.empty(need + 256, dtype=torch.uint8, device=torch.device(device))
        _ws_cache[key] = ws
    return ws


def _act_dtype(x: torch.Tensor) -> int:
    if x.dtype == torch.float32:
        return _lib.DTYPE_F32
    if x.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if x.dtype == torch.float16:
        return _lib.DTYPE_F16
    raise GDNError(-3, f"activation dtype {x.dtype} is not supported")


def decode_step(w: DeltaNetWeights, state: DeltaNetState, x: torch.Tensor, out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None, ref_projections: bool = False) -> torch.Tensor:
    """One decode token for every sequence of `state`: x [B][hidden] -> out [B][hidden] fp32.
    ref_projections=True (fp32 x, Q8_0): the projections as the reference's CPU
    computes them (Q8_K activations, gdn_decode_step_ex)."""
    B = state.batch
    cfg = w.cfg
    if x.shape != (B, cfg.hidden) or not x.is_cuda or not x.is_contiguous():
        raise GDNError(-2, f"x must be a contiguous CUDA tensor of shape ({B}, {cfg.hidden})")
    if out is None:
        out = torch.empty((B, cfg.hidden), dtype=torch.float32, device=x.device)
    ws = workspace(cfg, B, x.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    nbytes = ws.numel() - (base - ws.data_ptr())
    check(lib().gdn_decode_step_ex(C.byref(w.struct()), B, x.data_ptr(), _act_dtype(x), out.data_ptr(),
                                   state.S.data_ptr(), state.conv_buf.data_ptr(), state.conv_pos.data_ptr(),
                                   base, nbytes, 1 if ref_projections else 0, _stream(stream, x.device)))
    return out


class DecodeGraph:
    """A decode step captured once as a CUDA graph on fixed buffers: write the
    next token's activations into `x`, call replay(), read `out`.  Each replay
    advances `state` exactly as decode_step does (same kernels, same order); one
    graph launch replaces the step's six kernel launches."""

    def __init__(self, w: DeltaNetWeights, state: DeltaNetState, x_dtype=torch.float32):
        dev = state.S.device
        B, H = state.batch, w.cfg.hidden
        self.x = torch.zeros((B, H), dtype=x_dtype, device=dev)
        self.out = torch.empty((B, H), dtype=torch.float32, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        # one eager step on a scratch state first: workspace, kernel attributes and the
        # library's per-device lookups are set up outside the capture
        scratch = DeltaNetState.zeros(w.cfg, B, dev)
        decode_step(w, scratch, self.x, self.out, stream=s)
        s.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):  # captured, not run: `state` is untouched
            decode_step(w, state, self.x, self.out, stream=s)
        torch.cuda.current_stream(dev).wait_stream(s)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out


def prefill_workspace(cfg: GDNConfig, T: int, device) -> torch.Tensor:
    """Cached scratch for gdn_prefill (allocated by torch, outside the C ABI)."""
    device = torch.device(device)
    dims = _lib.gdn_dims(cfg.hidden, cfg.num_k_heads, cfg.num_v_heads, cfg.head_dim)
    need = lib().gdn_prefill_workspace_size(C.byref(dims), T)
    key = (device, "prefill", need)
    ws = _ws_cache.get(key)
    if ws is None:
        ws = torch.empty(need + 256, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def prefill(w: DeltaNetWeights, state: DeltaNetState, x: torch.Tensor, seq: int = 0,
            out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """T prompt tokens of sequence `seq` of `state` (chunked WY form): x [T][hidden]
    -> out [T][hidden] fp32; the sequence's S, conv window and conv_pos end up
    as after T deltanet_forward calls, ready for decode_step."""
    cfg = w.cfg
    if x.dim() != 2 or x.shape[1] != cfg.hidden or not x.is_cuda or not x.is_contiguous():
        raise GDNError(-2, f"x must be a contiguous CUDA tensor of shape (T, {cfg.hidden})")
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=x.device)
    ws = prefill_workspace(cfg, T, x.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    nbytes = ws.numel() - (base - ws.data_ptr())
    check(lib().gdn_prefill(C.byref(w.struct()), T, x.data_ptr(), _act_dtype(x), out.data_ptr(),
                            state.S[seq].data_ptr(), state.conv_buf[seq].data_ptr(), state.conv_pos[seq:].data_ptr(),
                            base, nbytes, _stream(stream, x.device)))
    return out


def gemm_q8_0(qs: torch.Tensor, d: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None,
              fast: bool = False, stream=None, ref_exact: bool = False) -> torch.Tensor:
    """y[m][n] = x[m] . W[n] for Q8_0 planes (quant_matvec type 8, batched).
    fast=False keeps fp32-GEMV accuracy; fast=True lets m >= 64 fp16/bf16
    batches use one tensor-core weight operand (weights rounded once);
    ref_exact=True (fp32 x) reproduces the reference CPU's quant_matvec bit for
    bit (Q8_K activations for n >= 128 and k % 256 == 0)."""
    n, k = qs.shape
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    flags = _lib.GEMM_REF_EXACT if ref_exact else _lib.GEMM_FAST if fast else _lib.GEMM_EXACT
    check(lib().gdn_q8_0_gemm(qs.data_ptr(), d.data_ptr(), n, k, x.data_ptr(), _act_dtype(x), m, out.data_ptr(),
                              flags, _stream(stream, x.device)))
    return out


def quantize_q8_K(x: torch.Tensor, stream=None) -> torch.Tensor:
    """quantize_row_q8_K: fp32 x (numel % 256 == 0) -> GGUF block_q8_K bytes (292 per 256 values)."""
    n = x.numel()
    out = torch.empty(n // 256 * 292, dtype=torch.uint8, device=x.device)
    check(lib().gdn_quantize_q8_K(x.data_ptr(), out.data_ptr(), n, _stream(stream, x.device)))
    return out


def gemm_q4_k(blocks: torch.Tensor, n: int, k: int, x: torch.Tensor, out: torch.Tensor | None = None,
              stream=None) -> torch.Tensor:
    """y[m][n] = x[m] . W[n] for GGUF Q4_K blocks (quant_matvec type 12, batched)."""
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    check(lib().gdn_q4_k_gemm(blocks.data_ptr(), n, k, x.data_ptr(), _act_dtype(x), m, out.data_ptr(),
                              _stream(stream, x.device)))
    return out


def dequant_q8_0(qs: torch.Tensor, d: torch.Tensor, stream=None) -> torch.Tensor:
    rows, cols = qs.shape
    out = torch.empty((rows, cols), dtype=torch.float32, device=qs.device)
    check(lib().gdn_q8_0_dequant(qs.data_ptr(), d.data_ptr(), out.data_ptr(), rows, cols, _stream(stream, qs.device)))
    return out


def dequant_q4_k(blocks: torch.Tensor, rows: int, cols: int, stream=None) -> torch.Tensor:
    out = torch.empty((rows, cols), dtype=torch.float32, device=blocks.device)
    check(lib().gdn_q4_k_dequant(blocks.data_ptr(), out.data_ptr(), rows, cols, _stream(stream, blocks.device)))
    return out


def dequant_q5_k(blocks: torch.Tensor, rows: int, cols: int, stream=None) -> torch.Tensor:
    out = torch.empty((rows, cols), dtype=torch.float32, device=blocks.device)
    check(lib().gdn_q5_k_dequant(blocks.data_ptr(), out.data_ptr(), rows, cols, _stream(stream, blocks.device)))
    return out


def gemm_q5_k(blocks: torch.Tensor, n: int, k: int, x: torch.Tensor, out: torch.Tensor | None = None,
              stream=None) -> torch.Tensor:
    """y[m][n] = x[m] . W[n] for GGUF Q5_K blocks (quant_matvec type 13, fp32 activations)."""
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    check(lib().gdn_q5_k_gemm(blocks.data_ptr(), n, k, x.data_ptr(), _act_dtype(x), m, out.data_ptr(),
                              _stream(stream, x.device)))
    return out


def expert_ffn(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, gate_type: int, down_type: int,
               hidden: int, inter: int, x: torch.Tensor, out: torch.Tensor | None = None, weight: float = 1.0,
               accumulate: bool = False, workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """One MoE expert's FFN for the m rows of x (gpu_expert_ffn_fused): down(SwiGLU(gate x, up x));
    accumulate=True adds weight * y into `out` (the batched expert path)."""
    m = x.shape[0]
    if out is None:
        out = torch.zeros((m, hidden), dtype=torch.float32, device=x.device)
    need = lib().gdn_expert_ffn_workspace_size(m, hidden, inter)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    check(lib().gdn_expert_ffn(w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), gate_type, down_type, hidden,
                               inter, x.data_ptr(), _act_dtype(x), m, out.data_ptr(), float(weight), int(accumulate),
                               workspace.data_ptr(), workspace.numel(), _stream(stream, x.device)))
    return out


MAX_EXPERTS_PER_CALL = 8


def experts_ffn(w_gate: list, w_up: list, w_down: list, gate_type: int, down_type: int, hidden: int, inter: int,
                x: torch.Tensor, weights=None, out: torch.Tensor | None = None, accumulate: bool = False,
                workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """The batched expert block of m tokens (gpu_expert_batch_start / _add / _finish):
    out (+)= sum_e weights[e] * down_e(SwiGLU(gate_e x, up_e x)), summed in expert
    order up to rounding, in two launches for up to MAX_EXPERTS_PER_CALL experts."""
    ne = len(w_gate)
    if not (len(w_up) == len(w_down) == ne):
        raise GDNError(-1, "w_gate, w_up and w_down must list the same experts")
    m = x.shape[0]
    if out is None:
        out = torch.zeros((m, hidden), dtype=torch.float32, device=x.device)
    need = lib().gdn_experts_ffn_workspace_size(ne, m, hidden, inter)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    ptrs = lambda ts: (C.c_void_p * max(ne, 1))(*[t.data_ptr() for t in ts])
    wts = None if weights is None else (C.c_float * max(ne, 1))(*[float(w) for w in weights])
    check(lib().gdn_experts_ffn(ne, ptrs(w_gate), ptrs(w_up), ptrs(w_down), gate_type, down_type, hidden, inter,
                                x.data_ptr(), _act_dtype(x), m, wts, out.data_ptr(), int(accumulate),
                                workspace.data_ptr(), workspace.numel(), _stream(stream, x.device)))
    return out


# ------------------------------------------------------------------ drop-in mirror

_weight_cache: dict[tuple, DeltaNetWeights] = {}


def deltanet_forward(output, x, state: DeltaNetState, w_qkv, w_qkv_type, w_gate, w_gate_type, w_alpha,
                     w_alpha_type, w_beta, w_beta_type, w_out, w_out_type, conv1d_w, a_log, dt_bias, head_norm,
                     hidden_dim, cfg: GDNConfig | None = None):
    """deltanet_forward (engine/runtime/deltanet_impl.h:145-162) with the same
    arguments: one token of one sequence, `output` [hidden] written in place,
    `state` (a DeltaNetState of batch 1) updated in place.

    Weights are GGUF bytes on the host, as the engine passes them; they are
    uploaded on first use and cached by buffer identity.  `a_log` is the GGUF
    ssm_a tensor (= -exp(A_log)), as in the reference.  All five projections
    must share one type (8 = Q8_0 or 12 = Q4_K).  Unlike the reference (which
    has no return code), bad shapes or types raise GDNError.
    """
    types = {w_qkv_type, w_gate_type, w_out_type} | ({w_alpha_type} if w_alpha is not None else set()) | (
        {w_beta_type} if w_beta is not None else set())
    if len(types) != 1:
        raise GDNError(-3, f"mixed projection types {sorted(types)} are not supported")
    if w_alpha is None or w_beta is None:
        raise GDNError(-6, "w_alpha and w_beta are required")
    wt = types.pop()
    if cfg is None:
        cfg = GDNConfig(hidden=hidden_dim, num_k_heads=16, num_v_heads=32, head_dim=128)
    device = state.S.device
    key = (id(w_qkv), id(w_gate), id(w_alpha), id(w_beta), id(w_out), id(conv1d_w), wt, cfg, device)
    w = _weight_cache.get(key)
    if w is None:
        w = DeltaNetWeights.from_reference_tensors(cfg, w_qkv, w_gate, w_alpha, w_beta, w_out, wt, conv1d_w, a_log,
                                                   dt_bias, head_norm, device=device)
        _weight_cache[key] = w
    xt = torch.as_tensor(np.asarray(x, dtype=np.float32)).reshape(1, hidden_dim).to(device)
    y = decode_step(w, state, xt)
    res = y.reshape(-1).cpu().numpy()
    if output is not None:
        np.copyto(np.asarray(output).reshape(-1), res)
    return res
