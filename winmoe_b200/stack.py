"""A stack of DeltaNet layers over one long prompt, value heads sharded over GPUs.

The reference runs its layers one after the other on one device
(engine/runtime/winmoe_inference.c:1155-1162, 1648-1653): per layer
    normed = rmsnorm(hidden, attn_norm)          (attention.h:29-44)
    o      = deltanet_forward(normed)            (deltanet_impl.h:145-377)
    hidden = residual + o.
Here a whole prompt of T tokens goes through each layer at once (chunked
prefill), and with G ranks in a process group every rank owns Hv / G value
heads with their key groups:

  1. rank r slices the layer to heads [r Hv/G, (r+1) Hv/G) (`slice_layer`):
     q/k rows of its key groups, v/z/beta/alpha rows and conv channels of its
     heads -- a smaller layer of the same form, whose rows compute exactly as
     in the whole layer;
  2. `gdn_prefill_gated` runs the chunked prefill up to the output gate;
  3. an NCCL all-gather stacks the G head blocks [G][T][inner / G];
  4. each rank runs out_proj for its T / G tokens over the gathered blocks
     (`gdn_out_proj_gathered`, the single-GPU k order, so bit-identical);
  5. an all-gather of those [T / G][hidden] rows gives every rank the layer
     output, and the next layer's `gdn_add_rmsnorm` adds it to the residual.

With a `PeerStack` (CUDA IPC buffers on every rank) the collectives move into
the kernels instead: the residual stays sharded by tokens, the RMSNorm stores
each rank's rows into every rank's copy of the layer input, and the prefill's
last kernel stores each token slice's head columns into the out_proj operand
of the rank that owns the slice -- peer stores over NVLink, each byte
crossing once (`_prefill_stack_fused`).

With G = 1 the same code runs without collectives.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import GDNError, check, lib
from .config import CONV_WIDTH, GDNConfig
from .layer import DeltaNetState, DeltaNetWeights, _stream, prefill_workspace, q8_0_planes
from .synth import LayerTensors


def head_range(cfg: GDNConfig, rank: int, world: int) -> tuple[int, int]:
    """Value heads [h0, h1) of `rank`; whole key groups per rank (grouped map)."""
    hv, hpg = cfg.num_v_heads, cfg.heads_per_group
    if hv % world or (hv // world) % hpg:
        raise GDNError(-2, f"{hv} value heads in groups of {hpg} do not split over {world} ranks")
    per = hv // world
    return rank * per, (rank + 1) * per


def slice_layer(cfg: GDNConfig, t: LayerTensors, h0: int, h1: int) -> tuple[GDNConfig, LayerTensors]:
    """The layer restricted to value heads [h0, h1) (grouped head map), GGUF bytes.

    in_proj rows (qkv | z | beta | alpha): q and k rows of key groups
    [h0/hpg, h1/hpg), v and z rows of the heads, their beta and alpha rows.
    out_proj keeps the heads' 32-column blocks of every row (the layer's own
    out_proj is run on gathered heads instead, see module doc)."""
    d, hpg = cfg.head_dim, cfg.heads_per_group
    if h0 % hpg or h1 % hpg or not 0 <= h0 < h1 <= cfg.num_v_heads:
        raise GDNError(-2, f"heads [{h0}, {h1}) are not whole key groups of {hpg}")
    g0, g1 = h0 // hpg, h1 // hpg
    key, qkv, inner, hv = cfg.key_dim, cfg.qkv_dim, cfg.inner, cfg.num_v_heads
    rows = np.concatenate([np.arange(g0 * d, g1 * d), key + np.arange(g0 * d, g1 * d),
                           2 * key + np.arange(h0 * d, h1 * d), qkv + np.arange(h0 * d, h1 * d),
                           qkv + inner + np.arange(h0, h1), qkv + inner + hv + np.arange(h0, h1)])
    sub = GDNConfig(cfg.hidden, g1 - g0, h1 - h0, d)
    if isinstance(t.in_proj, torch.Tensor):  # device bytes: slice on the device
        in_proj = t.in_proj[torch.from_numpy(rows).to(t.in_proj.device)].contiguous()
    else:
        in_proj = np.ascontiguousarray(t.in_proj[rows])
    conv_rows = rows[rows < qkv]  # the qkv channels, in the same order
    conv = np.ascontiguousarray(t.conv1d_w.reshape(qkv, CONV_WIDTH)[conv_rows])
    if t.weight_type == 8:
        bpr = inner // 32  # Q8_0 blocks per out_proj row; head h owns blocks [h d/32, (h+1) d/32)
        ob = t.out_proj.reshape(cfg.hidden, bpr, 34)[:, h0 * d // 32:h1 * d // 32]
        out_proj = (ob.contiguous().reshape(cfg.hidden, -1) if isinstance(ob, torch.Tensor)
                    else np.ascontiguousarray(ob.reshape(cfg.hidden, -1)))
    else:
        raise GDNError(-3, "head sharding is implemented for Q8_0 layers")
    return sub, LayerTensors(sub, t.weight_type, in_proj, out_proj, conv, np.ascontiguousarray(t.ssm_a[h0:h1]),
                             np.ascontiguousarray(t.dt_bias[h0:h1]), t.head_norm)


@dataclass
class StackLayer:
    """One layer of the stack on this rank: its head slice and the full out_proj."""
    cfg: GDNConfig          # the whole layer
    heads: DeltaNetWeights  # this rank's slice (gdn_prefill_gated)
    out_qs: torch.Tensor    # full out_proj planes [hidden][inner] (gdn_out_proj_gathered)
    out_d: torch.Tensor
    h0: int
    h1: int

    @classmethod
    def upload(cls, cfg: GDNConfig, t: LayerTensors, rank: int = 0, world: int = 1, device="cuda") -> "StackLayer":
        h0, h1 = head_range(cfg, rank, world)
        sub, ts = slice_layer(cfg, t, h0, h1)
        w = DeltaNetWeights.upload(sub, ts.in_proj, ts.out_proj, ts.conv1d_w, ts.ssm_a, ts.dt_bias, ts.head_norm,
                                   device=device)
        out_qs, out_d = q8_0_planes(t.out_proj, cfg.hidden, cfg.inner, torch.device(device))
        return cls(cfg, w, out_qs, out_d, h0, h1)

    def state(self, device="cuda") -> DeltaNetState:
        """Zero state of this rank's heads (S [1][Hv/G][d][d], conv window of its channels)."""
        return DeltaNetState.zeros(self.heads.cfg, 1, device)


def prefill_gated(w: DeltaNetWeights, state: DeltaNetState, x: torch.Tensor, out: torch.Tensor | None = None,
                  stream=None) -> torch.Tensor:
    """gdn_prefill_gated: x [T][hidden] -> gated head outputs [T][Hv*d] fp16."""
    cfg = w.cfg
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, cfg.inner), dtype=torch.float16, device=x.device)
    ws = prefill_workspace(cfg, T, x.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    check(lib().gdn_prefill_gated(C.byref(w.struct()), T, x.data_ptr(), _lib_dtype(x), out.data_ptr(),
                                  state.S[0].data_ptr(), state.conv_buf[0].data_ptr(), state.conv_pos.data_ptr(),
                                  base, ws.numel() - (base - ws.data_ptr()), _stream(stream, x.device)))
    return out


def out_proj_gathered(out_qs: torch.Tensor, out_d: torch.Tensor, cfg: GDNConfig, gathered: torch.Tensor, t0: int,
                      t1: int, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """gdn_out_proj_gathered over gathered [G][T][inner/G] fp16 -> [t1-t0][hidden] fp32."""
    G, T = gathered.shape[0], gathered.shape[1]
    if out is None:
        out = torch.empty((t1 - t0, cfg.hidden), dtype=torch.float32, device=gathered.device)
    check(lib().gdn_out_proj_gathered(out_qs.data_ptr(), out_d.data_ptr(), cfg.hidden, cfg.inner,
                                      gathered.data_ptr(), G, T, t0, t1, out.data_ptr(),
                                      _stream(stream, gathered.device)))
    return out


def add_rmsnorm(x: torch.Tensor, add: torch.Tensor | None, w: torch.Tensor | None, y: torch.Tensor,
                stream=None) -> torch.Tensor:
    """gdn_add_rmsnorm: x += add (in place, if given); y = rmsnorm(x) * w."""
    T, H = x.shape
    check(lib().gdn_add_rmsnorm(x.data_ptr(), add.data_ptr() if add is not None else None,
                                w.data_ptr() if w is not None else None, y.data_ptr(), _lib_dtype(y), T, H,
                                _stream(stream, x.device)))
    return y


def out_proj_blocks(out_qs: torch.Tensor, out_d: torch.Tensor, cfg: GDNConfig, ptrs: list[int], T: int, t0: int,
                    t1: int, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """gdn_out_proj_blocks: block b of the heads at device pointer ptrs[b] ([T][inner/G] fp16,
    this GPU's or a peer's) -> out rows [t1-t0][hidden] fp32."""
    dev = out_qs.device
    if out is None:
        out = torch.empty((t1 - t0, cfg.hidden), dtype=torch.float32, device=dev)
    arr = (C.c_void_p * len(ptrs))(*ptrs)
    check(lib().gdn_out_proj_blocks(out_qs.data_ptr(), out_d.data_ptr(), cfg.hidden, cfg.inner, arr, len(ptrs), T,
                                    t0, t1, out.data_ptr(), _stream(stream, dev)))
    return out


class _DeviceArray:
    """A device pointer seen by torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": typestr,
                                         "strides": None, "version": 3}


class IpcBuffer:
    """`nbytes` of this GPU's memory shared over CUDA IPC with every rank of the
    group: ptrs[r] is rank r's buffer as mapped here (this rank's own at r =
    rank), opened for peer loads and stores over NVLink."""

    def __init__(self, nbytes: int, rank: int, world: int, group=None, device="cuda"):
        import torch.distributed as dist
        self.group, self.device = group, torch.device(device)
        ptr, handle = C.c_void_p(), (C.c_uint8 * 64)()
        check(lib().gdn_ipc_alloc(nbytes, C.byref(ptr), handle))
        self._own = ptr.value
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        every = torch.empty((world, 64), dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().numpy()
        self.ptrs, self._opened = [], []
        for r in range(world):
            if r == rank:
                self.ptrs.append(self._own)
                continue
            p = C.c_void_p()
            check(lib().gdn_ipc_open((C.c_uint8 * 64)(*every[r].tolist()), C.byref(p)))
            self.ptrs.append(p.value)
            self._opened.append(p.value)

    def view(self, shape: tuple, dtype: torch.dtype) -> torch.Tensor:
        """This rank's buffer as a tensor (no copy)."""
        typestr = {torch.float16: "<f2", torch.float32: "<f4", torch.int32: "<i4"}
        if dtype == torch.bfloat16:  # no bf16 in the array interface: alias the bits
            return torch.as_tensor(_DeviceArray(self._own, shape, "<i2"), device=self.device).view(torch.bfloat16)
        return torch.as_tensor(_DeviceArray(self._own, shape, typestr[dtype]), device=self.device)

    def close(self) -> None:
        """Every rank closes its peers' mappings, then frees its own buffer (a
        collective: every rank calls it)."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            check(lib().gdn_ipc_close(p))
        self._opened = []
        dist.barrier(group=self.group)
        if self._own:
            check(lib().gdn_ipc_free(self._own))
            self._own = 0


class PeerStack:
    """The buffers of a head-sharded stack whose collectives are fused into its
    kernels (`prefill_stack(..., peers=)`): on every rank a [T][hidden] copy of
    the layer input (each rank's RMSNorm stores its token slice into all of
    them) and a [T/G][inner] out_proj operand (each rank's prefill stores its
    head columns of that slice into it)."""

    def __init__(self, cfg: GDNConfig, T: int, rank: int, world: int, group=None, device="cuda",
                 norm_dtype=torch.bfloat16):
        import torch.distributed as dist
        if T % world or T // world < 64:
            raise GDNError(-2, f"T={T} over {world} ranks: the fused stack needs T/G >= 64 tokens per rank")
        self.cfg, self.T, self.rank, self.world, self.group = cfg, T, rank, world, group
        self.ts = T // world
        self.norm_dtype = norm_dtype
        esz = torch.empty((), dtype=norm_dtype).element_size()
        self.normed = IpcBuffer(T * cfg.hidden * esz, rank, world, group, device)
        self.gated = IpcBuffer(self.ts * cfg.inner * 2, rank, world, group, device)
        self.normed_local = self.normed.view((T, cfg.hidden), norm_dtype)
        self.gated_local = self.gated.view((1, self.ts, cfg.inner), torch.float16)
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._dist = dist

    def barrier(self) -> None:
        """Orders this GPU's next kernel after every rank's kernels so far (a
        one-element NCCL all-reduce on the stream)."""
        self._dist.all_reduce(self.flag, group=self.group)

    def close(self) -> None:
        self.normed.close()
        self.gated.close()


def _lib_dtype(t: torch.Tensor) -> int:
    return {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[t.dtype]


def layer_forward(layer: StackLayer, state: DeltaNetState, normed: torch.Tensor, group=None,
                  rank: int = 0, world: int = 1) -> torch.Tensor:
    """One layer on its rank's heads: normed [T][hidden] (the same on every rank)
    -> the layer output [T][hidden] fp32 (the same on every rank)."""
    import torch.distributed as dist
    cfg = layer.cfg
    T = normed.shape[0]
    if T % world:
        raise GDNError(-2, f"T={T} does not split over {world} ranks")
    ts = T // world
    gated = prefill_gated(layer.heads, state, normed)
    if world > 1:
        gathered = torch.empty((world * T, gated.shape[1]), dtype=gated.dtype, device=gated.device)
        dist.all_gather_into_tensor(gathered, gated, group=group)
        gathered = gathered.view(world, T, -1)
    else:
        gathered = gated.view(1, T, -1)
    part = out_proj_gathered(layer.out_qs, layer.out_d, cfg, gathered, rank * ts, (rank + 1) * ts)
    if world == 1:
        return part
    out = torch.empty((T, cfg.hidden), dtype=torch.float32, device=part.device)
    dist.all_gather_into_tensor(out, part, group=group)
    return out


def prefill_scatter(w: DeltaNetWeights, state: DeltaNetState, x: torch.Tensor, dst: list[int], ld: int, col0: int,
                    stream=None) -> None:
    """gdn_prefill_scatter: x [T][hidden] -> token slice r of the gated heads
    stored at device pointer dst[r] ([T/len(dst)][ld] fp16, from column col0)."""
    T = x.shape[0]
    ws = prefill_workspace(w.cfg, T, x.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    arr = (C.c_void_p * len(dst))(*dst)
    check(lib().gdn_prefill_scatter(C.byref(w.struct()), T, x.data_ptr(), _lib_dtype(x), arr, len(dst), ld, col0,
                                    state.S[0].data_ptr(), state.conv_buf[0].data_ptr(), state.conv_pos.data_ptr(),
                                    base, ws.numel() - (base - ws.data_ptr()), _stream(stream, x.device)))


def add_rmsnorm_bcast(x: torch.Tensor, add: torch.Tensor | None, w: torch.Tensor | None, dst: list[int],
                      dtype: torch.dtype, row0: int, stream=None) -> None:
    """gdn_add_rmsnorm_bcast: x [t][hidden] += add; rmsnorm(x) * w stored as rows
    [row0, row0 + t) of every [T][hidden] buffer at the device pointers dst."""
    T, H = x.shape
    arr = (C.c_void_p * len(dst))(*dst)
    check(lib().gdn_add_rmsnorm_bcast(x.data_ptr(), add.data_ptr() if add is not None else None,
                                      w.data_ptr() if w is not None else None, arr, len(dst),
                                      _lib_dtype(torch.empty((), dtype=dtype)), T, H, row0,
                                      _stream(stream, x.device)))


def _prefill_stack_fused(layers: list[StackLayer], states: list[DeltaNetState], x: torch.Tensor, group, rank: int,
                         world: int, ps: PeerStack) -> torch.Tensor:
    """The residual stays sharded by tokens (rank r owns rows [r T/G, (r+1) T/G));
    per layer:
      1. RMSNorm of this rank's rows, stored into every rank's copy of the
         layer input (gdn_add_rmsnorm_bcast: all-gather fused into the norm);
      2. barrier;
      3. chunked prefill of this rank's heads over all T tokens, the gated rows
         of token slice s stored into rank s's out_proj operand
         (gdn_prefill_scatter: all-to-all fused into the last prefill kernel);
      4. barrier;
      5. out_proj of this rank's token slice, read from local memory (the
         single-GPU k order: bit-identical), kept as the next residual add.
    The barriers also keep a rank from overwriting a buffer a peer still
    reads: step 1 of layer l+1 follows every rank's step 3 of layer l, step 3
    of layer l+1 every rank's step 5 of layer l.  One all-gather of the fp32
    residual at the end.  Per layer a rank receives (G-1)/G T hidden x 2 B of
    input rows and (G-1)/G (T/G) inner x 2 B of head columns, against
    (G-1)/G T (inner x 2 + hidden x 4) B for the all-gathers of `layer_forward`."""
    import torch.distributed as dist
    T, H = x.shape
    ts = T // world
    xs = x[rank * ts:(rank + 1) * ts]
    delta = None
    for layer, st in zip(layers, states):
        cfg = layer.cfg
        add_rmsnorm_bcast(xs, delta, None, ps.normed.ptrs, ps.norm_dtype, rank * ts)
        ps.barrier()
        inner_local = layer.heads.cfg.inner
        prefill_scatter(layer.heads, st, ps.normed_local, ps.gated.ptrs, cfg.inner, rank * inner_local)
        ps.barrier()
        delta = out_proj_gathered(layer.out_qs, layer.out_d, cfg, ps.gated_local, 0, ts)
    add_rmsnorm(xs, delta, None, ps.normed_local[rank * ts:(rank + 1) * ts])  # the last residual add
    full = torch.empty_like(x)
    dist.all_gather_into_tensor(full, xs, group=group)
    x.copy_(full)
    return x


def prefill_stack(layers: list[StackLayer], states: list[DeltaNetState], x: torch.Tensor, group=None,
                  rank: int = 0, world: int = 1, norm_dtype=torch.bfloat16,
                  peers: PeerStack | None = None) -> torch.Tensor:
    """x [T][hidden] fp32 hidden states -> after len(layers) residual DeltaNet
    layers (x <- x + DN_l(rmsnorm(x))), in place; rmsnorm weights are ones.
    With `peers` (world > 1) the exchanges are stores over NVLink fused into
    the kernels (`_prefill_stack_fused`); without, NCCL all-gathers."""
    if peers is not None and world > 1:
        if peers.T != x.shape[0] or peers.norm_dtype != norm_dtype:
            raise GDNError(-2, "PeerStack was made for another prompt length or input type")
        return _prefill_stack_fused(layers, states, x, group, rank, world, peers)
    T, H = x.shape
    normed = torch.empty((T, H), dtype=norm_dtype, device=x.device)
    delta = None
    for layer, st in zip(layers, states):
        add_rmsnorm(x, delta, None, normed)
        delta = layer_forward(layer, st, normed, group, rank, world)
    add_rmsnorm(x, delta, None, normed)  # the last residual add (normed: the next block's input)
    return x
