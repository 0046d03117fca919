"""Host logic of the sharded layer stack (no GPU): head ranges, layer slicing
pinned against the CPU oracle, and the collective layout on gloo ranks."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from winmoe_b200 import GDNConfig, GDNError, synth
from winmoe_b200.stack import head_range, slice_layer


def test_head_ranges():
    cfg = GDNConfig(2048, 16, 32, 128)
    for world in (1, 2, 4, 8, 16):
        spans = [head_range(cfg, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 32
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all((h1 - h0) % cfg.heads_per_group == 0 for h0, h1 in spans)
    with pytest.raises(GDNError):
        head_range(cfg, 0, 3)
    with pytest.raises(GDNError):
        head_range(cfg, 0, 32)  # one value head per rank would split a key group


@pytest.mark.parametrize("world", [2, 4])
def test_slices_match_the_whole_layer(world):
    """Every slice's projections and gated head outputs equal the whole layer's,
    bit for bit, over three tokens (state carried)."""
    cfg = GDNConfig(512, 4, 8, 128)
    t = synth.layer_tensors(cfg, layer=1)
    P = O.port()
    xs = synth.hidden_states(3, cfg.hidden, seed=21)

    def run(c, tt):
        parts = tt.split_in_proj()
        S = np.zeros((c.num_v_heads, 128, 128), np.float32)
        cb = np.zeros((4, c.qkv_dim), np.float32)
        pos = np.zeros(1, np.int32)
        outs = []
        for x in xs:
            qkv = P.quant_matvec(parts["w_qkv"], x, c.qkv_dim, c.hidden, 8, O.ACT_FP32)
            z = P.quant_matvec(parts["w_gate"], x, c.inner, c.hidden, 8, O.ACT_FP32)
            b = P.quant_matvec(parts["w_beta"], x, c.num_v_heads, c.hidden, 8, O.ACT_FP32)
            a = P.quant_matvec(parts["w_alpha"], x, c.num_v_heads, c.hidden, 8, O.ACT_FP32)
            outs.append(P.gdn_core(c, qkv, z, a, b, S, cb, pos, tt)[0])
        return np.stack(outs), S

    full, S_full = run(cfg, t)
    for r in range(world):
        h0, h1 = head_range(cfg, r, world)
        sub, ts = slice_layer(cfg, t, h0, h1)
        assert (sub.num_v_heads, sub.num_k_heads) == (h1 - h0, (h1 - h0) // cfg.heads_per_group)
        got, S_sub = run(sub, ts)
        np.testing.assert_array_equal(got, full[:, h0 * 128:h1 * 128])
        np.testing.assert_array_equal(S_sub, S_full[h0:h1])


def _gather_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    T, il = 6, 4
    gated = torch.arange(T * il, dtype=torch.float32).reshape(T, il) + 1000 * rank
    bufs = [torch.empty_like(gated) for _ in range(world)]
    dist.all_gather(bufs, gated)
    gathered = torch.stack(bufs)  # [G][T][iL], the layout gdn_out_proj_gathered reads
    concat = torch.cat([gathered[g] for g in range(world)], dim=1)  # token rows of the whole layer's heads
    ts = T // world
    part = concat[rank * ts:(rank + 1) * ts].sum(dim=1, keepdim=True)  # stand-in for this rank's out_proj rows
    parts = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(parts, part)
    q.put((rank, torch.cat(parts).squeeze(1).tolist()))
    dist.destroy_process_group()


def test_gather_layout_world2():
    """Head blocks gathered as [G][T][iL], token slices of the output gathered
    back in token order: every rank ends with the whole layer's rows."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    T, il = 6, 4
    base = np.arange(T * il, dtype=np.float64).reshape(T, il)
    want = sum((base + 1000 * r).sum(axis=1) for r in range(world))
    for r in range(world):
        np.testing.assert_allclose(res[r], want)
