"""Host-side logic on CPU: dims derivation, GGUF block helpers, sharding and the
multi-rank timing reduction (gloo, world size 2)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O
from winmoe_b200 import dist as D, synth
from winmoe_b200.config import DIMS_35B, GDNConfig


def test_dims_follow_dn_init_dims():
    c = GDNConfig.from_gguf(2048, 4096, 16, 128)
    assert (c.num_v_heads, c.heads_per_group, c.key_dim, c.qkv_dim, c.inner) == (32, 2, 2048, 8192, 4096)
    assert c.in_proj_rows == 8192 + 4096 + 64
    # missing keys fall back to the reference defaults (deltanet_impl.h:33-35)
    d = GDNConfig.from_gguf(4096, 0, 0, 0)
    assert (d.head_dim, d.num_k_heads, d.num_v_heads) == (128, 16, 64)
    with pytest.raises(ValueError):
        GDNConfig(2048, 16, 30, 128).validate()
    with pytest.raises(ValueError):
        GDNConfig(2048, 16, 32, 64).validate()


def test_q8_0_planes_and_dequant_match_the_oracle():
    b = synth.q8_0_blocks(40, 256, seed=3)
    qs, d = synth.q8_0_split(b, 40, 256)
    assert qs.shape == (40, 256) and d.shape == (40, 8)
    w = synth.q8_0_dequant_np(b, 40, 256)
    want = O.port().q8_0_dequant(b, 40 * 256).reshape(40, 256)
    assert np.array_equal(w.view(np.uint32), want.view(np.uint32))


def test_block_generators_are_in_range():
    b = synth.q8_0_blocks(8, 64, seed=1).reshape(8, 2, 34)
    q = b[:, :, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    d = np.ascontiguousarray(b[:, :, :2]).view(np.float16).astype(np.float32)
    assert (d >= 0).all()
    b4 = synth.q4_k_blocks(4, 512, seed=2)
    assert b4.shape == (4, 2 * 144)


def test_in_proj_split_is_row_exact():
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg)
    parts = t.split_in_proj()
    assert parts["w_qkv"].shape[0] == cfg.qkv_dim
    assert parts["w_gate"].shape[0] == cfg.inner
    assert parts["w_beta"].shape[0] == parts["w_alpha"].shape[0] == cfg.num_v_heads
    again = np.concatenate([parts["w_qkv"], parts["w_gate"], parts["w_beta"], parts["w_alpha"]])
    assert np.array_equal(again, t.in_proj)


def test_layer_seeds_differ_per_layer():
    cfg = GDNConfig(256, 1, 2, 128)
    a, b = synth.layer_tensors(cfg, 0), synth.layer_tensors(cfg, 1)
    assert not np.array_equal(a.in_proj, b.in_proj)
    assert np.array_equal(a.in_proj, synth.layer_tensors(cfg, 0).in_proj)


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (7, 3), (2, 4)])
def test_shard_range_partitions(n, world):
    seen = []
    for r in range(world):
        a, b = D.shard_range(n, r, world)
        seen += list(range(a, b))
        assert abs((b - a) - n / world) < 1
    assert seen == list(range(n))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, stop = D.shard_range(256, rank, world)
        out[rank] = D.max_over_ranks(float(10 * (rank + 1)))
        out[world + rank] = float(stop - start)
    finally:
        torch.distributed.destroy_process_group()


def test_max_over_ranks_gloo_two_ranks():
    world = 2
    out = mp.get_context("spawn").Array("d", 2 * world)
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    assert list(out[:world]) == [20.0, 20.0]
    assert sum(out[world:]) == 256


def test_max_over_ranks_without_group():
    assert D.max_over_ranks(3.5) == 3.5
    assert DIMS_35B.hidden == 2048
