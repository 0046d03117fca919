"""A DeltaNet layer loaded from a GGUF file through the bridge decodes like
the oracle on the same tensors (Q8_0 and Q4_K layers)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from winmoe_b200 import GDNConfig, layer as L, synth
from winmoe_b200.gguf import GGUFFile, layer_tensor_list, model_kv, write_gguf

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


@pytest.mark.parametrize("wtype", [8, 12])
def test_layer_from_gguf_decodes(tmp_path, wtype):
    cfg = GDNConfig(512, 2, 4, 128)
    t = synth.layer_tensors(cfg, layer=3, weight_type=wtype)
    path = tmp_path / "layer.gguf"
    write_gguf(path, model_kv(cfg, 4), layer_tensor_list(3, t))
    w = L.DeltaNetWeights.from_gguf(GGUFFile(path), 3, device="cuda")
    assert w.cfg == cfg and w.weight_type == wtype
    st = L.DeltaNetState.zeros(cfg, 1, "cuda")
    P = O.port()
    S = np.zeros((cfg.num_v_heads, 128, 128), np.float32)
    cb = np.zeros((4, cfg.qkv_dim), np.float32)
    pos = np.zeros(1, np.int32)
    for i, x in enumerate(synth.hidden_states(3, cfg.hidden, seed=30)):
        y = L.decode_step(w, st, torch.from_numpy(x[None]).cuda()).cpu().numpy()[0]
        want = P.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=O.ACT_FP32)
        assert rel_l2(y, want) <= 1e-3, i
