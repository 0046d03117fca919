"""GGUF bridge (winmoe_b200.gguf) on the CPU: files written here read back
exactly, and the reference's own parser (gguf_parser.h, compiled in the
oracle build) reads them the same way -- names, types, dims, offsets, the
data start and the metadata keys."""
import numpy as np
import pytest

from oracle import oracle as O
from winmoe_b200 import GDNConfig, synth
from winmoe_b200.gguf import GGML_F32, GGUFFile, layer_tensor_list, model_kv, write_gguf

CFG = GDNConfig(512, 2, 4, 128)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    """A 3-layer DeltaNet file: layers 0 and 2 Q8_0, layer 1 Q4_K."""
    path = tmp_path_factory.mktemp("gguf") / "dn.gguf"
    layers = {0: synth.layer_tensors(CFG, layer=0), 1: synth.layer_tensors(CFG, layer=1, weight_type=12),
              2: synth.layer_tensors(CFG, layer=2)}
    tensors = [t for l, lt in layers.items() for t in layer_tensor_list(l, lt)]
    tensors.append(("output_norm.weight", GGML_F32, (CFG.hidden,), np.ones(CFG.hidden, np.float32)))
    write_gguf(path, model_kv(CFG, 3), tensors)
    return path, layers


def test_round_trip(model):
    path, layers = model
    g = GGUFFile(path)
    assert g.version == 3 and g.config() == CFG
    assert g.deltanet_layers() == [0, 1, 2]
    for l, want in layers.items():
        cfg, t = g.deltanet_layer(l)
        assert cfg == CFG and t.weight_type == want.weight_type
        np.testing.assert_array_equal(t.in_proj, want.in_proj)
        np.testing.assert_array_equal(t.out_proj, want.out_proj)
        for name in ("conv1d_w", "ssm_a", "dt_bias", "head_norm"):
            np.testing.assert_array_equal(getattr(t, name), getattr(want, name))


def test_reference_parser_reads_the_file(model):
    if not O.ref_available():
        pytest.skip("the reference build needs AVX-512 on this host")
    path, layers = model
    g = GGUFFile(path)
    R = O.ref()
    meta = R.gguf_probe(path)
    assert meta["n_tensors"] == len(g.tensors)
    assert (meta["hidden"], meta["ssm_inner"], meta["ssm_groups"], meta["ssm_state"], meta["ssm_conv"],
            meta["layers"]) == (CFG.hidden, CFG.inner, CFG.num_k_heads, CFG.head_dim, 4, 3)
    assert meta["data_start"] == g.data_start
    for name, t in g.tensors.items():
        r = R.gguf_tensor(path, name)
        assert (r["type"], r["dims"], r["offset"]) == (t.ggml_type, t.dims, t.offset), name


def test_bad_layer_is_rejected(model, tmp_path):
    path, layers = model
    bad = tmp_path / "bad.gguf"
    t = layer_tensor_list(0, layers[0])
    t = [x for x in t if not x[0].endswith("ssm_beta.weight")]
    write_gguf(bad, model_kv(CFG, 1), t)
    with pytest.raises(KeyError):
        GGUFFile(bad).deltanet_layer(0)
