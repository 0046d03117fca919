"""Generates the golden fixtures of tests/golden/ from the reference itself.

Runs the reference's own CPU code (oracle/_ref/libref_gdn.so, compiled in
place from the reference tree by oracle/Makefile) on the seeded synthetic
inputs of winmoe_b200.synth and stores its outputs.  Inputs are regenerated
from their seeds at test time; their SHA-256 is stored so that a change in
the generators is caught instead of silently comparing different inputs.

  python tests/golden/make_golden.py     (needs the reference tree and an AVX-512 host)
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402
from winmoe_b200 import synth  # noqa: E402
from winmoe_b200.config import DIMS_35B, GDNConfig  # noqa: E402

OUT = Path(__file__).resolve().parent

SMALL = GDNConfig(hidden=256, num_k_heads=1, num_v_heads=2, head_dim=128)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def layer_case(R, cfg, steps, act_mode, layer=0, s0_std=0.0):
    t = synth.layer_tensors(cfg, layer=layer)
    xs = synth.hidden_states(steps, cfg.hidden, seed=100 + layer)
    S = (synth.prefilled_state(cfg, 0, std=s0_std) if s0_std else
         np.zeros((cfg.num_v_heads, cfg.head_dim, cfg.head_dim), np.float32))
    cb = np.zeros((4, cfg.qkv_dim), np.float32)
    pos = np.zeros(1, np.int32)
    outs = np.stack([R.deltanet_forward(cfg, x, S, cb, pos, t, act_mode=act_mode) for x in xs])
    inputs = sha(t.in_proj, t.out_proj, t.conv1d_w, t.ssm_a, t.dt_bias, t.head_norm, xs)
    return outs, S, cb, pos, inputs


def main():
    if not O.ref_available():
        raise SystemExit("needs oracle/_ref/libref_gdn.so and an AVX-512/VNNI host")
    R = O.ref()
    fx = {}

    # Q8_0 row dequant (q8_dequant_row) and the two projection semantics.
    blocks = synth.q8_0_blocks(96, 256, seed=11)
    x = synth.hidden_states(1, 256, seed=12)[0]
    fx["q8_blocks_sha"] = np.frombuffer(bytes.fromhex(sha(blocks, x)), np.uint8)
    fx["q8_dequant"] = R.q8_0_dequant(blocks, 96 * 256)
    fx["q8_matvec_exact"] = R.quant_matvec(blocks, x, 96, 256, 8, O.ACT_EXACT)    # out_dim < 128: fp32 path
    blocks_l = synth.q8_0_blocks(160, 512, seed=13)
    xl = synth.hidden_states(1, 512, seed=14)[0]
    fx["q8l_sha"] = np.frombuffer(bytes.fromhex(sha(blocks_l, xl)), np.uint8)
    fx["q8l_matvec_exact"] = R.quant_matvec(blocks_l, xl, 160, 512, 8, O.ACT_EXACT)  # Q8_K int8 path
    fx["q8l_matvec_fp32"] = R.quant_matvec(blocks_l, xl, 160, 512, 8, O.ACT_FP32)

    # Q8_K activation quantisation (quantize_row_q8_K): d, qs, bsums bytes.
    xq = synth.hidden_states(1, 1024, seed=15)[0] * 3.0
    xq[300:556] = 0.0  # an all-zero block takes the amax < 1e-10 branch
    fx["q8k_x_sha"] = np.frombuffer(bytes.fromhex(sha(xq)), np.uint8)
    fx["q8k_bytes"] = R.quantize_q8_K(xq)

    # Q4_K: scale decode of every 12-byte pattern class, and q4k_matvec (int8 activations).
    b4 = synth.q4_k_blocks(64, 512, seed=16)
    x4 = synth.hidden_states(1, 512, seed=17)[0]
    fx["q4_sha"] = np.frombuffer(bytes.fromhex(sha(b4, x4)), np.uint8)
    fx["q4_matvec_exact"] = R.quant_matvec(b4, x4, 64, 512, 12, O.ACT_EXACT)
    fx["q4_matvec_fp32"] = R.quant_matvec(b4, x4, 64, 512, 12, O.ACT_FP32)
    sc = np.stack([np.concatenate(R.q4k_scales(b4.reshape(64, 2, 144)[r, 0, 4:16])) for r in range(64)])
    fx["q4_scales"] = sc

    # test_q4k.c:21-43: d = 1.0, scales[0] = 1, every qs byte 0x0F, x = 1 -> 240.0
    # through the reference's float fallback q4k_dot_block.
    kat = np.zeros(144, np.uint8)
    kat[0:2] = np.array([0x00, 0x3C], np.uint8)
    kat[4] = 1
    kat[16:] = 0x0F
    fx["q4k_kat_dot_block"] = np.array([R.q4k_dot_block(kat, np.ones(256, np.float32))], np.float32)

    # RMSNorm (attention.h:29-44).
    xr = synth.hidden_states(1, 2048, seed=18)[0]
    wr = (1.0 + 0.1 * synth.hidden_states(1, 2048, seed=19)[0]).astype(np.float32)
    fx["rms_sha"] = np.frombuffer(bytes.fromhex(sha(xr, wr)), np.uint8)
    fx["rmsnorm"] = R.rmsnorm(xr, wr)

    # Full layer, small dims, both modes, 6 steps from zero and from a prefilled state.
    for mode, name in ((O.ACT_EXACT, "exact"), (O.ACT_FP32, "fp32")):
        outs, S, cb, pos, h = layer_case(R, SMALL, 6, mode)
        fx[f"small_{name}_out"], fx[f"small_{name}_S"], fx[f"small_{name}_conv"] = outs, S, cb
        fx[f"small_{name}_pos"] = pos
        fx["small_inputs_sha"] = np.frombuffer(bytes.fromhex(h), np.uint8)
    outs, S, cb, pos, h = layer_case(R, SMALL, 5, O.ACT_FP32, layer=1, s0_std=0.05)
    fx["small_prefilled_out"], fx["small_prefilled_S"] = outs, S
    fx["small_prefilled_sha"] = np.frombuffer(bytes.fromhex(h), np.uint8)

    # Full layer at the benchmark dims (config 1), 4 steps, fp32 activations.
    outs, S, cb, pos, h = layer_case(R, DIMS_35B, 4, O.ACT_FP32)
    fx["d35_out"] = outs
    fx["d35_S_head_sums"] = S.astype(np.float64).sum(axis=(1, 2))
    fx["d35_S_sha"] = np.frombuffer(bytes.fromhex(sha(S)), np.uint8)
    fx["d35_conv_sha"] = np.frombuffer(bytes.fromhex(sha(cb)), np.uint8)
    fx["d35_inputs_sha"] = np.frombuffer(bytes.fromhex(h), np.uint8)

    np.savez_compressed(OUT / "reference_cpu.npz", **fx)
    print("wrote", OUT / "reference_cpu.npz", sum(v.nbytes for v in fx.values()), "bytes raw")


if __name__ == "__main__":
    main()
