"""bench.py on the CPU: the algorithmic byte/FLOP figures its rooflines divide
by, and the reference arm's JSON line (it needs no GPU)."""
import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from winmoe_b200.config import DIMS_35B as cfg

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_decode_step_bytes(bench):
    # state r+w, conv window, conv weights, Q8_0 weights, bf16 x in, fp32 out
    want = (256 * 32 * 128 * 128 * 8 + 256 * 4 * 8192 * 4 + 8192 * 16 + 35_790_848 + 256 * 2048 * 2
            + 256 * 2048 * 4)
    assert bench.step_bytes(cfg, 256) == want
    assert abs(want - 1.146e9) / 1.146e9 < 1e-3


def test_q4k_call_bytes(bench):
    w = 18_948_096  # Q4_K bytes of the four projections
    for B in (1, 8, 32):
        assert bench.q4k_call_bytes(cfg, B) == w + B * (2048 + 4096) * 4 * 2


def test_state_kernel_bytes(bench):
    assert bench.state_kernel_bytes(cfg, 256) == 1_088_487_424


def test_prefill_flops(bench):
    # projections + chunk form per token (C = 64, d = 128, Hv = 32)
    assert abs(bench.prefill_flops_per_token(cfg) - 73.23e6) / 73.23e6 < 1e-3


def test_reference_arm_line():
    env = dict(os.environ, OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    # stdout carries the JSON line alone: what native code prints (the reference build's own
    # diagnostics, NCCL's version banner) goes to stderr
    lines = r.stdout.strip().splitlines()
    assert len(lines) == 1, lines[:3]
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
