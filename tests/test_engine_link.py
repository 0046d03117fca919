"""The reference engine's link line against this library.

engine/runtime/winmoe_inference.c calls 18 gpu_* functions of gpu_offload.h:
the DeltaNet / GQA offload and lifetime calls, which libwinmoe_gdn.so exports,
and four expert-cache calls, which stay the reference's own code.  A C
translation unit that calls all of them plus gdn_layer_forward
(tests/c/engine_link.c) is compiled against include/*.h and linked with the
library and the reference's gpu_offload.cu built with
include/gpu_offload_coexist.h forced in (when the reference tree is here; a
stand-in object otherwise): no gpu_* symbol is defined twice, none is missing,
and the library's gpu_init finds the expert module.  On a GPU the binary runs
every call once (tests/c/engine_link.c --run).
"""
import shutil
import subprocess
from pathlib import Path

import pytest

from oracle import oracle as O

ROOT = Path(__file__).resolve().parent.parent
INCLUDE = ROOT / "include"
LIBDIR = ROOT / "winmoe_b200"
CUDA = Path("/usr/local/cuda")
ENGINE_CALLS = {
    "gpu_init", "gpu_set_expert_limit", "gpu_upload_deltanet_weights", "gpu_vram_used_mb",
    "gpu_upload_gqa_weights", "gpu_launch_qkv_gate", "gpu_wait_qkv_gate", "gpu_get_qkv_out", "gpu_get_gate_out",
    "gpu_launch_ssm_out", "gpu_wait_ssm_out", "gpu_get_ssm_out_buf", "gpu_gqa_projections", "gpu_gqa_output",
    "gpu_find_cached_expert", "gpu_expert_ffn_fused", "gpu_cache_expert", "gpu_shutdown",
}


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, f"{' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}"
    return r.stdout


def experts_object(tmp: Path, stub: bool):
    """The expert-cache object: the reference's gpu_offload.cu with the renames, or the stand-in."""
    rd = None if stub else O.ref_dir()
    if rd is not None:
        obj = tmp / "gpu_offload_experts.o"
        _run([str(CUDA / "bin" / "nvcc"), "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-w", "-c",
              str(rd / "engine" / "runtime" / "gpu_offload.cu"), "-include", str(INCLUDE / "gpu_offload_coexist.h"),
              "-o", str(obj)])
        return obj, ["-lcublas"], "reference"
    obj = tmp / "expert_stub.o"
    _run(["gcc", "-O2", "-c", str(ROOT / "tests" / "c" / "expert_stub.c"), "-o", str(obj)])
    return obj, [], "stub"


def link(tmp: Path, stub: bool = False):
    obj, libs, kind = experts_object(tmp, stub)
    exe = tmp / "engine_link"
    _run(["gcc", "-O2", "-std=c11", "-Wall", "-Werror", f"-I{INCLUDE}", f"-I{CUDA / 'include'}",
          str(ROOT / "tests" / "c" / "engine_link.c"), str(obj), f"-L{LIBDIR}", "-lwinmoe_gdn",
          f"-Wl,-rpath,{LIBDIR}", f"-L{CUDA / 'lib64'}", "-lcudart", *libs, "-lm", "-o", str(exe)])
    return exe, kind


def test_engine_calls_are_the_reference_engines():
    src = (ROOT / "tests" / "c" / "engine_link.c").read_text()
    called = {n for n in ENGINE_CALLS if f"{n}(" in src}
    assert called == ENGINE_CALLS
    assert "gdn_layer_forward(" in src


@pytest.mark.skipif(shutil.which("gcc") is None or not (CUDA / "bin" / "nvcc").exists(), reason="needs gcc and nvcc")
def test_engine_links_beside_the_expert_cache(tmp_path):
    exe, kind = link(tmp_path)
    out = _run([str(exe)])
    assert "experts_linked=1" in out, (kind, out)
    # one definition of every gpu_* symbol the engine calls: in the library or in the expert object
    lib_syms = _run(["nm", "-D", "--defined-only", str(LIBDIR / "libwinmoe_gdn.so")]).split()
    obj_syms = _run(["nm", "--defined-only", str(tmp_path / ("gpu_offload_experts.o" if kind == "reference"
                                                             else "expert_stub.o"))]).split()
    for name in ENGINE_CALLS:
        assert (name in lib_syms) + (name in obj_syms) == 1, name


@pytest.mark.gpu
def test_engine_calls_run_on_gpu(tmp_path):
    """Every engine call once on tiny dims, the expert cache a stand-in (the
    reference's source is not on the GPU host), then gdn_layer_forward with
    host weights: a 70-token prompt and a decode token."""
    exe, _ = link(tmp_path, stub=True)
    out = _run([str(exe), "--run"])
    assert "engine calls ok" in out, out
