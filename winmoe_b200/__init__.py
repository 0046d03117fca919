"""winmoe_b200: the Gated DeltaNet layer of WinMoE's Qwen3.5-MoE engine, on B200 (sm_100a).

The compute path is the CUDA library winmoe_b200/libwinmoe_gdn.so (C ABI in
include/winmoe_gdn.h and include/gpu_offload_gdn.h); this package is its host
side.  There is no CPU fallback: without the library every entry point raises.
"""
from ._lib import GDNError, GGML_Q4_K, GGML_Q8_0, HEAD_MAP_GROUPED, HEAD_MAP_INTERLEAVED, lib
from .config import DIMS_35B, GDNConfig
from .gguf import GGUFFile
from .layer import (DeltaNetState, DeltaNetWeights, decode_step, deltanet_forward, dequant_q4_k, dequant_q8_0,
                    gemm_q4_k, gemm_q8_0, prefill, q8_0_planes)

__all__ = [
    "GDNError", "GGML_Q4_K", "GGML_Q8_0", "HEAD_MAP_GROUPED", "HEAD_MAP_INTERLEAVED", "lib",
    "DIMS_35B", "GDNConfig", "GGUFFile", "DeltaNetState", "DeltaNetWeights", "decode_step", "deltanet_forward",
    "dequant_q4_k", "dequant_q8_0", "gemm_q4_k", "gemm_q8_0", "prefill", "q8_0_planes",
]
