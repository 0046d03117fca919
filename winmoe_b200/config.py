"""Layer dimensions of the Gated DeltaNet layer.

Mirrors dn_init_dims (engine/runtime/deltanet_impl.h:32-44): from the GGUF
keys ssm.inner_size, ssm.group_count and ssm.state_size the layer derives
Hv = inner / d value heads, Hk key heads, hpg = Hv / Hk, KEY = Hk*d,
QKV = 2*KEY + inner and the gate width = inner.
"""
from __future__ import annotations

from dataclasses import dataclass

CONV_WIDTH = 4  # DN_CONV_WIDTH, engine/runtime/deltanet_impl.h:45


@dataclass(frozen=True)
class GDNConfig:
    hidden: int = 2048
    num_k_heads: int = 16
    num_v_heads: int = 32
    head_dim: int = 128

    @classmethod
    def from_gguf(cls, hidden: int, ssm_inner_size: int, ssm_group_count: int, ssm_state_size: int) -> "GDNConfig":
        """dn_init_dims with the reference's defaults for missing (<= 0) keys."""
        d = ssm_state_size if ssm_state_size > 0 else 128
        hk = ssm_group_count if ssm_group_count > 0 else 16
        inner = ssm_inner_size if ssm_inner_size > 0 else 8192
        return cls(hidden=hidden, num_k_heads=hk, num_v_heads=inner // d, head_dim=d)

    @property
    def heads_per_group(self) -> int:
        return self.num_v_heads // self.num_k_heads

    @property
    def key_dim(self) -> int:
        return self.num_k_heads * self.head_dim

    @property
    def inner(self) -> int:
        return self.num_v_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return 2 * self.key_dim + self.inner

    @property
    def in_proj_rows(self) -> int:
        """Rows of the fused input projection: qkv | z | beta | alpha."""
        return self.qkv_dim + self.inner + 2 * self.num_v_heads

    def validate(self) -> None:
        if self.head_dim != 128:
            raise ValueError(f"head_dim must be 128 (got {self.head_dim})")
        if self.num_v_heads % self.num_k_heads:
            raise ValueError("num_v_heads must be a multiple of num_k_heads")
        if self.hidden % 256:
            raise ValueError("hidden must be a multiple of 256")


# The 35B-class dims of the benchmark configs (hidden 2048, 16 QK / 32 V heads).
DIMS_35B = GDNConfig(2048, 16, 32, 128)
