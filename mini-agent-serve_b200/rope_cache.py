"""fp32 cos|sin caches for the rotary-embedding kernels (built once on the host, as the reference does).

`yarn_cos_sin_cache` produces the cache Devstral2Model registers as a buffer
(miniagentserve/models/devstral2/devstral2.py:44-90, :265): YaRN-blended inverse frequencies times
the attention scaling, cos in the first rotary_dim/2 columns and sin in the rest, every step in fp32
on the CPU. The arithmetic is the reference's, step for step, because the cache must be bit-identical
to the one the reference model would hold; the code around it is this package's own.

`plain_cos_sin_cache` is the un-scaled special case (inv_freq = theta^(-2i/D), no YaRN blend, no
attention scaling) that the benchmark configurations use with theta = 1e9.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any

import torch

__all__ = ["YarnParams", "yarn_params_from_config", "yarn_inv_freq", "yarn_cos_sin_cache",
           "plain_inv_freq", "plain_cos_sin_cache"]


@dataclass(frozen=True)
class YarnParams:
    """The rope fields of Devstral2Config (miniagentserve/models/devstral2/configs.py:16-25)."""

    head_dim: int
    rope_theta: float
    max_position_embeddings: int
    rope_factor: float
    rope_original_max_position_embeddings: int
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    rope_mscale: float = 0.0
    rope_mscale_all_dim: float = 0.0
    rope_truncate: bool = True


def yarn_params_from_config(config: Any) -> YarnParams:
    """Reads the rope fields off a Devstral2Config-like object (same attribute names)."""
    return YarnParams(**{f: getattr(config, f) for f in YarnParams.__dataclass_fields__})


def _mscale(scale: float, mscale: float = 1.0) -> float:
    return 1.0 if scale <= 1 else 0.1 * mscale * math.log(scale) + 1.0


def _correction_dim(rotations: float, dim: int, base: float, original_max: int) -> float:
    """The rotary dimension index whose wavelength fits `rotations` turns into original_max positions."""
    return (dim * math.log(original_max / (rotations * 2 * math.pi))) / (2 * math.log(base))


def yarn_inv_freq(p: YarnParams) -> tuple[torch.Tensor, float]:
    """YaRN inverse frequencies (fp32, [head_dim/2]) and the attention scaling factor."""
    dim, base, factor = p.head_dim, p.rope_theta, p.rope_factor
    lo = _correction_dim(p.rope_beta_fast, dim, base, p.rope_original_max_position_embeddings)
    hi = _correction_dim(p.rope_beta_slow, dim, base, p.rope_original_max_position_embeddings)
    if p.rope_truncate:
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, dim - 1)
    if lo == hi:
        hi += 0.001
    freq_base = base ** (torch.arange(0, dim, 2, dtype=torch.float, device="cpu") / dim)
    extrapolated = 1.0 / freq_base
    interpolated = 1.0 / (factor * freq_base)
    ramp = torch.clamp((torch.arange(dim // 2, dtype=torch.float, device="cpu") - lo) / (hi - lo), 0, 1)
    keep = 1 - ramp
    inv_freq = interpolated * (1 - keep) + extrapolated * keep
    if p.rope_mscale and p.rope_mscale_all_dim:
        scaling = _mscale(factor, p.rope_mscale) / _mscale(factor, p.rope_mscale_all_dim)
    else:
        scaling = _mscale(factor)
    return inv_freq, scaling


def _cache_from(inv_freq: torch.Tensor, scaling: float, max_positions: int) -> torch.Tensor:
    pos = torch.arange(max_positions, dtype=torch.float, device="cpu")
    angles = pos[:, None] * inv_freq
    return torch.cat((angles.cos(), angles.sin()), dim=-1) * scaling


def yarn_cos_sin_cache(p: YarnParams) -> torch.Tensor:
    """fp32 [max_position_embeddings, head_dim] cache, bit-identical to the reference's buffer."""
    inv_freq, scaling = yarn_inv_freq(p)
    return _cache_from(inv_freq, scaling, p.max_position_embeddings)


def plain_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float, device="cpu") / head_dim))


def plain_cos_sin_cache(head_dim: int, max_positions: int, theta: float) -> torch.Tensor:
    """fp32 [max_positions, head_dim] cache with inv_freq = theta^(-2i/head_dim), no scaling."""
    pos = torch.arange(max_positions, dtype=torch.float, device="cpu")
    angles = pos[:, None] * plain_inv_freq(head_dim, theta)
    return torch.cat((angles.cos(), angles.sin()), dim=-1)
