"""The oracle's number formats against torch's conversions (CPU, no GPU).

bf16 and fp16 rounding (RNE) on random and edge values, and the e4m3fn format in both directions:
all 256 codes decoded, and encoding (RNE, saturating at +-448) on random, boundary, subnormal and
tie values, against torch's float8_e4m3fn (which is RNE for in-range values).
"""
from __future__ import annotations

import math

import torch

import oracle


def _bits16(t: torch.Tensor) -> list[int]:
    return [int(v) & 0xFFFF for v in t.view(torch.int16).tolist()]


def test_bf16_rounding_matches_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.randn(4000, generator=g) * 10, torch.randn(1000, generator=g) * 1e-30,
                   torch.tensor([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.0e38, -3.4e38, 1e-45, float("inf")])])
    want = _bits16(x.to(torch.bfloat16))
    got = [oracle.f32_to_bf16_bits(float(v)) for v in x]
    assert got == want


def test_fp16_rounding_matches_torch():
    g = torch.Generator().manual_seed(1)
    x = torch.cat([torch.randn(4000, generator=g) * 100, torch.tensor([65504.0, 65520.0, 6e-8, 3e-8, -0.0])])
    want = _bits16(x.to(torch.float16))
    got = [oracle.f32_to_f16_bits(float(v)) for v in x]
    assert got == want


def test_e4m3_decode_all_codes():
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    want = codes.view(torch.float8_e4m3fn).float().tolist()
    for c, w in zip(range(256), want):
        got = oracle.e4m3_to_f32(c)
        assert (math.isnan(got) and math.isnan(w)) or got == w, (c, got, w)


def test_e4m3_encode_matches_torch_in_range():
    g = torch.Generator().manual_seed(2)
    grid = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    grid = grid[~torch.isnan(grid)]
    mids = (grid[:-1] + grid[1:]) / 2  # exact ties between neighbouring codes (both signs interleaved)
    x = torch.cat([torch.randn(20000, generator=g) * 100, torch.randn(4000, generator=g) * 0.01, grid,
                   mids[torch.isfinite(mids)], torch.tensor([447.99, 448.0, -448.0, 2.0 ** -10, 2.0 ** -9 * 1.5])])
    x = x.clamp(-448, 448)
    want = x.to(torch.float8_e4m3fn).view(torch.uint8).tolist()
    got = [oracle.f32_to_e4m3(float(v)) for v in x]
    bad = [(float(v), a, b) for v, a, b in zip(x, got, want) if a != b]
    assert not bad, bad[:10]


def test_e4m3_saturates_and_keeps_nan():
    assert oracle.f32_to_e4m3(1e6) == 0x7E
    assert oracle.f32_to_e4m3(-1e6) == 0xFE
    assert oracle.f32_to_e4m3(float("inf")) == 0x7E
    assert oracle.f32_to_e4m3(float("-inf")) == 0xFE
    assert oracle.f32_to_e4m3(float("nan")) & 0x7F == 0x7F
    assert oracle.f32_to_e4m3(464.0) == 0x7E  # beyond the max finite, saturated rather than rounded to NaN
