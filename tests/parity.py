"""Parity measures shared by the tests: distance in units in the last place (ulp) between tensors.

The bar for the floating-point ops is <= 1 ulp of the output type (bf16, fp16, or one e4m3 step)
against the oracle; integer/byte work (the gather, the residual sum) is bit-exact.
"""
from __future__ import annotations

import torch

TOL_ULP = 1  # north-star bar for norm / silu / rope outputs


def _ordered16(t: torch.Tensor) -> torch.Tensor:
    i = t.contiguous().view(torch.int16).to(torch.int32)
    return torch.where(i < 0, -(i & 0x7FFF), i)


def _ordered8(t: torch.Tensor) -> torch.Tensor:
    i = t.contiguous().view(torch.uint8).to(torch.int32)
    return torch.where(i >= 0x80, -(i & 0x7F), i)


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Elementwise |a - b| in ulps of their (common) 16-bit or 8-bit float type, on the CPU."""
    a, b = a.detach().cpu(), b.detach().cpu()
    assert a.dtype == b.dtype and a.shape == b.shape, (a.dtype, b.dtype, a.shape, b.shape)
    if a.element_size() == 2:
        return (_ordered16(a) - _ordered16(b)).abs()
    if a.element_size() == 1:
        return (_ordered8(a) - _ordered8(b)).abs()
    raise TypeError(f"ulp_distance: unsupported dtype {a.dtype}")


def assert_ulp(actual: torch.Tensor, expected: torch.Tensor, tol: int = TOL_ULP, what: str = "") -> dict:
    """Asserts max ulp distance <= tol (NaNs must coincide); returns stats for reporting."""
    a, e = actual.detach().cpu(), expected.detach().cpu()
    fa, fe = a.float(), e.float()
    nan_a, nan_e = torch.isnan(fa), torch.isnan(fe)
    assert torch.equal(nan_a, nan_e), f"{what}: NaN positions differ"
    d = ulp_distance(a, e)
    d = torch.where(nan_a, torch.zeros_like(d), d)
    mx = int(d.max()) if d.numel() else 0
    stats = {"max_ulp": mx, "n": d.numel(), "exact_frac": float((d == 0).float().mean()) if d.numel() else 1.0}
    if mx > tol:
        idx = int(d.flatten().argmax())
        raise AssertionError(f"{what}: max ulp distance {mx} > {tol} at flat index {idx} "
                             f"(got {fa.flatten()[idx].item()!r}, expected {fe.flatten()[idx].item()!r}); {stats}")
    return stats


def assert_bits_equal(actual: torch.Tensor, expected: torch.Tensor, what: str = "") -> None:
    a, e = actual.detach().cpu().contiguous(), expected.detach().cpu().contiguous()
    assert a.shape == e.shape and a.dtype == e.dtype, (what, a.shape, e.shape, a.dtype, e.dtype)
    ia = a.view(torch.uint8) if a.element_size() == 1 else a.view(torch.int16 if a.element_size() == 2 else torch.int32)
    ie = e.view(ia.dtype)
    if not torch.equal(ia, ie):
        n = int((ia != ie).sum())
        raise AssertionError(f"{what}: {n} of {ia.numel()} elements differ bitwise")
