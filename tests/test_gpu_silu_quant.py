"""Parity of the fused SiLU-and-mul + fp8 activation quantisation kernel.

Two bars: (1) against the oracle, <= 1 e4m3 step (the activation may sit 1 bf16 ulp apart, which
can move the quantised byte by one step); (2) against the unfused pair the reference runs,
``quantize_fp8(silu_and_mul(x), scale)``, computed here from this package's own silu_and_mul output
and torch's quantisation expression on the GPU: bit-exact, because the fused kernel rounds the
activation exactly as silu_and_mul stores it before quantising. Covers the vector path, the scalar
path (odd d, unaligned strides), saturation at +-448, fp16, leading batch dimensions, empty batches,
a 0-dim scale (FP8Linear.activation_scale) and configuration 2's shape.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_bits_equal, assert_ulp

pytestmark = pytest.mark.gpu

FP8 = torch.float8_e4m3fn


def _unfused(act: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """quantize_fp8 of devstral2.py:93-95 as its compiled kernel evaluates it: fp32 quotient of the
    upcast activation, clamp, one rounding to e4m3."""
    return (act.float() / scale.float()).clamp(-448.0, 448.0).to(FP8)


def _check(cuda, T, d, scale, xscale=3.0, dtype=torch.bfloat16, seed=3):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, 2 * d, generator=g) * xscale).to(dtype)
    xd = x.to(cuda)
    s = torch.tensor(scale, dtype=torch.float32, device=cuda)
    q = mas_b200.silu_and_mul_quant(xd, s)
    assert q.dtype == FP8 and q.shape == (T, d)
    assert_bits_equal(q, _unfused(mas_b200.silu_and_mul(xd), s), f"fused vs unfused T={T} d={d}")
    return assert_ulp(q.cpu(), oracle.silu_and_mul_quant(x, scale), what=f"silu quant T={T} d={d} s={scale}")


@pytest.mark.parametrize("T,d", [(1, 8), (8, 4096), (3, 28672), (17, 1000), (130, 256), (5, 12)])
def test_silu_quant_shapes(cuda, T, d):
    _check(cuda, T, d, 0.0137)


@pytest.mark.parametrize("scale", [1e-3, 0.05, 1.7, 300.0, 0.125, 4.0])
def test_silu_quant_scales_and_saturation(cuda, scale):
    """A small scale drives most outputs to +-448 (saturation); a large one into e4m3 subnormals.
    Power-of-two scales put many quotients exactly on e4m3 ties (the kernel's exact fallback)."""
    _check(cuda, 6, 2048, scale)


def test_silu_quant_fp16(cuda):
    _check(cuda, 9, 1024, 0.02, dtype=torch.float16)


def test_silu_quant_out_arg_batch_dims_and_0dim_scale(cuda):
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(2, 3, 2 * 512, generator=g) * 2).to(torch.bfloat16)
    out = torch.empty(2, 3, 512, dtype=FP8, device=cuda)
    scale = torch.tensor(0.01, device=cuda)  # 0-dim, as FP8Linear registers activation_scale
    ret = mas_b200.silu_and_mul_quant(x.to(cuda), scale, out=out)
    assert ret is out
    assert_ulp(out.cpu().view(6, 512), oracle.silu_and_mul_quant(x.view(6, 1024), 0.01), what="batch dims")


def test_silu_quant_empty_and_checks(cuda):
    s = torch.ones((), device=cuda)
    out = mas_b200.silu_and_mul_quant(torch.empty(0, 64, dtype=torch.bfloat16, device=cuda), s)
    assert out.shape == (0, 32) and out.dtype == FP8
    with pytest.raises(ValueError):
        mas_b200.silu_and_mul_quant(torch.empty(2, 6, dtype=torch.bfloat16, device=cuda), s)
    with pytest.raises(ValueError):
        mas_b200.silu_and_mul_quant(torch.empty(2, 32, dtype=torch.bfloat16, device=cuda), s,
                                    out=torch.empty(2, 16, dtype=torch.bfloat16, device=cuda))


@pytest.mark.parametrize("d,in_stride,out_stride", [(13, 26, 13), (64, 132, 64), (64, 128, 72), (64, 128, 68)])
def test_silu_quant_c_abi_scalar_and_strided(cuda, d, in_stride, out_stride):
    """Odd d and unaligned strides reach the scalar kernel through the C ABI; bytes past d untouched."""
    T = 7
    g = torch.Generator().manual_seed(9)
    buf = (torch.randn(T, in_stride, generator=g) * 3).to(torch.bfloat16)
    outd = torch.zeros(T, out_stride, dtype=torch.uint8, device=cuda)
    ind = buf.to(cuda)
    sd = torch.tensor([0.03], device=cuda)
    rc = mas_b200._lib.lib.mas_silu_and_mul_quant(outd.data_ptr(), ind.data_ptr(), sd.data_ptr(), T, d, out_stride,
                                                  in_stride, 0, 3, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, mas_b200.status_string(rc)
    ref = oracle.silu_and_mul_quant(buf[:, : 2 * d].contiguous(), 0.03)
    assert_ulp(outd.cpu()[:, :d].contiguous().view(FP8), ref, what="C ABI")
    assert torch.count_nonzero(outd.cpu()[:, d:]) == 0
    # a non-e4m3 output type and a missing scale are rejected
    assert mas_b200._lib.lib.mas_silu_and_mul_quant(outd.data_ptr(), ind.data_ptr(), sd.data_ptr(), T, d,
                                                    out_stride, in_stride, 0, 0, 1, None) == -2
    assert mas_b200._lib.lib.mas_silu_and_mul_quant(outd.data_ptr(), ind.data_ptr(), None, T, d, out_stride,
                                                    in_stride, 0, 3, 1, None) == -1


def test_silu_quant_config2_shape(cuda):
    """Configuration 2's gate_up [8192, 65536] quantised with a down_proj-like scale; fused == unfused."""
    x = workloads.silu_inputs(cuda)
    s = torch.tensor(0.0137, device=cuda)
    q = mas_b200.silu_and_mul_quant(x, s)
    assert_bits_equal(q, _unfused(mas_b200.silu_and_mul(x), s), "config 2 fused vs unfused")
    rows = torch.arange(0, x.shape[0], 97)
    assert_ulp(q[rows].cpu(), oracle.silu_and_mul_quant(x[rows].cpu(), 0.0137), what="config 2 sampled rows")
