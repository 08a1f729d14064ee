"""Parity of the SiLU-and-mul kernel against the oracle (<= 1 ulp), including configuration 2 at full size.

Covers the vector path (d % 8 == 0, aligned rows), the scalar path (d % 8 != 0 through the C ABI, and
unaligned row strides), wide value ranges (exp overflow on both sides), empty batches, leading batch
dimensions and the flashinfer argument checks of the Python wrapper.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_ulp

pytestmark = pytest.mark.gpu


def _check(cuda, T, d, scale=1.0, dtype=torch.bfloat16, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(T, 2 * d, generator=g) * scale).to(dtype)
    out = mas_b200.silu_and_mul(x.to(cuda))
    ref = oracle.silu_and_mul(x)
    return assert_ulp(out.cpu(), ref, what=f"silu T={T} d={d} scale={scale}")


@pytest.mark.parametrize("T,d", [(1, 8), (3, 4096), (4, 28672), (17, 1000), (2, 32768), (130, 256), (5, 12)])
def test_silu_shapes(cuda, T, d):
    _check(cuda, T, d)


@pytest.mark.parametrize("scale", [8.0, 40.0, 120.0])
def test_silu_wide_range(cuda, scale):
    _check(cuda, 6, 2048, scale=scale)


def test_silu_fp16(cuda):
    _check(cuda, 9, 1024, scale=3.0, dtype=torch.float16)


def test_silu_out_arg_and_batch_dims(cuda):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 3, 2 * 512, generator=g).to(torch.bfloat16)
    out = torch.empty(2, 3, 512, dtype=torch.bfloat16, device=cuda)
    ret = mas_b200.silu_and_mul(x.to(cuda), out=out)
    assert ret is out
    assert_ulp(out.cpu().view(6, 512), oracle.silu_and_mul(x.view(6, 1024)), what="batch dims")


def test_silu_empty(cuda):
    out = mas_b200.silu_and_mul(torch.empty(0, 64, dtype=torch.bfloat16, device=cuda))
    assert out.shape == (0, 32)


def test_silu_checks(cuda):
    with pytest.raises(ValueError):
        mas_b200.silu_and_mul(torch.empty(2, 6, dtype=torch.bfloat16, device=cuda))  # 12 B rows
    with pytest.raises(AssertionError):
        mas_b200.silu_and_mul(torch.empty(2, 16, dtype=torch.bfloat16, device=cuda),
                              out=torch.empty(2, 16, dtype=torch.bfloat16, device=cuda))


@pytest.mark.parametrize("d,in_stride,out_stride", [(13, 26, 13), (64, 132, 64), (64, 128, 72)])
def test_silu_c_abi_scalar_and_strided(cuda, d, in_stride, out_stride):
    """Odd d and unaligned strides reach the scalar kernel through the C ABI."""
    T = 7
    g = torch.Generator().manual_seed(9)
    buf = torch.randn(T, in_stride, generator=g).to(torch.bfloat16)
    xin = buf[:, : 2 * d]
    outd = torch.zeros(T, out_stride, dtype=torch.bfloat16, device=cuda)
    ind = buf.to(cuda)
    rc = mas_b200._lib.lib.mas_silu_and_mul(outd.data_ptr(), ind.data_ptr(), T, d, out_stride, in_stride, 0, 1,
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, mas_b200.status_string(rc)
    ref = oracle.silu_and_mul(xin.contiguous())
    assert_ulp(outd.cpu()[:, :d], ref, what="C ABI")
    assert torch.count_nonzero(outd.cpu()[:, d:]) == 0


def test_silu_config2_full(cuda):
    """Configuration 2: gate_up ~ N(0,1) bf16 [8192, 65536] -> [8192, 32768], seed 1."""
    x = workloads.silu_inputs(cuda)
    out = mas_b200.silu_and_mul(x)
    ref = oracle.silu_and_mul(x.cpu())
    assert_ulp(out.cpu(), ref, what="config 2")
