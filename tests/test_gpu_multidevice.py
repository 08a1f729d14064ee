"""Ops on a device other than the current one (skipped with fewer than two GPUs).

The serving engine runs one process per GPU, but nothing stops a caller from handing tensors on
cuda:1 while cuda:0 is current. Each operator guards the tensors' device, the library prepares each
device on first use, and the status word is per device: results must match the oracle and an
out-of-range id must be reported on the right device only.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_bits_equal, assert_ulp

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs"),
]


def test_every_op_on_the_second_device_while_the_first_is_current():
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 1)
    g = torch.Generator().manual_seed(77)
    # norm
    x = torch.randn(7, 5120, generator=g).to(torch.bfloat16)
    r = torch.randn(7, 5120, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(5120, generator=g)).to(torch.bfloat16)
    xd, rd = x.to(dev), r.to(dev)
    mas_b200.fused_add_rmsnorm(xd, rd, w.to(dev), 1e-5)
    oracle.fused_add_rmsnorm(x, r, w, 1e-5)
    assert_ulp(xd, x, what="norm on cuda:1")
    assert_bits_equal(rd, r, "residual on cuda:1")
    # silu, both forms
    gu = torch.randn(5, 2 * 4096, generator=g).to(torch.bfloat16)
    assert_ulp(mas_b200.silu_and_mul(gu.to(dev)), oracle.silu_and_mul(gu), what="silu on cuda:1")
    assert_ulp(mas_b200.silu_and_mul_quant(gu.to(dev), torch.tensor(0.02, device=dev)),
               oracle.silu_and_mul_quant(gu, 0.02), what="silu fp8 on cuda:1")
    # rope + paged append
    b = workloads.paged_batch(seed=78, num_decodes=3, prompt_lens=(11,), page_size=16, max_cached=100)
    T, Hq, Hkv, D = b.positions.shape[0], 4, 2, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(256, D // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    kc = torch.zeros(b.num_pages, 16, Hkv, D, dtype=torch.bfloat16)
    vc = kc.clone()
    bd, qkv_d, kc_d, vc_d = b.to(dev), qkv.to(dev), kc.to(dev), vc.to(dev)
    qs, ks = Hq * D, Hkv * D
    mas_b200.apply_rope_and_append_paged_kv_cache(bd.positions, qkv_d[:, :qs], qkv_d[:, qs: qs + ks], qkv_d[:, qs + ks:],
                                                  D, cache.to(dev), bd.batch_indices, (kc_d, vc_d), bd.kv_indices,
                                                  bd.kv_indptr, bd.kv_last_page_len)
    oracle.rope_append_paged_kv_cache(b.positions, qkv[:, :qs], qkv[:, qs: qs + ks], qkv[:, qs + ks:], D, cache,
                                      b.batch_indices, (kc, vc), b.kv_indices, b.kv_indptr)
    assert_ulp(qkv_d.cpu(), qkv, what="rope on cuda:1")
    assert_bits_equal(vc_d, vc, "v cache on cuda:1")
    # gather, with an out-of-range id reported on cuda:1 only
    table = torch.randn(100, 256, generator=g).to(torch.bfloat16)
    ids = torch.tensor([3, 99, 100, 0])
    mas_b200.read_status(0)
    mas_b200.read_status(1)
    got = mas_b200.embedding_gather(ids.to(dev), table.to(dev))
    want, st = oracle.embedding(ids, table)
    assert st == 1
    assert_bits_equal(got, want, "gather on cuda:1")
    assert mas_b200.read_status(1) & mas_b200._lib.STATUS_EMBED_ID_OUT_OF_RANGE
    assert mas_b200.read_status(0) == 0
    assert torch.cuda.current_device() == 0
