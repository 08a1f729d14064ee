"""Seeded random shapes, strides and dtypes for every op, each against the oracle.

The hand-picked cases elsewhere cover the named configurations and edges; these draw 12 cases per
op from wide ranges (rows 1..300, widths from 8 to 16k elements including odd ones, row padding,
bf16 and fp16, int32 and int64 indices) so that each kernel's path selection, vector width and
tail handling meet shapes nobody picked. Same bars: bit-exact for copies and the residual,
<= 1 ulp (or one e4m3 step) elsewhere.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_bits_equal, assert_ulp

pytestmark = pytest.mark.gpu

CASES = range(12)


def _rng(op: str, i: int) -> torch.Generator:
    return torch.Generator().manual_seed(1000 * sum(map(ord, op)) + i)  # str hash() varies per process


def _pick(g, choices):
    return choices[int(torch.randint(0, len(choices), (1,), generator=g))]


@pytest.mark.parametrize("i", CASES)
def test_random_norm(cuda, i):
    g = _rng("norm", i)
    T = int(torch.randint(1, 300, (1,), generator=g))
    H = _pick(g, [8, 64, 1000, 1024, 2048, 4000, 5120, 6144, 8192, 12288, 16384, 24])
    pad = _pick(g, [0, 0, 8, 24])
    dtype = _pick(g, [torch.bfloat16, torch.float16])
    quant = bool(torch.randint(0, 2, (1,), generator=g))
    x = torch.randn(T, H + pad, generator=g).to(dtype)
    r = (2 * torch.randn(T, H + pad, generator=g)).to(dtype)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(dtype)
    xd, rd = x.to(cuda), r.to(cuda)
    xo, ro = x.clone(), r.clone()
    if quant:
        out = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=cuda)
        mas_b200.fused_add_rmsnorm_quant(out, xd[:, :H], rd[:, :H], w.to(cuda), torch.tensor([0.03], device=cuda),
                                         1e-5)
        ref = torch.empty(T, H, dtype=torch.float8_e4m3fn)
        oracle.fused_add_rmsnorm_quant(ref, xo[:, :H], ro[:, :H], w, 0.03, 1e-5)
        assert_ulp(out, ref, what=f"norm fp8 T={T} H={H}")
        assert_bits_equal(xd, x, "input untouched")
    else:
        mas_b200.fused_add_rmsnorm(xd[:, :H], rd[:, :H], w.to(cuda), 1e-5)
        oracle.fused_add_rmsnorm(xo[:, :H], ro[:, :H], w, 1e-5)
        assert_ulp(xd, xo, what=f"norm T={T} H={H} pad={pad} {dtype}")
    assert_bits_equal(rd, ro, f"residual T={T} H={H}")


@pytest.mark.parametrize("i", CASES)
def test_random_silu(cuda, i):
    g = _rng("silu", i)
    T = int(torch.randint(1, 300, (1,), generator=g))
    d = _pick(g, [8, 16, 104, 1000, 2048, 4096, 11008, 14336, 28672])
    dtype = _pick(g, [torch.bfloat16, torch.float16])
    quant = bool(torch.randint(0, 2, (1,), generator=g))
    scale = float(torch.rand(1, generator=g)) * 4 + 0.5
    x = (scale * torch.randn(T, 2 * d, generator=g)).to(dtype)
    if quant:
        s = float(torch.rand(1, generator=g)) * 0.1 + 1e-3
        got = mas_b200.silu_and_mul_quant(x.to(cuda), torch.tensor(s, device=cuda))
        assert_ulp(got, oracle.silu_and_mul_quant(x, s), what=f"silu fp8 T={T} d={d}")
    else:
        assert_ulp(mas_b200.silu_and_mul(x.to(cuda)), oracle.silu_and_mul(x), what=f"silu T={T} d={d} {dtype}")


@pytest.mark.parametrize("i", CASES)
def test_random_rope_and_append(cuda, i):
    g = _rng("rope", i)
    Hq = _pick(g, [1, 4, 8, 32, 96])
    Hkv = _pick(g, [1, 2, 8])
    D = _pick(g, [64, 128, 256])
    rd = _pick(g, [D, D, D // 2])
    neox = bool(torch.randint(0, 2, (1,), generator=g))
    pdt = _pick(g, [torch.int32, torch.int64])
    page = _pick(g, [1, 8, 16, 64])
    b = workloads.paged_batch(seed=int(torch.randint(0, 1 << 20, (1,), generator=g)),
                              num_decodes=int(torch.randint(0, 9, (1,), generator=g)),
                              prompt_lens=(int(torch.randint(1, 90, (1,), generator=g)),), page_size=page,
                              max_cached=200)
    T = b.positions.shape[0]
    P = 512
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, rd // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    kc = torch.randn(b.num_pages, page, Hkv, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(b.num_pages, page, Hkv, D, generator=g).to(torch.bfloat16)
    beta = _pick(g, [0.0, 0.1])
    bd = b.to(cuda)
    qkv_d, kc_d, vc_d = qkv.to(cuda), kc.to(cuda), vc.to(cuda)
    qs, ks = Hq * D, Hkv * D
    mas_b200.apply_rope_and_append_paged_kv_cache(
        bd.positions.to(pdt), qkv_d[:, :qs], qkv_d[:, qs: qs + ks], qkv_d[:, qs + ks:], D, cache.to(cuda),
        bd.batch_indices, (kc_d, vc_d), bd.kv_indices, bd.kv_indptr, bd.kv_last_page_len, is_neox=neox,
        llama_4_scaling_beta=beta, original_max_position_embeddings=64)
    st = oracle.rope_append_paged_kv_cache(b.positions.to(pdt), qkv[:, :qs], qkv[:, qs: qs + ks], qkv[:, qs + ks:], D,
                                           cache, b.batch_indices, (kc, vc), b.kv_indices, b.kv_indptr, is_neox=neox,
                                           beta=beta, original_max_position_embeddings=64)
    assert st == 0
    what = f"Hq={Hq} Hkv={Hkv} D={D} rd={rd} neox={neox} page={page} beta={beta}"
    assert_ulp(qkv_d.cpu(), qkv, what="qkv " + what)
    assert_ulp(kc_d.cpu(), kc, what="k cache " + what)
    assert_bits_equal(vc_d, vc, "v cache " + what)


@pytest.mark.parametrize("i", CASES)
def test_random_gather(cuda, i):
    g = _rng("gather", i)
    V = int(torch.randint(1, 5000, (1,), generator=g))
    H = _pick(g, [1, 3, 8, 100, 256, 5120, 12288])
    T = int(torch.randint(0, 400, (1,), generator=g))
    dtype = _pick(g, [torch.bfloat16, torch.float16, torch.float32])
    idt = _pick(g, [torch.int32, torch.int64])
    table = torch.randn(V, H, generator=g).to(dtype)
    ids = torch.randint(0, V, (T,), generator=g).to(idt)
    got = mas_b200.embedding_gather(ids.to(cuda), table.to(cuda))
    want, st = oracle.embedding(ids, table)
    assert st == 0
    assert_bits_equal(got, want, f"gather V={V} H={H} T={T} {dtype} {idt}")
