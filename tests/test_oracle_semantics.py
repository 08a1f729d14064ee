"""The C oracle against a second, independent restatement in torch on the CPU (small cases).

Two restatements of flashinfer's arithmetic written separately -- the C one (oracle/oracle.c, used as
the checker of the GPU kernels) and the torch one below (fp32 elementwise ops, each rounded; the
rope's one fused multiply-add evaluated exactly in float64) -- must agree: bit-exact for the gather
and the residual, <= 1 ulp for the rest (they differ only in how the sum of squares and exp are
accumulated). This guards the oracle's indexing:
strides, leading dimensions, neox vs interleaved pairs, partial rotary, int32/int64 indices.
"""
from __future__ import annotations

import pytest
import torch

import oracle
from parity import assert_bits_equal, assert_ulp


def torch_norm(x, r, w, eps, scale=None):
    h = x.float() + r.float()
    rstd = (1.0 / torch.sqrt(h.double().pow(2).mean(-1, keepdim=True) + eps)).float()
    y = h * rstd * w.float()
    if scale is not None:
        return (y * (1.0 / torch.tensor(scale, dtype=torch.float32))).clamp(-448, 448).to(torch.float8_e4m3fn), h.to(x.dtype)
    return y.to(x.dtype), h.to(x.dtype)


def torch_silu(x):
    d = x.shape[-1] // 2
    g, u = x[..., :d].float(), x[..., d:].float()
    e = torch.exp(-g.double()).float()
    den = 1.0 + e
    s = torch.where(den >= 2.0 ** 126, g * 0.0, g / den)  # the approximate divide's zero reciprocal
    return (s * u).to(x.dtype)


def torch_rope(pos, q, k, D, cache, neox=True):
    rd = cache.shape[1]
    half = rd // 2
    out = []
    for t in (q, k):
        v = t.view(t.shape[0], -1, D).float().clone()
        c = cache[pos.long()][:, None, :half]
        s = cache[pos.long()][:, None, half:]
        if neox:
            a, b = v[..., :half].clone(), v[..., half:rd].clone()
        else:
            a, b = v[..., 0:rd:2].clone(), v[..., 1:rd:2].clone()
        # one fused multiply-add after a rounded second product (evaluated exactly in float64)
        na = (a.double() * c.double() - (b * s).double()).float()
        nb = (b.double() * c.double() + (a * s).double()).float()
        if neox:
            v[..., :half], v[..., half:rd] = na, nb
        else:
            v[..., 0:rd:2], v[..., 1:rd:2] = na, nb
        out.append(v.to(t.dtype).view(t.shape))
    return out


@pytest.mark.parametrize("T,H,dtype", [(5, 64, torch.bfloat16), (3, 1000, torch.bfloat16), (4, 96, torch.float16)])
def test_norm(T, H, dtype):
    g = torch.Generator().manual_seed(T * H)
    x, r = torch.randn(T, H, generator=g).to(dtype), (torch.randn(T, H, generator=g) * 3).to(dtype)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(dtype)
    y_t, r_t = torch_norm(x, r, w, 1e-5)
    xo, ro = x.clone(), r.clone()
    oracle.fused_add_rmsnorm(xo, ro, w, 1e-5)
    assert_bits_equal(ro, r_t, "residual")
    assert_ulp(xo, y_t, what="norm")


def test_norm_strided_rows():
    g = torch.Generator().manual_seed(3)
    big_x, big_r = torch.randn(4, 300, generator=g).to(torch.bfloat16), torch.randn(4, 300, generator=g).to(torch.bfloat16)
    w = torch.randn(128, generator=g).to(torch.bfloat16)
    y_t, r_t = torch_norm(big_x[:, :128], big_r[:, :128], w, 1e-6)
    xo, ro = big_x.clone(), big_r.clone()
    oracle.fused_add_rmsnorm(xo[:, :128], ro[:, :128], w, 1e-6)
    assert_ulp(xo[:, :128], y_t, what="strided norm")
    assert_bits_equal(ro[:, :128], r_t, "strided residual")
    assert_bits_equal(xo[:, 128:], big_x[:, 128:], "outside the rows")


@pytest.mark.parametrize("scale", [0.5, 0.01])
def test_norm_quant(scale):
    g = torch.Generator().manual_seed(4)
    x, r = torch.randn(6, 256, generator=g).to(torch.bfloat16), torch.randn(6, 256, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16)
    y_t, r_t = torch_norm(x, r, w, 1e-5, scale=scale)
    out = torch.empty(6, 256, dtype=torch.float8_e4m3fn)
    xo, ro = x.clone(), r.clone()
    oracle.fused_add_rmsnorm_quant(out, xo, ro, w, scale, 1e-5)
    assert_bits_equal(xo, x, "input unchanged")
    assert_bits_equal(ro, r_t, "residual")
    assert_ulp(out, y_t, what="fp8")


@pytest.mark.parametrize("shape,scale", [((7, 64), 1.0), ((2, 3, 40), 5.0), ((4, 16), 100.0)])
def test_silu(shape, scale):
    x = (torch.randn(*shape, generator=torch.Generator().manual_seed(5)) * scale).to(torch.bfloat16)
    assert_ulp(oracle.silu_and_mul(x.reshape(-1, shape[-1])).view(*shape[:-1], shape[-1] // 2), torch_silu(x),
               what="silu")


@pytest.mark.parametrize("scale", [1e-3, 0.0137, 0.5, 400.0])
def test_silu_quant_is_quantize_fp8_of_silu(scale):
    """silu_and_mul_quant == quantize_fp8(silu_and_mul(x), scale) (devstral2.py:93-95) bit for bit,
    with the quotient in fp32 from the upcast activation; saturation and subnormal ranges included."""
    x = (torch.randn(9, 2 * 48, generator=torch.Generator().manual_seed(6)) * 4).to(torch.bfloat16)
    act = oracle.silu_and_mul(x)
    want = (act.float() / torch.tensor(scale, dtype=torch.float32)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    assert_bits_equal(oracle.silu_and_mul_quant(x, scale), want, f"scale {scale}")


def test_silu_quant_nan_and_strides():
    x = torch.randn(3, 2 * 16, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    x[1, 3] = float("nan")
    q = oracle.silu_and_mul_quant(x, 0.1)
    assert torch.isnan(q[1, 3].float()) and not torch.isnan(q[0].float()).any()
    out = torch.zeros(3, 24, dtype=torch.float8_e4m3fn)
    oracle.silu_and_mul_quant(x, 0.1, out=out[:, :16])
    assert_bits_equal(out[:, :16], q, "strided out")
    assert torch.count_nonzero(out[:, 16:].view(torch.uint8)) == 0


@pytest.mark.parametrize("D,rd,neox,pdt", [(128, 128, True, torch.int32), (128, 128, False, torch.int64),
                                           (64, 32, True, torch.int32), (40, 40, False, torch.int32)])
def test_rope(D, rd, neox, pdt):
    g = torch.Generator().manual_seed(D + rd)
    T, Hq, Hkv, P = 9, 3, 2, 50
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, rd // 2, generator=g) * 6.28
    cache = torch.cat([ang.cos(), ang.sin()], -1)
    pos = torch.randint(0, P, (T,), generator=g).to(pdt)
    q, k = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D]
    qt, kt = torch_rope(pos, q, k, D, cache, neox)
    qo = qkv.clone()
    st = oracle.apply_rope_with_cos_sin_cache_inplace(pos, qo[:, : Hq * D], qo[:, Hq * D: (Hq + Hkv) * D], D, cache,
                                                      is_neox=neox)
    assert st == 0
    assert_ulp(qo[:, : Hq * D], qt, what="q")
    assert_ulp(qo[:, Hq * D: (Hq + Hkv) * D], kt, what="k")
    assert_bits_equal(qo[:, (Hq + Hkv) * D:], qkv[:, (Hq + Hkv) * D:], "v untouched")


def test_rope_out_of_range_position_untouched():
    qkv = torch.randn(3, 3 * 64).to(torch.bfloat16)
    cache = torch.randn(10, 64)
    pos = torch.tensor([0, 10, -1], dtype=torch.int32)
    qo = qkv.clone()
    st = oracle.apply_rope_with_cos_sin_cache_inplace(pos, qo[:, :128], qo[:, 128:], 64, cache)
    assert st == 2
    assert_bits_equal(qo[1:], qkv[1:], "bad positions untouched")


def test_embedding_out_of_range_and_dtypes():
    table = torch.randn(20, 6)
    ids = torch.tensor([[3, 19], [0, 20]], dtype=torch.int64)
    out, st = oracle.embedding(ids, table)
    assert st == 1
    assert torch.equal(out[0, 0], table[3]) and torch.equal(out[0, 1], table[19]) and torch.equal(out[1, 0], table[0])
    assert torch.count_nonzero(out[1, 1]) == 0
    out32, st32 = oracle.embedding(ids[0].to(torch.int32), table.to(torch.bfloat16))
    assert st32 == 0 and torch.equal(out32, table.to(torch.bfloat16)[ids[0]])


@pytest.mark.parametrize("neox,orig,beta", [(True, 8192, 0.1), (False, 4096, 0.25), (True, 16384, 1.0)])
def test_rope_llama4_query_scale_matches_reference_expression(neox, orig, beta):
    """The fused rope + query scale against the reference's own torch expression (devstral2.py:175-179)
    applied to the rotated q; original_max is a power of two, so `/` and `* (1/x)` agree exactly."""
    g = torch.Generator().manual_seed(orig)
    T, Hq, Hkv, D, P = 11, 3, 2, 64, 200000
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g) * 6.28
    cache = torch.cat([ang.cos(), ang.sin()], -1)
    pos = torch.randint(0, P, (T,), generator=g).to(torch.int32)
    pos[0], pos[1], pos[2] = 0, orig - 1, orig  # scale 1, 1, 1 + beta*log(2)
    q, k = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + Hkv) * D]
    qt, kt = torch_rope(pos, q, k, D, cache, neox)
    attn_scale = 1 + beta * torch.log1p(torch.floor(pos.float() / orig))
    q_ref = qt.view(T, Hq, D) * attn_scale[:, None, None].to(torch.bfloat16)
    qo = qkv.clone()
    st = oracle.apply_rope_and_llama4_query_scale_inplace(pos, qo[:, : Hq * D], qo[:, Hq * D: (Hq + Hkv) * D], D,
                                                          cache, beta, orig, is_neox=neox)
    assert st == 0
    assert_ulp(qo[:, : Hq * D], q_ref.reshape(T, -1), what="scaled q")
    assert_ulp(qo[:, Hq * D: (Hq + Hkv) * D], kt, what="k (rotated only)")


def test_embedding_fill_placeholders_matches_reference_expression():
    """The oracle's fused fill + gather against ModelRunner.fill_placeholders' own torch expression
    (model_runner.py:149-154) followed by the embedding."""
    g = torch.Generator().manual_seed(9)
    V, H = 300, 24
    table = torch.randn(V, H, generator=g).to(torch.bfloat16)
    last_tokens = torch.randint(0, V, (5,), generator=g, dtype=torch.int32)
    ids = torch.tensor([7, -1, 299, -5, 0, -3, 12], dtype=torch.int64)
    ref_ids = ids.clone()
    rows = (-1 - ref_ids).clamp(min=0)
    ref_ids.copy_(torch.where(ref_ids < 0, last_tokens[rows], ref_ids))
    ref = table[ref_ids]
    mine_ids = ids.clone()
    out, st = oracle.embedding_fill_placeholders(mine_ids, table, last_tokens)
    assert st == 0
    assert torch.equal(mine_ids, ref_ids)
    assert_bits_equal(out, ref, "rows")
    bad = torch.tensor([-6, 3], dtype=torch.int64)  # row 5 of a 5-entry last_tokens
    out, st = oracle.embedding_fill_placeholders(bad, table, last_tokens)
    assert st == 1 and torch.count_nonzero(out[0].float()) == 0 and int(bad[0]) == -6


def _append_loop(k, v, bi, pos, k_cache, v_cache, kv_indices, kv_indptr, page_size, hnd=False):
    """flashinfer's append kernel (page.cuh:259-284) as a plain loop, no index checks."""
    for i in range(k.shape[0]):
        flat = int(kv_indptr[int(bi[i])]) * page_size + int(pos[i])
        page, entry = int(kv_indices[flat // page_size]), flat % page_size
        if hnd:
            k_cache[page, :, entry] = k[i]
            v_cache[page, :, entry] = v[i]
        else:
            k_cache[page, entry] = k[i]
            v_cache[page, entry] = v[i]


@pytest.mark.parametrize("hnd,pdt", [(False, torch.int32), (True, torch.int64)])
def test_append_paged_kv_matches_formula(hnd, pdt):
    from mas_b200 import workloads
    b = workloads.paged_batch(seed=11, page_size=16)
    T, H, D = b.positions.shape[0], 2, 64
    g = torch.Generator().manual_seed(12)
    qkv = torch.randn(T, (4 + 2 * H) * D, generator=g).to(torch.bfloat16)
    k = qkv[:, 4 * D: (4 + H) * D].view(T, H, D)
    v = qkv[:, (4 + H) * D:].view(T, H, D)
    shape = (b.num_pages, H, b.page_size, D) if hnd else (b.num_pages, b.page_size, H, D)
    kc, vc = torch.randn(shape, generator=g).to(torch.bfloat16), torch.randn(shape, generator=g).to(torch.bfloat16)
    kw, vw = kc.clone(), vc.clone()
    _append_loop(k, v, b.batch_indices, b.positions, kw, vw, b.kv_indices, b.kv_indptr, b.page_size, hnd)
    st = oracle.append_paged_kv_cache(k, v, b.batch_indices, b.positions.to(pdt), (kc, vc), b.kv_indices,
                                      b.kv_indptr, kv_layout="HND" if hnd else "NHD")
    assert st == 0
    assert_bits_equal(kc, kw, "k cache")
    assert_bits_equal(vc, vw, "v cache")


def test_append_paged_kv_out_of_range_slots_flagged():
    from mas_b200 import workloads
    b = workloads.paged_batch(seed=13, num_decodes=4, prompt_lens=(5,))
    T, H, D = b.positions.shape[0], 1, 16
    k = torch.randn(T, H, D).to(torch.bfloat16)
    v = torch.randn(T, H, D).to(torch.bfloat16)
    kc = torch.zeros(b.num_pages, b.page_size, H, D, dtype=torch.bfloat16)
    vc = kc.clone()
    bi = b.batch_indices.clone()
    pos = b.positions.clone()
    bi[0] = 99          # no such sequence
    pos[1] = -3         # negative position
    pos[2] = 10 ** 6    # past the page table
    table = b.block_tables.clone()
    table[int(bi[3]), int(pos[3]) // b.page_size] = b.num_pages + 7  # page id out of range
    st = oracle.append_paged_kv_cache(k, v, bi, pos, (kc, vc), table.flatten(), b.kv_indptr)
    assert st == 8
    kw, vw = torch.zeros_like(kc), torch.zeros_like(vc)
    keep = torch.arange(4, T)
    _append_loop(k[keep], v[keep], bi[keep], pos[keep], kw, vw, table.flatten(), b.kv_indptr, b.page_size)
    assert_bits_equal(kc, kw, "only in-range tokens appended")
    assert_bits_equal(vc, vw, "only in-range tokens appended")


def test_rope_append_is_rope_then_append_then_scale():
    """The fused oracle equals its parts run in the reference's order (devstral2.py:163-179)."""
    from mas_b200 import workloads
    b = workloads.paged_batch(seed=14, page_size=8)
    T, Hq, H, D, P = b.positions.shape[0], 4, 2, 64, 2048
    g = torch.Generator().manual_seed(15)
    qkv = torch.randn(T, (Hq + 2 * H) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    kc = torch.zeros(b.num_pages, b.page_size, H, D, dtype=torch.bfloat16)
    vc = kc.clone()
    a = qkv.clone()
    st = oracle.rope_append_paged_kv_cache(b.positions, a[:, : Hq * D], a[:, Hq * D: (Hq + H) * D],
                                           a[:, (Hq + H) * D:], D, cache, b.batch_indices, (kc, vc), b.kv_indices,
                                           b.kv_indptr, beta=0.1, original_max_position_embeddings=64)
    assert st == 0
    r = qkv.clone()
    oracle.apply_rope_with_cos_sin_cache_inplace(b.positions, r[:, : Hq * D], r[:, Hq * D: (Hq + H) * D], D, cache)
    kw, vw = torch.zeros_like(kc), torch.zeros_like(vc)
    oracle.append_paged_kv_cache(r[:, Hq * D: (Hq + H) * D].view(T, H, D), r[:, (Hq + H) * D:].view(T, H, D),
                                 b.batch_indices, b.positions, (kw, vw), b.kv_indices, b.kv_indptr)
    scale = (1 + 0.1 * torch.log1p(torch.floor(b.positions.float() * (1.0 / 64)))).to(torch.bfloat16)
    r[:, : Hq * D] = (r[:, : Hq * D].view(T, Hq, D) * scale[:, None, None]).view(T, -1)
    assert_bits_equal(a, r, "q scaled, k rotated, v untouched")
    assert_bits_equal(kc, kw, "k cache")
    assert_bits_equal(vc, vw, "v cache")
