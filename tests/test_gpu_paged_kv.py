"""Parity of the paged KV append, alone and fused with rope (and the llama-4 query scale).

The append is a byte copy: bit-exact against the oracle. Rotated q/k are <= 1 ulp against the
oracle, and the k rows written to the cache are bit-identical to the k rows written back in place.
Metadata is built the way ModelRunner / Devstral2Model.forward build it (decode rows first, then
prompt chunks; kv_indices = block_tables.flatten(), kv_indptr = arange(batch + 1) * max_blocks),
with NHD and HND caches, a 5-D combined cache, int32 and int64 positions, q/k/v as strided views of
one qkv row, padded heads (the unfused fallback), partial rotary, out-of-range slots and positions
(flagged, nothing written), empty batches, and fused == rope then append.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_bits_equal, assert_ulp

pytestmark = pytest.mark.gpu


def _setup(seed, Hq, H, D, page_size=16, hnd=False, rd=None, P=4096, num_decodes=8, prompt_lens=(37, 64)):
    b = workloads.paged_batch(seed=seed, num_decodes=num_decodes, prompt_lens=prompt_lens, page_size=page_size)
    T = b.positions.shape[0]
    g = torch.Generator().manual_seed(seed + 100)
    qkv = torch.randn(T, (Hq + 2 * H) * D, generator=g).to(torch.bfloat16)
    rd = D if rd is None else rd
    ang = torch.rand(P, rd // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    shape = (b.num_pages, H, page_size, D) if hnd else (b.num_pages, page_size, H, D)
    kc = torch.randn(shape, generator=g).to(torch.bfloat16)
    vc = torch.randn(shape, generator=g).to(torch.bfloat16)
    return b, qkv, cache, kc, vc


def _split(qkv, Hq, H, D):
    T = qkv.shape[0]
    return (qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + H) * D], qkv[:, (Hq + H) * D:].view(T, H, D))


@pytest.mark.parametrize("hnd,pdt,page_size", [(False, torch.int32, 16), (True, torch.int64, 16),
                                               (False, torch.int32, 64), (False, torch.int64, 1)])
def test_append_matches_oracle(cuda, hnd, pdt, page_size):
    Hq, H, D = 4, 8, 128
    b, qkv, _, kc, vc = _setup(21, Hq, H, D, page_size=page_size, hnd=hnd)
    T = qkv.shape[0]
    bd = b.to(cuda)
    qkv_d, kc_d, vc_d = qkv.to(cuda), kc.to(cuda), vc.to(cuda)
    _, k_d, v_d = _split(qkv_d, Hq, H, D)
    layout = "HND" if hnd else "NHD"
    mas_b200.read_status(cuda)
    mas_b200.append_paged_kv_cache(k_d.view(T, H, D), v_d, bd.batch_indices, bd.positions.to(pdt), (kc_d, vc_d),
                                   bd.kv_indices, bd.kv_indptr, bd.kv_last_page_len, kv_layout=layout)
    assert mas_b200.read_status(cuda) == 0
    _, k, v = _split(qkv, Hq, H, D)
    st = oracle.append_paged_kv_cache(k.view(T, H, D), v, b.batch_indices, b.positions.to(pdt), (kc, vc),
                                      b.kv_indices, b.kv_indptr, kv_layout=layout)
    assert st == 0
    assert_bits_equal(kc_d, kc, "k cache")
    assert_bits_equal(vc_d, vc, "v cache")
    assert_bits_equal(qkv_d, qkv, "qkv untouched")


def test_append_combined_5d_cache_and_scalar_path(cuda):
    """A (pages, 2, page_size, H, D) cache, and head_dim 36 (not a multiple of 8: scalar kernel)."""
    for D in (64, 36):
        Hq, H = 2, 2
        b, qkv, _, _, _ = _setup(22, Hq, H, D, page_size=8)
        T = qkv.shape[0]
        kv = torch.randn(b.num_pages, 2, b.page_size, H, D, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
        bd = b.to(cuda)
        qkv_d, kv_d = qkv.to(cuda), kv.to(cuda)
        _, k_d, v_d = _split(qkv_d, Hq, H, D)
        mas_b200.append_paged_kv_cache(k_d.view(T, H, D), v_d, bd.batch_indices, bd.positions, kv_d, bd.kv_indices,
                                       bd.kv_indptr, bd.kv_last_page_len)
        _, k, v = _split(qkv, Hq, H, D)
        oracle.append_paged_kv_cache(k.view(T, H, D), v, b.batch_indices, b.positions, (kv[:, 0], kv[:, 1]),
                                     b.kv_indices, b.kv_indptr)
        assert_bits_equal(kv_d, kv, f"5-D cache D={D}")


def test_append_out_of_range_flagged_not_written(cuda):
    Hq, H, D = 2, 2, 64
    b, qkv, _, kc, vc = _setup(23, Hq, H, D, num_decodes=6, prompt_lens=(9,))
    T = qkv.shape[0]
    bi, pos, table = b.batch_indices.clone(), b.positions.clone(), b.block_tables.clone()
    bi[0] = 77
    pos[1] = -1
    pos[2] = 1 << 24
    table[int(bi[3]), int(pos[3]) // b.page_size] = b.num_pages + 3
    kc_d, vc_d, qkv_d = kc.to(cuda), vc.to(cuda), qkv.to(cuda)
    _, k_d, v_d = _split(qkv_d, Hq, H, D)
    mas_b200.read_status(cuda)
    mas_b200.append_paged_kv_cache(k_d.view(T, H, D), v_d, bi.to(cuda), pos.to(cuda), (kc_d, vc_d),
                                   table.flatten().to(cuda), b.kv_indptr.to(cuda), b.kv_last_page_len.to(cuda))
    assert mas_b200.read_status(cuda) & mas_b200._lib.STATUS_KV_SLOT_OUT_OF_RANGE
    _, k, v = _split(qkv, Hq, H, D)
    st = oracle.append_paged_kv_cache(k.view(T, H, D), v, bi, pos, (kc, vc), table.flatten(), b.kv_indptr)
    assert st == 8
    assert_bits_equal(kc_d, kc, "k cache")
    assert_bits_equal(vc_d, vc, "v cache")


def _fused(cuda, seed, Hq, H, D, rd=None, hnd=False, beta=0.0, orig=8192, pdt=torch.int32, neox=True,
           page_size=16):
    b, qkv, cache, kc, vc = _setup(seed, Hq, H, D, page_size=page_size, hnd=hnd, rd=rd)
    T = qkv.shape[0]
    layout = "HND" if hnd else "NHD"
    bd = b.to(cuda)
    qkv_d, kc_d, vc_d, cache_d = qkv.to(cuda), kc.to(cuda), vc.to(cuda), cache.to(cuda)
    q_d, k_d, v_d = _split(qkv_d, Hq, H, D)
    mas_b200.read_status(cuda)
    mas_b200.apply_rope_and_append_paged_kv_cache(
        bd.positions.to(pdt), q_d, k_d, v_d, D, cache_d, bd.batch_indices, (kc_d, vc_d), bd.kv_indices, bd.kv_indptr,
        bd.kv_last_page_len, is_neox=neox, kv_layout=layout, llama_4_scaling_beta=beta,
        original_max_position_embeddings=orig)
    assert mas_b200.read_status(cuda) == 0
    q, k, v = _split(qkv, Hq, H, D)
    st = oracle.rope_append_paged_kv_cache(b.positions.to(pdt), q, k, v, D, cache, b.batch_indices, (kc, vc),
                                           b.kv_indices, b.kv_indptr, is_neox=neox, kv_layout=layout, beta=beta,
                                           original_max_position_embeddings=orig)
    assert st == 0
    got = qkv_d.cpu()
    assert_ulp(got, qkv, what=f"q/k (seed {seed})")
    assert_bits_equal(got[:, (Hq + H) * D:], qkv[:, (Hq + H) * D:], "v untouched")
    assert_bits_equal(vc_d, vc, "v cache")
    assert_ulp(kc_d.cpu(), kc, what="k cache vs oracle")
    # the cache holds exactly the k rows written back in place
    k_rows = got[:, Hq * D: (Hq + H) * D].view(T, H, D)
    kw = kc_d.cpu().clone()
    oracle.append_paged_kv_cache(k_rows, v, b.batch_indices, b.positions, (kw, vc.clone()), b.kv_indices,
                                 b.kv_indptr, kv_layout=layout)
    assert_bits_equal(kc_d, kw, "cache k == in-place k")
    return b, qkv_d, kc_d, vc_d


@pytest.mark.parametrize("Hq,H,D", [(4, 2, 128), (32, 8, 128), (96, 8, 128), (8, 8, 64), (4, 1, 256)])
def test_rope_append_matches_oracle(cuda, Hq, H, D):
    _fused(cuda, 31, Hq, H, D)


@pytest.mark.parametrize("hnd,pdt,neox", [(True, torch.int32, True), (False, torch.int64, False)])
def test_rope_append_layouts(cuda, hnd, pdt, neox):
    _fused(cuda, 32, 8, 2, 128, hnd=hnd, pdt=pdt, neox=neox)


def test_rope_append_llama4_scale(cuda):
    _fused(cuda, 33, 8, 2, 128, beta=0.1, orig=64)


@pytest.mark.parametrize("rd", [64, 32, 96])  # 96: consumers walk the (head, pair group) list
def test_rope_append_partial_rotary_with_scale(cuda, rd):
    """The k tail past rotary_dim goes to the cache unrotated; q's tail is scaled by the tail launch."""
    _fused(cuda, 34, 4, 2, 128, rd=rd, beta=0.2, orig=128)


def test_rope_append_equals_unfused_sequence(cuda):
    Hq, H, D = 32, 8, 128
    b, qkv, cache, kc, vc = _setup(35, Hq, H, D)
    T = qkv.shape[0]
    bd = b.to(cuda)
    cache_d = cache.to(cuda)
    a_qkv, a_kc, a_vc = qkv.to(cuda), kc.to(cuda), vc.to(cuda)
    q, k, v = _split(a_qkv, Hq, H, D)
    mas_b200.apply_rope_and_append_paged_kv_cache(bd.positions, q, k, v, D, cache_d, bd.batch_indices, (a_kc, a_vc),
                                                  bd.kv_indices, bd.kv_indptr, bd.kv_last_page_len,
                                                  llama_4_scaling_beta=0.1, original_max_position_embeddings=256)
    u_qkv, u_kc, u_vc = qkv.to(cuda), kc.to(cuda), vc.to(cuda)
    q, k, v = _split(u_qkv, Hq, H, D)
    mas_b200.apply_rope_with_cos_sin_cache_inplace(bd.positions, q, k, D, cache_d)
    mas_b200.append_paged_kv_cache(k.view(T, H, D), v, bd.batch_indices, bd.positions, (u_kc, u_vc), bd.kv_indices,
                                   bd.kv_indptr, bd.kv_last_page_len)
    scale = (1 + 0.1 * torch.log1p(torch.floor(bd.positions.float() / 256))).to(torch.bfloat16)
    q.view(T, Hq, D).mul_(scale[:, None, None])
    assert_bits_equal(a_qkv, u_qkv, "qkv")
    assert_bits_equal(a_kc, u_kc, "k cache")
    assert_bits_equal(a_vc, u_vc, "v cache")


def test_rope_append_padded_heads_fallback(cuda):
    """k/v heads with a head stride of 2*D: the fused ring does not apply; rope then append run."""
    Hq, H, D, P = 2, 2, 128, 256
    b = workloads.paged_batch(seed=36, num_decodes=5, prompt_lens=(7,), page_size=16, max_cached=200)
    T = b.positions.shape[0]
    g = torch.Generator().manual_seed(37)
    qbuf = torch.randn(T, Hq, 2 * D, generator=g).to(torch.bfloat16)
    kbuf = torch.randn(T, H, 2 * D, generator=g).to(torch.bfloat16)
    vbuf = torch.randn(T, H, 2 * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    kc = torch.zeros(b.num_pages, b.page_size, H, D, dtype=torch.bfloat16)
    vc = kc.clone()
    bd = b.to(cuda)
    qd, kd, vd, kcd, vcd, cd = qbuf.to(cuda), kbuf.to(cuda), vbuf.to(cuda), kc.to(cuda), vc.to(cuda), cache.to(cuda)
    mas_b200.apply_rope_and_append_paged_kv_cache(bd.positions, qd[..., :D], kd[..., :D], vd[..., :D], D, cd,
                                                  bd.batch_indices, (kcd, vcd), bd.kv_indices, bd.kv_indptr,
                                                  bd.kv_last_page_len)
    qo, ko, vo = qbuf[..., :D].contiguous(), kbuf[..., :D].contiguous(), vbuf[..., :D].contiguous()
    oracle.rope_append_paged_kv_cache(b.positions, qo, ko, vo, D, cache, b.batch_indices, (kc, vc), b.kv_indices,
                                      b.kv_indptr)
    assert_ulp(qd[..., :D].cpu(), qo, what="padded q")
    assert_ulp(kd[..., :D].cpu(), ko, what="padded k")
    assert_ulp(kcd.cpu(), kc, what="k cache")
    assert_bits_equal(vcd, vc, "v cache")
    assert_bits_equal(kd[..., D:], kbuf[..., D:], "k padding")


def test_rope_append_out_of_range_position_neither_rotated_nor_appended(cuda):
    Hq, H, D, P = 2, 1, 128, 512
    b = workloads.paged_batch(seed=38, num_decodes=4, prompt_lens=(6,), page_size=16, max_cached=400)
    T = b.positions.shape[0]
    g = torch.Generator().manual_seed(39)
    qkv = torch.randn(T, (Hq + 2 * H) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    pos = b.positions.clone()
    pos[0] = P + 5  # beyond the cos/sin cache, but a valid cache slot
    kc = torch.zeros(b.num_pages, b.page_size, H, D, dtype=torch.bfloat16)
    vc = kc.clone()
    bd = b.to(cuda)
    qkv_d, kcd, vcd = qkv.to(cuda), kc.to(cuda), vc.to(cuda)
    q, k, v = _split(qkv_d, Hq, H, D)
    mas_b200.read_status(cuda)
    mas_b200.apply_rope_and_append_paged_kv_cache(pos.to(cuda), q, k, v, D, cache.to(cuda), bd.batch_indices,
                                                  (kcd, vcd), bd.kv_indices, bd.kv_indptr, bd.kv_last_page_len)
    assert mas_b200.read_status(cuda) == mas_b200._lib.STATUS_ROPE_POS_OUT_OF_RANGE
    q, k, v = _split(qkv, Hq, H, D)
    st = oracle.rope_append_paged_kv_cache(pos, q, k, v, D, cache, b.batch_indices, (kc, vc), b.kv_indices,
                                           b.kv_indptr)
    assert st == 2
    assert_bits_equal(qkv_d.cpu()[0], qkv[0], "token 0 untouched")
    assert_ulp(qkv_d.cpu(), qkv, what="qkv")
    assert_bits_equal(vcd, vc, "v cache")
    assert_ulp(kcd.cpu(), kc, what="k cache")


def test_paged_empty_batches(cuda):
    H, D = 2, 64
    kc = torch.zeros(4, 16, H, D, dtype=torch.bfloat16, device=cuda)
    z32 = torch.zeros(0, dtype=torch.int32, device=cuda)
    indptr = torch.zeros(2, dtype=torch.int32, device=cuda)
    last = torch.ones(1, dtype=torch.int32, device=cuda)
    e = torch.empty(0, H, D, dtype=torch.bfloat16, device=cuda)
    mas_b200.append_paged_kv_cache(e, e, z32, z32, (kc, kc.clone()), z32, indptr, last)
    q = torch.empty(0, 4 * D, dtype=torch.bfloat16, device=cuda)
    mas_b200.apply_rope_and_append_paged_kv_cache(z32, q, q[:, : H * D], e, D, torch.zeros(8, D, device=cuda), z32,
                                                  (kc, kc.clone()), z32, indptr, last)
    assert int(kc.abs().sum()) == 0


def test_append_and_fused_fp16(cuda):
    """fp16 k/v/cache (the kv_cache_dtype override of model_config.py:57-66 keeps the model dtype)."""
    Hq, H, D = 4, 2, 128
    b, qkv, cache, kc, vc = _setup(51, Hq, H, D)
    qkv, kc, vc = qkv.to(torch.float16), kc.to(torch.float16), vc.to(torch.float16)
    T = qkv.shape[0]
    bd = b.to(cuda)
    qkv_d, kc_d, vc_d = qkv.to(cuda), kc.to(cuda), vc.to(cuda)
    q_d, k_d, v_d = _split(qkv_d, Hq, H, D)
    mas_b200.apply_rope_and_append_paged_kv_cache(bd.positions, q_d, k_d, v_d, D, cache.to(cuda), bd.batch_indices,
                                                  (kc_d, vc_d), bd.kv_indices, bd.kv_indptr, bd.kv_last_page_len)
    q, k, v = _split(qkv, Hq, H, D)
    oracle.rope_append_paged_kv_cache(b.positions, q, k, v, D, cache, b.batch_indices, (kc, vc), b.kv_indices,
                                      b.kv_indptr)
    assert_ulp(qkv_d.cpu(), qkv, what="fp16 q/k")
    assert_ulp(kc_d.cpu(), kc, what="fp16 k cache")
    assert_bits_equal(vc_d, vc, "fp16 v cache")
    # and the standalone append of the (now rotated) k rows
    kc2, vc2 = torch.zeros_like(kc_d), torch.zeros_like(vc_d)
    mas_b200.append_paged_kv_cache(k_d.view(T, H, D), v_d, bd.batch_indices, bd.positions, (kc2, vc2), bd.kv_indices,
                                   bd.kv_indptr, bd.kv_last_page_len)
    kw, vw = torch.zeros_like(kc), torch.zeros_like(vc)
    oracle.append_paged_kv_cache(k_d.cpu().view(T, H, D), v_d.cpu(), b.batch_indices, b.positions, (kw, vw),
                                 b.kv_indices, b.kv_indptr)
    assert_bits_equal(kc2, kw, "fp16 append k")
    assert_bits_equal(vc2, vw, "fp16 append v")


def test_rope_append_hnd_partial_rotary_interleaved(cuda):
    _fused(cuda, 52, 8, 2, 128, rd=64, hnd=True, neox=False, beta=0.05, orig=512)
