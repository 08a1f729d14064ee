"""Rope fused with Devstral 2's llama-4 query scale (devstral2.py:163-166 + :175-179) on the GPU.

The fused op must equal the oracle, and -- where flashinfer is importable -- the reference's own
two-step sequence run on the same GPU: flashinfer's apply_rope_with_cos_sin_cache_inplace, then
`q * (1 + beta * log1p(floor(pos.float() / original_max))).to(q.dtype)` in eager torch. Covers the
ring and vector paths, neox and interleaved pairing, partial rotary (the tail of q is scaled too),
int32/int64 positions, non-power-of-two original_max, and out-of-range positions.
"""
from __future__ import annotations

import importlib.util

import pytest
import torch

import mas_b200
import oracle
from parity import assert_bits_equal, assert_ulp

pytestmark = pytest.mark.gpu


def _inputs(T, Hq, Hkv, D, rd, P, seed, pdt=torch.int32):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, rd // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    pos = torch.randint(0, P, (T,), generator=g)
    pos[0] = P - 1
    return qkv, cache, pos.to(pdt)


@pytest.mark.parametrize("T,Hq,Hkv,D,rd,neox,orig,pdt", [
    (64, 32, 8, 128, 128, True, 8192, torch.int32),
    (37, 96, 8, 128, 128, True, 16384, torch.int64),
    (20, 4, 2, 128, 128, False, 4096, torch.int32),
    (15, 4, 2, 128, 64, True, 8192, torch.int32),
    (9, 3, 1, 128, 128, True, 3000, torch.int32),
])
def test_fused_rope_q_scale_matches_oracle(cuda, T, Hq, Hkv, D, rd, neox, orig, pdt):
    P, beta = 131072, 0.1
    qkv, cache, pos = _inputs(T, Hq, Hkv, D, rd, P, seed=T + rd, pdt=pdt)
    qd, pos_d, cache_d = qkv.to(cuda), pos.to(cuda), cache.to(cuda)
    mas_b200.apply_rope_and_llama4_query_scale_inplace(pos_d, qd[:, : Hq * D], qd[:, Hq * D: (Hq + Hkv) * D], D,
                                                       cache_d, beta, orig, is_neox=neox)
    qo = qkv.clone()
    st = oracle.apply_rope_and_llama4_query_scale_inplace(pos, qo[:, : Hq * D], qo[:, Hq * D: (Hq + Hkv) * D], D, cache,
                                                          beta, orig, is_neox=neox)
    assert st == 0
    got = qd.cpu()
    assert_bits_equal(got[:, (Hq + Hkv) * D:], qkv[:, (Hq + Hkv) * D:], "v untouched")
    assert_ulp(got, qo, what="fused rope + q scale")


def test_fused_rope_q_scale_vector_path(cuda):
    """Padded heads (head stride 2*D) take the per-unit vector kernel."""
    T, Hq, Hkv, D, P = 13, 3, 2, 128, 64
    g = torch.Generator().manual_seed(5)
    qbuf = torch.randn(T, Hq, 2 * D, generator=g).to(torch.bfloat16)
    kbuf = torch.randn(T, Hkv, 2 * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    pos = torch.randint(0, P, (T,), generator=g).to(torch.int32)
    qd, kd, pos_d, cache_d = qbuf.to(cuda), kbuf.to(cuda), pos.to(cuda), cache.to(cuda)
    q, k = qd[..., :D], kd[..., :D]
    rc = mas_b200._lib.lib.mas_rope_cos_sin_cache_q_scale_inplace(
        pos_d.data_ptr(), 4, q.data_ptr(), k.data_ptr(), cache_d.data_ptr(), T, Hq, Hkv, D, D, P,
        q.stride(0), q.stride(1), k.stride(0), k.stride(1), 1, 0.5, 16, 0, None, 1,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, mas_b200.status_string(rc)
    qc, kc = qbuf[..., :D].contiguous().view(T, -1), kbuf[..., :D].contiguous().view(T, -1)
    oracle.apply_rope_and_llama4_query_scale_inplace(pos, qc, kc, D, cache, 0.5, 16)
    assert_ulp(qd[..., :D].cpu().contiguous().view(T, -1), qc, what="padded q")
    assert_ulp(kd[..., :D].cpu().contiguous().view(T, -1), kc, what="padded k")


def test_fused_rope_q_scale_rejects_bad_original_max(cuda):
    q = torch.zeros(2, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        mas_b200.apply_rope_and_llama4_query_scale_inplace(torch.zeros(2, dtype=torch.int32, device=cuda), q,
                                                           q.clone(), 128, torch.zeros(4, 128, device=cuda), 0.1, 0)


@pytest.mark.skipif(importlib.util.find_spec("flashinfer") is None, reason="flashinfer not installed")
@pytest.mark.parametrize("orig", [8192, 3000])
def test_fused_rope_q_scale_matches_reference_sequence(cuda, orig):
    """Bit-exact against the reference's own two steps on this GPU (flashinfer rope, eager torch scale)."""
    from flashinfer.rope import apply_rope_with_cos_sin_cache_inplace as fi_rope

    T, Hq, Hkv, D, P, beta = 96, 32, 8, 128, 131072, 0.1
    qkv, cache, pos = _inputs(T, Hq, Hkv, D, D, P, seed=orig)
    cache_d, pos_d = cache.to(cuda), pos.to(cuda)
    ref = qkv.to(cuda)
    q, k = ref[:, : Hq * D], ref[:, Hq * D: (Hq + Hkv) * D]
    fi_rope(pos_d, q, k, D, cache_d, is_neox=True)
    attn_scale = 1 + beta * torch.log1p(torch.floor(pos_d.float() / orig))
    q_ref = q.unflatten(-1, (-1, D)) * attn_scale[:, None, None].to(q.dtype)
    mine = qkv.to(cuda)
    mas_b200.apply_rope_and_llama4_query_scale_inplace(pos_d, mine[:, : Hq * D], mine[:, Hq * D: (Hq + Hkv) * D], D,
                                                       cache_d, beta, orig)
    assert_bits_equal(mine[:, : Hq * D].cpu(), q_ref.flatten(1).cpu(), "q vs reference sequence")
    assert_bits_equal(mine[:, Hq * D: (Hq + Hkv) * D].cpu(), k.cpu(), "k vs flashinfer")
