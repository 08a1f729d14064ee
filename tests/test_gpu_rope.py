"""Parity of the rotary-embedding kernels against the oracle (<= 1 ulp), in place on q and k.

Covers q/k as strided views of one fused qkv row (as Devstral2Attention.forward passes them), the
v part and the non-rotary tail staying bit-identical, neox and interleaved pairing, head_dim 64/128/
256, partial rotary_dim, a rotary_dim off the vector path, int32 and int64 positions, positions at
0 and max_positions - 1, out-of-range positions (flagged, token untouched), no kv heads, empty
batches, and configuration 3 at full size.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_bits_equal, assert_ulp

pytestmark = pytest.mark.gpu


def _case(T, Hq, Hkv, D, rd, P, pos_dtype=torch.int32, seed=2):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, rd // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    pos = torch.randint(0, P, (T,), generator=g)
    if T:
        pos[0] = P - 1
        pos[-1] = 0
    return qkv, cache, pos.to(pos_dtype)


def _run(cuda, T, Hq, Hkv, D, rd, P, neox=True, pos_dtype=torch.int32):
    qkv, cache, pos = _case(T, Hq, Hkv, D, rd, P, pos_dtype)
    qd = qkv.to(cuda)
    mas_b200.apply_rope_with_cos_sin_cache_inplace(pos.to(cuda), qd[:, : Hq * D], qd[:, Hq * D: (Hq + Hkv) * D], D,
                                                   cache.to(cuda), is_neox=neox)
    qo = qkv.clone()
    st = oracle.apply_rope_with_cos_sin_cache_inplace(pos, qo[:, : Hq * D], qo[:, Hq * D: (Hq + Hkv) * D], D, cache,
                                                      is_neox=neox)
    assert st == 0
    got = qd.cpu()
    assert_bits_equal(got[:, (Hq + Hkv) * D:], qkv[:, (Hq + Hkv) * D:], "v untouched")
    if rd < D:
        heads = got[:, : (Hq + Hkv) * D].view(T, Hq + Hkv, D)
        assert_bits_equal(heads[..., rd:], qkv[:, : (Hq + Hkv) * D].view(T, Hq + Hkv, D)[..., rd:], "tail untouched")
    return assert_ulp(got, qo, what=f"rope T={T} Hq={Hq} Hkv={Hkv} D={D} rd={rd} neox={neox}")


@pytest.mark.parametrize("T,Hq,Hkv,D", [(16, 4, 2, 128), (1, 32, 8, 128), (37, 96, 8, 128), (9, 2, 2, 64),
                                        (5, 2, 1, 256), (300, 8, 8, 128)])
@pytest.mark.parametrize("neox", [True, False])
def test_rope_shapes(cuda, T, Hq, Hkv, D, neox):
    _run(cuda, T, Hq, Hkv, D, D, 64, neox=neox)


def test_rope_int64_positions(cuda):
    _run(cuda, 23, 4, 2, 128, 128, 4096, pos_dtype=torch.int64)


# rotary_dim 48, 96, 112: rotary_dim/16 does not divide the ring's consumer count, so its consumers
# walk the (head, pair group) list instead of keeping one pair group each
@pytest.mark.parametrize("D,rd", [(128, 64), (128, 32), (40, 40), (128, 72), (128, 48), (128, 96), (128, 112)])
def test_rope_partial_and_generic_rotary(cuda, D, rd):
    _run(cuda, 11, 3, 1, D, rd, 64)


@pytest.mark.parametrize("neox", [True, False])
def test_rope_padded_heads_vector_path(cuda, neox):
    """Heads that are not contiguous within a token (head stride 2*D) take the per-unit vector kernel
    instead of the token-staged ring; the padding between heads stays untouched."""
    T, Hq, Hkv, D, P = 13, 3, 2, 128, 64
    g = torch.Generator().manual_seed(21)
    qbuf = torch.randn(T, Hq, 2 * D, generator=g).to(torch.bfloat16)
    kbuf = torch.randn(T, Hkv, 2 * D, generator=g).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    pos = torch.randint(0, P, (T,), generator=g).to(torch.int32)
    qd, kd = qbuf.to(cuda), kbuf.to(cuda)
    pos_d, cache_d = pos.to(cuda), cache.to(cuda)  # kept alive until the kernel has run
    q, k = qd[..., :D], kd[..., :D]
    rc = mas_b200._lib.lib.mas_rope_cos_sin_cache_inplace(
        pos_d.data_ptr(), 4, q.data_ptr(), k.data_ptr(), cache_d.data_ptr(), T, Hq, Hkv, D, D, P,
        q.stride(0), q.stride(1), k.stride(0), k.stride(1), int(neox), 0, None, 1,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, mas_b200.status_string(rc)
    # the oracle takes (tokens, heads*D) views; feed it compact copies and compare the rotated parts
    qc, kc = qbuf[..., :D].contiguous().view(T, -1), kbuf[..., :D].contiguous().view(T, -1)
    oracle.apply_rope_with_cos_sin_cache_inplace(pos, qc, kc, D, cache, is_neox=neox)
    assert_ulp(qd[..., :D].cpu().contiguous().view(T, -1), qc, what="padded q")
    assert_ulp(kd[..., :D].cpu().contiguous().view(T, -1), kc, what="padded k")
    assert_bits_equal(qd[..., D:].cpu(), qbuf[..., D:], "q padding")
    assert_bits_equal(kd[..., D:].cpu(), kbuf[..., D:], "k padding")


def test_rope_out_of_range_positions_flagged(cuda):
    T, Hq, Hkv, D, P = 6, 2, 1, 128, 32
    qkv, cache, pos = _case(T, Hq, Hkv, D, D, P)
    pos[2] = P
    pos[4] = -1
    mas_b200.read_status(cuda)
    qd = qkv.to(cuda)
    mas_b200.apply_rope_with_cos_sin_cache_inplace(pos.to(cuda), qd[:, : Hq * D], qd[:, Hq * D: (Hq + Hkv) * D], D,
                                                   cache.to(cuda))
    st = mas_b200.read_status(cuda)
    assert st & mas_b200._lib.STATUS_ROPE_POS_OUT_OF_RANGE
    qo = qkv.clone()
    ost = oracle.apply_rope_with_cos_sin_cache_inplace(pos, qo[:, : Hq * D], qo[:, Hq * D: (Hq + Hkv) * D], D, cache)
    assert ost == 2
    assert_bits_equal(qd.cpu()[2], qkv[2], "bad token untouched")
    assert_bits_equal(qd.cpu()[4], qkv[4], "bad token untouched")
    assert_ulp(qd.cpu(), qo, what="other tokens")


def test_rope_no_kv_heads_and_empty(cuda):
    _run(cuda, 5, 4, 0, 128, 128, 64)
    q = torch.empty(0, 256, dtype=torch.bfloat16, device=cuda)
    mas_b200.apply_rope_with_cos_sin_cache_inplace(torch.empty(0, dtype=torch.int32, device=cuda), q, q[:, :128], 128,
                                                   torch.zeros(4, 128, device=cuda))


def test_rope_rejects_non_fp32_cache(cuda):
    q = torch.zeros(2, 128, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        mas_b200.apply_rope_with_cos_sin_cache_inplace(torch.zeros(2, dtype=torch.int32, device=cuda), q, q.clone(),
                                                       128, torch.zeros(4, 128, dtype=torch.bfloat16, device=cuda))


def test_rope_config3_full(cuda):
    """Configuration 3: 64 ragged sequences, theta 1e9 cache of 131072 positions, q [T,32,128], k [T,8,128]."""
    pos, q, k, cache = workloads.rope_inputs(cuda)
    qo, ko = q.cpu(), k.cpu()
    mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, q, k, 128, cache)
    oracle.apply_rope_with_cos_sin_cache_inplace(pos.cpu(), qo, ko, 128, cache.cpu())
    assert_ulp(q, qo, what="config 3 q")
    assert_ulp(k, ko, what="config 3 k")
