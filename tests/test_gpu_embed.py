"""Bit-exact parity of the token-embedding gather with nn.Embedding's result (the oracle and aten).

Covers the TMA ring path (16-byte rows) and the generic path (odd row sizes, unaligned strides),
int32 and int64 ids, ids 0 and vocab-1, repeated ids, out-of-range ids (zero row, status bit),
fp32 tables, leading id dimensions, the Embedding module drop-in and configuration 4 at full size.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads
from parity import assert_bits_equal

pytestmark = pytest.mark.gpu


def _table(V, H, dtype=torch.bfloat16, seed=3):
    return (torch.randn(V, H, generator=torch.Generator().manual_seed(seed)) * 0.02).to(dtype)


@pytest.mark.parametrize("V,H,T", [(1000, 5120, 64), (512, 12288, 33), (300, 8, 100), (257, 7, 31), (64, 1000, 1),
                                   (4096, 2048, 3000)])
@pytest.mark.parametrize("id_dtype", [torch.int32, torch.int64])
def test_embed_shapes(cuda, V, H, T, id_dtype):
    table = _table(V, H)
    g = torch.Generator().manual_seed(T)
    ids = torch.randint(0, V, (T,), generator=g)
    ids[0] = V - 1
    if T > 1:
        ids[1] = 0
    ids = ids.to(id_dtype)
    out = mas_b200.embedding_gather(ids.to(cuda), table.to(cuda))
    assert_bits_equal(out.cpu(), torch.nn.functional.embedding(ids.long(), table), "gather")


def test_embed_out_of_range_ids(cuda):
    V, H = 100, 256
    table = _table(V, H)
    ids = torch.tensor([5, V, -1, 99, 0], dtype=torch.int64)
    mas_b200.read_status(cuda)
    out = mas_b200.embedding_gather(ids.to(cuda), table.to(cuda))
    assert mas_b200.read_status(cuda) & mas_b200._lib.STATUS_EMBED_ID_OUT_OF_RANGE
    ref, st = oracle.embedding(ids, table)
    assert st == 1
    assert_bits_equal(out.cpu(), ref, "gather with bad ids")
    assert torch.count_nonzero(out.cpu()[1:3].float()) == 0


def test_embed_fp32_table_and_batch_dims(cuda):
    table = torch.randn(50, 96)
    ids = torch.randint(0, 50, (3, 4))
    out = mas_b200.embedding_gather(ids.to(cuda), table.to(cuda))
    assert out.shape == (3, 4, 96)
    assert torch.equal(out.cpu(), table[ids])


def test_embed_strided_table_c_abi(cuda):
    """Row stride > hidden_size, aligned (TMA path) and unaligned (generic path)."""
    for stride in (1024, 1000 + 4):
        V, H, T = 64, 1000, 40
        big = _table(V, stride)
        ids = torch.randint(0, V, (T,), generator=torch.Generator().manual_seed(stride))
        out = torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
        bd, idd = big.to(cuda), ids.to(cuda)
        rc = mas_b200._lib.lib.mas_embedding_gather(out.data_ptr(), bd.data_ptr(), idd.data_ptr(), 5, T, H, V, H,
                                                    stride, 2, None, 1, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, mas_b200.status_string(rc)
        assert_bits_equal(out.cpu(), big[ids, :H], f"stride {stride}")


def test_embed_module_drop_in(cuda):
    emb = mas_b200.Embedding(1000, 64, device=cuda, dtype=torch.bfloat16)
    ref = torch.nn.Embedding(1000, 64, device=cuda, dtype=torch.bfloat16)
    ref.load_state_dict(emb.state_dict())
    ids = torch.randint(0, 1000, (77,), device=cuda)
    with torch.inference_mode():
        assert_bits_equal(emb(ids).cpu(), ref(ids).cpu(), "module")
    assert list(emb.state_dict()) == ["weight"]


def test_embed_empty(cuda):
    out = mas_b200.embedding_gather(torch.empty(0, dtype=torch.int64, device=cuda),
                                    torch.zeros(10, 16, dtype=torch.bfloat16, device=cuda))
    assert out.shape == (0, 16)


def test_embed_config4_full(cuda):
    """Configuration 4: table N(0, 0.02) bf16 [131072, 5120], int32 ids U[0, 131072), T = 16384."""
    table, ids = workloads.embed_inputs(cuda)
    out = mas_b200.embedding_gather(ids, table)
    ref, st = oracle.embedding(ids.cpu(), table.cpu())
    assert st == 0
    assert_bits_equal(out, ref, "config 4")
