"""The gather fused with ModelRunner.fill_placeholders (model_runner.py:149-154) on the GPU.

Placeholders (-1 - r) are resolved from the previous step's samples, written back into input_ids, and
their rows gathered in one launch; results must equal the reference's own two steps (torch's
fill_placeholders expression, then the embedding) bit for bit, on the TMA path and the generic path,
with int64 and int32 ids and int32 samples as the runner keeps them.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from parity import assert_bits_equal

pytestmark = pytest.mark.gpu


def _reference(ids, table, last_tokens):
    ids = ids.clone()
    rows = (-1 - ids).clamp(min=0)
    ids.copy_(torch.where(ids < 0, last_tokens[rows], ids))
    return ids, torch.nn.functional.embedding(ids.long(), table)


@pytest.mark.parametrize("V,H,T,id_dtype", [(4096, 5120, 300, torch.int64), (1000, 12288, 64, torch.int64),
                                            (500, 7, 40, torch.int32), (2048, 128, 1, torch.int64)])
def test_fill_and_gather_matches_reference(cuda, V, H, T, id_dtype):
    g = torch.Generator().manual_seed(V + T)
    table = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    last_tokens = torch.randint(0, V, (17,), generator=g, dtype=torch.int32).to(cuda)
    ids = torch.randint(0, V, (T,), generator=g)
    place = torch.rand(T, generator=g) < 0.4
    ids = torch.where(place, -1 - torch.randint(0, 17, (T,), generator=g), ids).to(id_dtype).to(cuda)
    ref_ids, ref = _reference(ids, table, last_tokens)
    mine_ids = ids.clone()
    out = mas_b200.embedding_fill_placeholders(mine_ids, table, last_tokens)
    assert torch.equal(mine_ids, ref_ids)
    assert_bits_equal(out, ref, "rows")
    o, st = oracle.embedding_fill_placeholders(ids.cpu().clone(), table.cpu(), last_tokens.cpu())
    assert st == 0
    assert_bits_equal(out, o, "oracle")


def test_fill_out_of_range_placeholder(cuda):
    table = torch.randn(50, 64).to(torch.bfloat16).to(cuda)
    last = torch.tensor([3, 4], dtype=torch.int32, device=cuda)
    ids = torch.tensor([-1, -3, 5], dtype=torch.int64, device=cuda)
    mas_b200.read_status(cuda)
    out = mas_b200.embedding_fill_placeholders(ids, table, last)
    assert mas_b200.read_status(cuda) & mas_b200._lib.STATUS_EMBED_ID_OUT_OF_RANGE
    assert ids.tolist() == [3, -3, 5]
    assert torch.count_nonzero(out[1].float()) == 0
    assert torch.equal(out[0], table[3]) and torch.equal(out[2], table[5])
