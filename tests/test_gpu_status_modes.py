"""Data errors are reported under every execution mode the reference uses.

The serving loop runs the model eagerly, traced by torch.compile(dynamic=True)
(miniagentserve/engine/model_runner.py:98) and replayed from CUDA graphs (model_runner.py:101-119).
aten's embedding raises on an id outside the table (devstral2.py:282); the kernels here zero the row
and set a bit in the library's per-device status word instead, which every launch reports into,
whichever mode issued it. These tests check the bit is set in all three modes, and that a clean step
leaves the word at zero.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
from mas_b200 import _lib

pytestmark = pytest.mark.gpu

V, H, D = 512, 256, 128


def _inputs(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    table = torch.randn(V, H, generator=g, device=cuda).to(torch.bfloat16)
    ids = torch.randint(0, V, (40,), generator=g, device=cuda)
    pos = torch.randint(0, 300, (40,), generator=g, device=cuda).to(torch.int32)
    q = torch.randn(40, 4 * D, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(40, 1 * D, generator=g, device=cuda).to(torch.bfloat16)
    ang = torch.rand(300, D // 2, generator=g, device=cuda) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    return table, ids, pos, q, k, cache


def _step(table, ids, pos, q, k, cache):
    mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, q, k, D, cache, is_neox=True)
    return mas_b200.embedding_gather(ids, table)


def test_status_set_in_eager_compiled_and_replayed_steps(cuda):
    table, ids, pos, q, k, cache = _inputs(cuda)
    mas_b200.read_status(cuda)  # clear
    _step(table, ids, pos, q, k, cache)
    assert mas_b200.read_status(cuda) == 0

    bad_ids = ids.clone()
    bad_ids[7] = V  # one past the table
    bad_pos = pos.clone()
    bad_pos[3] = 300  # one past the cache

    # eager
    out = _step(table, bad_ids, bad_pos, q, k, cache)
    torch.cuda.synchronize()
    assert mas_b200.read_status(cuda) == (_lib.STATUS_EMBED_ID_OUT_OF_RANGE | _lib.STATUS_ROPE_POS_OUT_OF_RANGE)
    assert torch.count_nonzero(out[7]) == 0

    # torch.compile(dynamic=True), as the model runner compiles the model
    compiled = torch.compile(_step, dynamic=True)
    compiled(table, ids, pos, q, k, cache)
    torch.cuda.synchronize()
    assert mas_b200.read_status(cuda) == 0
    out = compiled(table, bad_ids, bad_pos, q, k, cache)
    torch.cuda.synchronize()
    assert mas_b200.read_status(cuda) == (_lib.STATUS_EMBED_ID_OUT_OF_RANGE | _lib.STATUS_ROPE_POS_OUT_OF_RANGE)
    assert torch.count_nonzero(out[7]) == 0

    # CUDA-graph capture on a side stream, then replay with the bad inputs copied into the static ones
    s_ids, s_pos = ids.clone(), pos.clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        _step(table, s_ids, s_pos, q, k, cache)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    mas_b200.read_status(cuda)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        g_out = _step(table, s_ids, s_pos, q, k, cache)
    graph.replay()
    torch.cuda.synchronize()
    assert mas_b200.read_status(cuda) == 0
    s_ids.copy_(bad_ids)
    s_pos.copy_(bad_pos)
    graph.replay()
    torch.cuda.synchronize()
    assert mas_b200.read_status(cuda) == (_lib.STATUS_EMBED_ID_OUT_OF_RANGE | _lib.STATUS_ROPE_POS_OUT_OF_RANGE)
    assert torch.count_nonzero(g_out[7]) == 0
    del graph
    assert mas_b200.read_fault_word(cuda.index) == 0
