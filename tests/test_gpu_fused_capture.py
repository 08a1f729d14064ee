"""The fused next-row operators under the reference's two execution modes: CUDA-graph capture and
replay (model_runner.py:101-119) and torch.compile(dynamic=True) (model_runner.py:98). Each must
give bit-identical results to eager execution, with every scale and index read on the device.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
from mas_b200 import workloads
from parity import assert_bits_equal

pytestmark = pytest.mark.gpu

Hq, H, D, P = 8, 2, 128, 2048


def _inputs(cuda, seed=41):
    b = workloads.paged_batch(seed=seed, num_decodes=5, prompt_lens=(24, 9), page_size=16, max_cached=400).to(cuda)
    T = b.positions.shape[0]
    g = torch.Generator(device=cuda).manual_seed(seed)
    qkv = torch.randn(T, (Hq + 2 * H) * D, generator=g, device=cuda).to(torch.bfloat16)
    ang = torch.rand(P, D // 2, generator=g, device=cuda) * 6.283185307179586
    cache = torch.cat([ang.cos(), ang.sin()], dim=-1).float()
    kc = torch.zeros(b.num_pages, b.page_size, H, D, dtype=torch.bfloat16, device=cuda)
    gate_up = (torch.randn(T, 2 * 512, generator=g, device=cuda) * 3).to(torch.bfloat16)
    scale = torch.tensor(0.02, device=cuda)
    table = torch.randn(4096, 256, generator=g, device=cuda).to(torch.bfloat16)
    ids = torch.randint(0, 4096, (T,), generator=g, device=cuda)
    ids[:3] = torch.tensor([-1, -2, -1], device=cuda)
    last = torch.tensor([17, 4095], device=cuda)
    return dict(b=b, qkv=qkv, cache=cache, kc=kc, vc=kc.clone(), gate_up=gate_up, scale=scale, table=table,
                ids=ids, last=last)


def _step(s):
    b, qkv = s["b"], s["qkv"]
    q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + H) * D], qkv[:, (Hq + H) * D:]
    mas_b200.apply_rope_and_append_paged_kv_cache(b.positions, q, k, v, D, s["cache"], b.batch_indices,
                                                  (s["kc"], s["vc"]), b.kv_indices, b.kv_indptr, b.kv_last_page_len,
                                                  llama_4_scaling_beta=0.1, original_max_position_embeddings=256)
    act = mas_b200.silu_and_mul_quant(s["gate_up"], s["scale"])
    rows = mas_b200.embedding_fill_placeholders(s["ids"], s["table"], s["last"])
    return act, rows


def _snapshot(s, act, rows):
    return {"qkv": s["qkv"].clone(), "kc": s["kc"].clone(), "vc": s["vc"].clone(), "act": act.clone(),
            "rows": rows.clone(), "ids": s["ids"].clone()}


def test_fused_ops_graph_replay_equals_eager(cuda):
    eager_in = _inputs(cuda)
    want = _snapshot(eager_in, *_step(eager_in))

    s = _inputs(cuda)
    fresh = _inputs(cuda)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm up on a side stream, as the runner does
        _step(_inputs(cuda))
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        act, rows = _step(s)
    # restore the inputs the capture may not touch, then replay for real
    for key in ("qkv", "kc", "vc", "ids"):
        s[key].copy_(fresh[key])
    graph.replay()
    torch.cuda.synchronize()
    got = _snapshot(s, act, rows)
    for key in want:
        assert_bits_equal(got[key], want[key], f"graph {key}")
    del graph


def test_fused_ops_torch_compile_equals_eager(cuda):
    eager_in = _inputs(cuda)
    want = _snapshot(eager_in, *_step(eager_in))
    s = _inputs(cuda)
    fn = torch.compile(_step, dynamic=True, fullgraph=False)
    act, rows = fn(s)
    torch.cuda.synchronize()
    got = _snapshot(s, act, rows)
    for key in want:
        assert_bits_equal(got[key], want[key], f"compile {key}")
