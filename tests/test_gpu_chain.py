"""The per-layer op chain (configuration 5) against the oracle, and the three ways the engine runs it.

mini-agent-serve's model runner calls the per-token ops eagerly, under torch.compile(dynamic=True),
and replayed from CUDA graphs (miniagentserve/engine/model_runner.py:98-140). These tests run the
chain of ops (mas_b200.chain.LayerChain, the op sequence of Devstral2DecoderLayer.forward) and check:
  * one full step of configuration 5 -- 88 layers, T = 4352, H = 12288 -- on sampled token rows
    against the oracle replaying the same rows (every op is per-token, so rows are independent);
  * CUDA-graph capture and replay give bit-identical results to eager execution;
  * torch.compile(dynamic=True) of a decoder-layer-shaped function gives bit-identical results.
"""
from __future__ import annotations

import pytest
import torch

import mas_b200
import oracle
from mas_b200 import workloads as wl
from mas_b200.chain import ChainShape, LayerChain
from parity import assert_bits_equal, assert_ulp

pytestmark = pytest.mark.gpu

SMALL = ChainShape(hidden_size=2048, intermediate_size=4096, num_attention_heads=16, num_key_value_heads=4,
                   head_dim=128, vocab_size=8192, num_hidden_layers=3, rms_norm_eps=1e-5, rope_theta=1e9,
                   max_position_embeddings=16384)


def _oracle_rows(b_snap: dict, s: ChainShape, layers: int) -> dict:
    hidden, st = oracle.embedding(b_snap["ids"], b_snap["table"])
    assert st == 0
    residual = torch.zeros_like(hidden)
    attn, qkv, act = b_snap["attn_out"].clone(), b_snap["qkv"].clone(), None
    for l in range(layers):
        oracle.fused_add_rmsnorm(hidden, residual, b_snap["w_in"][l], s.rms_norm_eps)
        oracle.apply_rope_with_cos_sin_cache_inplace(b_snap["positions"], qkv[:, : s.q_size],
                                                     qkv[:, s.q_size: s.q_size + s.kv_size], s.head_dim,
                                                     b_snap["cache"])
        oracle.fused_add_rmsnorm(attn, residual, b_snap["w_post"][l], s.rms_norm_eps)
        act = oracle.silu_and_mul(b_snap["gate_up"])
    return {"hidden": hidden, "residual": residual, "attn_out": attn, "qkv": qkv, "act": act}


def test_chain_config5_full_step_sampled_rows(cuda):
    """88 layers at T = 4352, H = 12288 (256 decode + 2 x 2048 prefill); 9 token rows replayed on CPU."""
    s = wl.CHAIN_SHAPE
    ids, pos = wl.chain_host_inputs()
    b = wl.chain_buffers(ids, pos, device=cuda)
    rows = [0, 1, 128, 255, 256, 257, 2303, 2304, ids.shape[0] - 1]
    idx = torch.tensor(rows, device=cuda)
    snap = {n: getattr(b, n).index_select(0, idx).cpu() for n in ("attn_out", "qkv", "gate_up")}
    snap.update(ids=ids[rows], positions=pos[rows], w_in=b.w_in.cpu(), w_post=b.w_post.cpu(),
                cache=b.cos_sin_cache.cpu())
    snap["table"] = b.table.cpu()
    LayerChain(s).step(b)
    torch.cuda.synchronize()
    ref = _oracle_rows(snap, s, s.num_hidden_layers)
    for n in ("hidden", "residual", "attn_out", "qkv", "act"):
        got = getattr(b, n).index_select(0, idx).cpu()
        assert_ulp(got, ref[n], what=f"config 5 {n}")
    assert mas_b200.read_fault_word(cuda.index) == 0


def _small_buffers(cuda, T=320, seed=11):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, SMALL.vocab_size, (T,), generator=g)
    pos = torch.randint(0, SMALL.max_position_embeddings, (T,), generator=g).to(torch.int32)
    return wl.chain_buffers(ids, pos, device=cuda, seed=seed, shape=SMALL)


def _state(b):
    return {n: getattr(b, n).clone() for n in ("hidden", "residual", "attn_out", "qkv", "act")}


def test_chain_cuda_graph_replay_matches_eager(cuda):
    eager, graphed = _small_buffers(cuda), _small_buffers(cuda)
    chain = LayerChain(SMALL)
    chain.step(eager)
    # warm up on a side stream, then capture one step, as the model runner does
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    scratch = _small_buffers(cuda, seed=12)
    with torch.cuda.stream(side):
        for _ in range(2):
            chain.step(scratch)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    before = _state(graphed)
    with torch.cuda.graph(g):
        chain.step(graphed)
    # capture does not execute: restore the pre-capture state, then replay
    for n, t in before.items():
        getattr(graphed, n).copy_(t)
    g.replay()
    torch.cuda.synchronize()
    for n, t in _state(eager).items():
        assert_bits_equal(getattr(graphed, n), t, f"graph {n}")
    del g


def test_chain_torch_compile_matches_eager(cuda):
    s = SMALL

    def layer(hidden, residual, attn, qkv, gate_up, act, w_in, w_post, pos, cache):
        mas_b200.fused_add_rmsnorm(hidden, residual, w_in, s.rms_norm_eps, enable_pdl=True)
        mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, qkv[:, : s.q_size],
                                                       qkv[:, s.q_size: s.q_size + s.kv_size], s.head_dim, cache,
                                                       is_neox=True)
        mas_b200.fused_add_rmsnorm(attn, residual, w_post, s.rms_norm_eps, enable_pdl=True)
        return mas_b200.silu_and_mul(gate_up, out=act, enable_pdl=True)

    compiled = torch.compile(layer, dynamic=True)
    results = []
    for fn in (layer, compiled):
        b = _small_buffers(cuda)
        mas_b200.embedding_out(b.hidden, b.ids, b.table)
        with torch.inference_mode():
            fn(b.hidden, b.residual, b.attn_out, b.qkv, b.gate_up, b.act, b.w_in[0], b.w_post[0], b.positions,
               b.cos_sin_cache)
        torch.cuda.synchronize()
        results.append(_state(b))
    for n in results[0]:
        assert_bits_equal(results[1][n], results[0][n], f"compile {n}")


def test_chain_quant_form_graph(cuda):
    """The fp8-out norms the decoder layers call, captured in a graph (scale read on the device)."""
    b = _small_buffers(cuda)
    b.x_fp8 = torch.empty(b.hidden.shape, dtype=torch.float8_e4m3fn, device=cuda)
    b.act_scale = torch.tensor([0.05, 0.1], device=cuda)
    chain = LayerChain(SMALL, quant=True, layers=1)
    mas_b200.embedding_out(b.hidden, b.ids, b.table)
    ref_in = (b.hidden.cpu(), b.residual.cpu())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain.layer(b, 0)
    g.replay()
    torch.cuda.synchronize()
    out = torch.empty(b.hidden.shape, dtype=torch.float8_e4m3fn)
    # the graph's second norm wrote x_fp8 last: recompute both norms on the CPU in order
    h, r = ref_in[0].clone(), ref_in[1].clone()
    oracle.fused_add_rmsnorm_quant(out, h, r, b.w_in[0].cpu(), 0.05, SMALL.rms_norm_eps)
    attn_before = _small_buffers(cuda).attn_out.cpu()  # same seed: the attention stand-in before the step
    oracle.fused_add_rmsnorm_quant(out, attn_before, r, b.w_post[0].cpu(), 0.1, SMALL.rms_norm_eps)
    assert_bits_equal(b.residual.cpu(), r, "residual")
    assert_ulp(b.x_fp8.cpu(), out, what="fp8 out of the post-attention norm")
