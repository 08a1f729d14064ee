"""The per-layer op chain (configuration 5) against the oracle, and the three ways the engine runs it.

mini-agent-serve's model runner calls the per-token ops eagerly, under torch.compile(dynamic=True),
and replayed from CUDA graphs (miniagentserve/engine/model_runner.py:98-140). These tests run the
chain of ops (mas_b200.chain.LayerChain, the op sequence of Devstral2DecoderLayer.forward) and check:
  * one full step of configuration 5 -- 88 layers, T = 4352, H = 12288 -- every op checked on
    sampled token rows against the oracle applied to that op's inputs (ops are per-token, so rows
    are independent), and the chained launches equal to a synchronised op-by-op run;
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


def test_chain_config5_full_step_every_op_on_sampled_rows(cuda):
    """88 layers at T = 4352, H = 12288 (256 decode + 2 x 2048 prefill), op by op.

    After every op of every layer, the op's outputs on 9 sampled token rows are compared with the
    oracle applied to that op's own inputs on those rows (snapshotted from the GPU just before the
    op). Per-op comparison keeps the bar at <= 1 ulp: an end-to-end replay would let the last-bit
    differences of early layers feed later ones (the residual stream carries them forward).
    """
    s = wl.CHAIN_SHAPE
    ids, pos = wl.chain_host_inputs()
    b = wl.chain_buffers(ids, pos, device=cuda)
    rows = [0, 1, 128, 255, 256, 257, 2303, 2304, ids.shape[0] - 1]
    idx = torch.tensor(rows, device=cuda)
    take = lambda t: t.index_select(0, idx).cpu()  # noqa: E731
    pos_rows, cache = pos[rows], b.cos_sin_cache.cpu()
    w_in, w_post = b.w_in.cpu(), b.w_post.cpu()
    worst = {"embed": 0, "norm_in": 0, "rope": 0, "norm_post": 0, "silu": 0, "residual": 0}

    def check(name, got, want, exact=False):
        if exact:
            assert_bits_equal(got, want, name)
        else:
            worst[name] = max(worst[name], assert_ulp(got, want, what=name)["max_ulp"])

    mas_b200.embedding_out(b.hidden, b.ids, b.table)
    ref, st = oracle.embedding(ids[rows], b.table.cpu())
    check("embed", take(b.hidden), ref, exact=True)
    b.residual.zero_()
    q = b.qkv[:, : s.q_size]
    k = b.qkv[:, s.q_size: s.q_size + s.kv_size]
    act_in = take(b.gate_up)  # read-only through the step
    for l in range(s.num_hidden_layers):
        h0, r0 = take(b.hidden), take(b.residual)
        mas_b200.fused_add_rmsnorm(b.hidden, b.residual, b.w_in[l], s.rms_norm_eps)
        oracle.fused_add_rmsnorm(h0, r0, w_in[l], s.rms_norm_eps)
        check("norm_in", take(b.hidden), h0)
        check("residual", take(b.residual), r0, exact=True)

        qkv0 = take(b.qkv)
        mas_b200.apply_rope_with_cos_sin_cache_inplace(b.positions, q, k, s.head_dim, b.cos_sin_cache)
        oracle.apply_rope_with_cos_sin_cache_inplace(pos_rows, qkv0[:, : s.q_size],
                                                     qkv0[:, s.q_size: s.q_size + s.kv_size], s.head_dim, cache)
        check("rope", take(b.qkv), qkv0)

        a0, r1 = take(b.attn_out), take(b.residual)
        mas_b200.fused_add_rmsnorm(b.attn_out, b.residual, b.w_post[l], s.rms_norm_eps)
        oracle.fused_add_rmsnorm(a0, r1, w_post[l], s.rms_norm_eps)
        check("norm_post", take(b.attn_out), a0)
        check("residual", take(b.residual), r1, exact=True)

        mas_b200.silu_and_mul(b.gate_up, out=b.act)
        check("silu", take(b.act), oracle.silu_and_mul(act_in))
    assert max(worst.values()) <= 1, worst
    assert mas_b200.read_fault_word(cuda.index) == 0


def test_chain_config5_step_matches_op_by_op(cuda):
    """LayerChain.step (one launch after another, programmatic dependent launch on) gives exactly the
    op-by-op result: the chained launches add no ordering hazard."""
    s = wl.CHAIN_SHAPE
    ids, pos = wl.chain_host_inputs()
    layers = 8
    a = wl.chain_buffers(ids, pos, device=cuda, layers=layers)
    LayerChain(s, layers=layers).step(a)
    b = wl.chain_buffers(ids, pos, device=cuda, layers=layers)
    chain = LayerChain(s, layers=layers)
    chain.embed(b)
    torch.cuda.synchronize()
    b.residual.zero_()
    for l in range(layers):
        chain.layer(b, l)
        torch.cuda.synchronize()
    for n in ("hidden", "residual", "attn_out", "qkv", "act"):
        assert_bits_equal(getattr(a, n), getattr(b, n), f"chained vs synchronised {n}")


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
    """The fp8-out norms and the fp8-out SiLU-mul, captured in a graph (scales read on the device)."""
    b = _small_buffers(cuda)
    b.x_fp8 = torch.empty(b.hidden.shape, dtype=torch.float8_e4m3fn, device=cuda)
    b.act_fp8 = torch.empty(b.act.shape, dtype=torch.float8_e4m3fn, device=cuda)
    b.act_scale = torch.tensor([0.05, 0.1, 0.02], device=cuda)
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
    assert_ulp(b.act_fp8.cpu(), oracle.silu_and_mul_quant(b.gate_up.cpu(), 0.02), what="fp8 SiLU-mul")
