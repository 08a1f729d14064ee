"""Host-side logic of the drop-in API, without a GPU.

* the flashinfer-compatible argument checks (ValueError / AssertionError) of every wrapper;
* the custom ops are registered in the mas_b200 namespace with the mutation annotations torch.compile
  relies on, trace as opaque nodes under fake tensors, and have no CPU implementation;
* the Embedding module is an nn.Embedding (state dict, initialisation) with the gather as forward;
* byte accounting of the chain equals the figures the benchmark's roofline uses;
* the seeded host inputs are deterministic and within range.
"""
from __future__ import annotations

import pytest
import torch
from torch import nn

import mas_b200
from mas_b200 import workloads as wl
from mas_b200.chain import ChainShape, LayerChain

M = torch.device("meta")
BF = torch.bfloat16


def test_norm_checks():
    x = torch.empty(4, 64, dtype=BF, device=M)
    with pytest.raises(ValueError):
        mas_b200.fused_add_rmsnorm(x, torch.empty(4, 32, dtype=BF, device=M), torch.empty(64, dtype=BF, device=M))
    with pytest.raises(ValueError):
        mas_b200.fused_add_rmsnorm(x, x.clone(), torch.empty(32, dtype=BF, device=M))
    with pytest.raises(ValueError):
        mas_b200.fused_add_rmsnorm(x, x.clone().float(), torch.empty(64, dtype=BF, device=M))
    with pytest.raises(ValueError):
        mas_b200.fused_add_rmsnorm(x.float(), x.float(), torch.empty(64, device=M))
    out = torch.empty(4, 64, dtype=BF, device=M)
    with pytest.raises(ValueError):  # out must be e4m3
        mas_b200.fused_add_rmsnorm_quant(out, x, x.clone(), torch.empty(64, dtype=BF, device=M),
                                         torch.ones(1, device=M))
    with pytest.raises(ValueError):  # scale must be a scalar
        mas_b200.fused_add_rmsnorm_quant(torch.empty(4, 64, dtype=torch.float8_e4m3fn, device=M), x, x.clone(),
                                         torch.empty(64, dtype=BF, device=M), torch.ones(2, device=M))


def test_norm_accepts_meta_and_runs_fake_kernel():
    x = torch.empty(4, 64, dtype=BF, device=M)
    mas_b200.fused_add_rmsnorm(x, x.clone(), torch.empty(64, dtype=BF, device=M), 1e-5)
    mas_b200.fused_add_rmsnorm_quant(torch.empty(4, 64, dtype=torch.float8_e4m3fn, device=M), x, x.clone(),
                                     torch.empty(64, dtype=BF, device=M), torch.ones((), device=M))


def test_silu_checks_follow_flashinfer():
    with pytest.raises(ValueError, match="multiple of 16 bytes"):
        mas_b200.silu_and_mul(torch.empty(3, 6, dtype=BF, device=M))
    with pytest.raises(AssertionError):
        mas_b200.silu_and_mul(torch.empty(3, 16, dtype=BF, device=M), out=torch.empty(3, 16, dtype=BF, device=M))
    with pytest.raises(AssertionError):
        mas_b200.silu_and_mul(torch.empty(3, 16, dtype=BF, device=M), out=torch.empty(8, dtype=BF, device=M))
    out = mas_b200.silu_and_mul(torch.empty(2, 5, 32, dtype=BF, device=M))
    assert out.shape == (2, 5, 16) and out.dtype == BF


def test_rope_checks_follow_flashinfer():
    pos = torch.empty(3, dtype=torch.int32, device=M)
    q, k = torch.empty(3, 256, dtype=BF, device=M), torch.empty(3, 128, dtype=BF, device=M)
    with pytest.raises(ValueError, match="float32"):
        mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, q, k, 128, torch.empty(10, 128, dtype=BF, device=M))
    with pytest.raises(ValueError):
        mas_b200.apply_rope_with_cos_sin_cache_inplace(pos.float(), q, k, 128, torch.empty(10, 128, device=M))
    with pytest.raises(ValueError):
        mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, q, k, 128, torch.empty(10, 130, device=M))
    with pytest.raises(ValueError):
        mas_b200.apply_rope_with_cos_sin_cache_inplace(pos[:2], q, k, 128, torch.empty(10, 128, device=M))
    mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, q, k, 128, torch.empty(10, 128, device=M))


def test_embedding_checks():
    with pytest.raises(ValueError):
        mas_b200.embedding_gather(torch.empty(3, device=M), torch.empty(10, 4, device=M))
    with pytest.raises(ValueError):
        mas_b200.embedding_out(torch.empty(3, 5, device=M), torch.empty(3, dtype=torch.long, device=M),
                               torch.empty(10, 4, device=M))
    out = mas_b200.embedding_gather(torch.empty(2, 3, dtype=torch.long, device=M), torch.empty(10, 4, dtype=BF, device=M))
    assert out.shape == (2, 3, 4) and out.dtype == BF


def test_ops_registered_with_mutation_annotations():
    expect = {
        "fused_add_rmsnorm": ("input", "residual"),
        "fused_add_rmsnorm_quant": ("out", "residual"),
        "silu_and_mul": ("out",),
        "apply_rope_pos_ids_cos_sin_cache": ("q", "k"),
        "apply_rope_q_scale": ("q", "k"),
        "append_paged_kv_cache": ("k_cache", "v_cache"),
        "rope_append_paged_kv_cache": ("q", "k", "k_cache", "v_cache"),
        "embedding_out": ("out",),
        "embedding": (),
        "embedding_fill": ("input_ids",),
    }
    for name, mutated in expect.items():
        schema = getattr(torch.ops.mas_b200, name).default._schema
        got = tuple(a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write)
        assert got == mutated, (name, got)


def test_no_cpu_fallback():
    x = torch.randn(2, 16, dtype=BF)
    with pytest.raises(NotImplementedError):
        mas_b200.fused_add_rmsnorm(x, x.clone(), torch.ones(16, dtype=BF))
    with pytest.raises(NotImplementedError):
        mas_b200.silu_and_mul(x)
    with pytest.raises(NotImplementedError):
        mas_b200.embedding_gather(torch.tensor([1]), torch.randn(4, 8))


def test_layer_traces_as_opaque_custom_ops():
    from torch.fx.experimental.proxy_tensor import make_fx

    s = ChainShape(hidden_size=64, intermediate_size=32, num_attention_heads=2, num_key_value_heads=1, head_dim=32,
                   vocab_size=100, num_hidden_layers=1)

    def layer(hidden, residual, attn, qkv, gate_up, act, w, pos, cache):
        mas_b200.fused_add_rmsnorm(hidden, residual, w, 1e-5)
        mas_b200.apply_rope_with_cos_sin_cache_inplace(pos, qkv[:, :64], qkv[:, 64:96], 32, cache)
        mas_b200.fused_add_rmsnorm(attn, residual, w, 1e-5)
        return mas_b200.silu_and_mul(gate_up, out=act)

    T = 5
    args = (torch.randn(T, 64).to(BF), torch.randn(T, 64).to(BF), torch.randn(T, 64).to(BF),
            torch.randn(T, s.qkv_size).to(BF), torch.randn(T, 64).to(BF), torch.empty(T, 32, dtype=BF),
            torch.ones(64, dtype=BF), torch.zeros(T, dtype=torch.int32), torch.zeros(8, 32))
    gm = make_fx(layer, tracing_mode="fake")(*args)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert sum("mas_b200.fused_add_rmsnorm" in t for t in targets) == 2
    assert any("mas_b200.apply_rope_pos_ids_cos_sin_cache" in t for t in targets)
    assert any("mas_b200.silu_and_mul" in t for t in targets)


def test_embedding_module_is_nn_embedding():
    e = mas_b200.Embedding(10, 4)
    assert isinstance(e, nn.Embedding) and list(e.state_dict()) == ["weight"]
    parent = nn.Module()
    parent.embed_tokens = mas_b200.Embedding(10, 4)
    assert "embed_tokens.weight" in parent.state_dict()
    with pytest.raises(NotImplementedError):
        mas_b200.Embedding(10, 4, max_norm=1.0)(torch.tensor([1]))


def test_chain_bytes_match_the_benchmark_figures():
    s = wl.CHAIN_SHAPE
    T = 4352
    assert s.bytes_per_layer(T) == 1_838_351_360
    assert s.embed_bytes(T) == 213_944_320
    assert LayerChain(s).step_bytes(T) == 161_988_864_000
    assert LayerChain(s).kernel_launches() == 353
    assert 8 * 4096 * 5120 + 2 * 5120 == 167_782_400      # configuration 1
    assert 6 * 8192 * 32768 == 1_610_612_736               # configuration 2
    assert 2 * 2 * (32 + 8) * 128 + 4 * 128 + 4 == 20_996  # configuration 3, per token
    assert 2 * 2 * 16384 * 5120 + 4 * 16384 == 335_609_856  # configuration 4


def test_chain_shape_from_model_config():
    class Cfg:
        hidden_size, intermediate_size, num_attention_heads, num_key_value_heads = 12288, 28672, 96, 8
        head_dim, vocab_size, num_hidden_layers, rms_norm_eps = 128, 131072, 88, 1e-5
        rope_theta, max_position_embeddings = 1e9, 131072
    assert ChainShape.from_model_config(Cfg) == wl.CHAIN_SHAPE


def test_seeded_host_inputs():
    ids, pos = wl.chain_host_inputs()
    ids2, pos2 = wl.chain_host_inputs()
    assert torch.equal(ids, ids2) and torch.equal(pos, pos2)
    assert ids.shape == (4352,) and ids.dtype == torch.int64 and pos.dtype == torch.int32
    assert int(ids.min()) >= 0 and int(ids.max()) < 131072 and int(pos.min()) >= 0 and int(pos.max()) < 131072
    # the prefill chunks are consecutive positions
    assert torch.equal(pos[256 + 1: 256 + 2048] - pos[256: 256 + 2047], torch.ones(2047, dtype=torch.int32))
    ids4, _ = wl.chain_host_inputs(replicas=4)
    assert ids4.shape == (4 * 4352,) and torch.equal(ids4[:4352], ids)
    b = wl.rope_batch()
    assert b.seq_lens.shape == (64,) and int(b.seq_lens.min()) >= 1 and int(b.seq_lens.max()) <= 1024
    assert b.positions.shape[0] == int(b.seq_lens.sum()) and int(b.positions.max()) < 65536 + 1024


def test_operands_on_another_device_are_rejected_before_any_launch():
    """A host tensor among device operands raises (as aten does) instead of reaching a kernel as a
    host pointer. Meta tensors stand in for the device here; the mismatch is caught in Python."""
    C = torch.device("cpu")
    x = torch.empty(4, 64, dtype=BF, device=M)
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.fused_add_rmsnorm(x, torch.empty(4, 64, dtype=BF, device=M), torch.empty(64, dtype=BF, device=C))
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.fused_add_rmsnorm_quant(torch.empty(4, 64, dtype=torch.float8_e4m3fn, device=C), x,
                                         torch.empty(4, 64, dtype=BF, device=M), torch.empty(64, dtype=BF, device=M),
                                         torch.ones(1, device=M))
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.silu_and_mul(torch.empty(4, 64, dtype=BF, device=M), out=torch.empty(4, 32, dtype=BF, device=C))
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.silu_and_mul_quant(torch.empty(4, 64, dtype=BF, device=M), torch.ones(1, device=M),
                                    out=torch.empty(4, 32, dtype=torch.float8_e4m3fn, device=C))
    q, k = torch.empty(3, 2 * 128, dtype=BF, device=M), torch.empty(3, 128, dtype=BF, device=M)
    pos = torch.zeros(3, dtype=torch.int32, device=M)
    cache = torch.empty(16, 128, device=M)
    for bad in ({"positions": torch.zeros(3, dtype=torch.int32)}, {"cos_sin_cache": torch.empty(16, 128)}):
        args = {"positions": pos, "cos_sin_cache": cache} | bad
        with pytest.raises(RuntimeError, match="same device"):
            mas_b200.apply_rope_with_cos_sin_cache_inplace(args["positions"], q, k, 128, args["cos_sin_cache"])
        with pytest.raises(RuntimeError, match="same device"):
            mas_b200.apply_rope_and_llama4_query_scale_inplace(args["positions"], q, k, 128, args["cos_sin_cache"],
                                                               0.1, 8192)
    kc = torch.empty(4, 16, 1, 128, dtype=BF, device=M)
    ind = torch.zeros(4, dtype=torch.int32, device=M)
    indptr = torch.tensor([0, 4], dtype=torch.int32, device=M)
    last = torch.ones(1, dtype=torch.int32, device=M)
    bi = torch.zeros(3, dtype=torch.int32, device=M)
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.append_paged_kv_cache(k.view(3, 1, 128), k.view(3, 1, 128), bi, pos, (kc, kc), torch.zeros(4, dtype=torch.int32), indptr, last)
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.apply_rope_and_append_paged_kv_cache(pos, q, k, k.clone(), 128, cache, torch.zeros(3, dtype=torch.int32),
                                                      (kc, kc), ind,
                                                      indptr, last)
    table = torch.empty(10, 64, dtype=BF, device=M)
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.embedding_gather(torch.zeros(3, dtype=torch.int64), table)
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.embedding_out(torch.empty(3, 64, dtype=BF), torch.zeros(3, dtype=torch.int64, device=M), table)
    with pytest.raises(RuntimeError, match="same device"):
        mas_b200.embedding_fill_placeholders(torch.zeros(3, dtype=torch.int64, device=M), table,
                                             torch.zeros(2, dtype=torch.int64))
