"""Records the per-token op calls that the reference's OWN Devstral2Model.forward makes.

    PYTHONPATH=<mini-agent-serve checkout> python tests/golden/gen_reference_layer.py

(The reference's quantize_fp8 is torch.compile'd; on the CPU that needs a C++ compiler with OpenMP,
chosen through the CXX environment variable.)

The reference's model (miniagentserve/models/devstral2/devstral2.py:255-308, decoder layer :230-253,
attention :139-210, MLP :213-224) is built at small dimensions with seeded random weights and run
once, eagerly, on the CPU over a mixed step (decode rows, then prompt chunks) with a paged KV cache.
Its module globals for the five flashinfer functions it imports (devstral2.py:18-23) are replaced by
recorders that run this repository's C oracle (the CPU restatement of those kernels, pinned to
flashinfer's outputs by tests/test_golden_flashinfer.py) and log each call: the keyword and
positional arguments exactly as the forward passed them, and, for every tensor argument, its dtype,
shape, strides, storage offset and the bytes of its whole storage before and after the call (so q
and k keep their layout as strided views of one qkv row). The same is logged for the embedding
(nn.Embedding, :260/:282), for `quantize_fp8` (the reference's own compiled function, :93-95, run
as is) and for the query handed to attention, which carries the llama-4 query scale (:175-179).
The two trtllm attention kernels (CUDA-only, not part of this path) are replaced by a stand-in that
passes the query through to the output, so the step runs end to end on the CPU.

tests/test_gpu_reference_layer.py replays every logged call through mas_b200 (and through flashinfer
when it is importable) on the same inputs and layouts and compares with the logged outputs.

Writes reference_layer_calls.npz next to this file. Identical storage contents are stored once.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(OUT.parent.parent))  # the repository root, for the oracle

import oracle  # noqa: E402
import miniagentserve.models.devstral2.devstral2 as ref  # noqa: E402
from miniagentserve.models.devstral2.configs import Devstral2Config  # noqa: E402

FP8 = torch.float8_e4m3fn


class Log:
    def __init__(self):
        self.blobs: dict[str, np.ndarray] = {}
        self.calls: list[dict] = []

    def blob(self, t: torch.Tensor) -> str:
        st = t.untyped_storage()
        raw = torch.empty(0, dtype=torch.uint8).set_(st, 0, (st.nbytes(),)).clone().numpy()
        key = hashlib.sha1(raw.tobytes()).hexdigest()[:16]
        self.blobs.setdefault(key, raw)
        return key

    def call(self, name: str, fn, args: tuple, kwargs: dict):
        """Logs one call of `fn(*args, **kwargs)`: tensor layouts and storages before/after."""
        storages: dict[int, dict] = {}

        def describe(v):
            if isinstance(v, torch.Tensor):
                key = v.untyped_storage().data_ptr()
                if key not in storages:
                    storages[key] = {"id": len(storages), "tensor": v}
                return {"tensor": storages[key]["id"], "dtype": str(v.dtype).removeprefix("torch."),
                        "shape": list(v.shape), "stride": list(v.stride()),
                        "offset": v.storage_offset()}
            if isinstance(v, tuple):
                return {"tuple": [describe(x) for x in v]}
            return {"value": v}

        d_args = [describe(a) for a in args]
        d_kwargs = {k: describe(v) for k, v in kwargs.items()}
        before = {s["id"]: self.blob(s["tensor"]) for s in storages.values()}
        result = fn(*args, **kwargs)
        after = {s["id"]: self.blob(s["tensor"]) for s in storages.values()}
        entry = {"name": name, "args": d_args, "kwargs": d_kwargs,
                 "storages": [{"before": before[i], "after": after[i]} for i in range(len(storages))]}
        if isinstance(result, torch.Tensor):
            r = result.contiguous()
            entry["result"] = {"blob": self.blob(r), "dtype": str(r.dtype).removeprefix("torch."),
                               "shape": list(r.shape)}
        self.calls.append(entry)
        return result


LOG = Log()


# The oracle behind each flashinfer function, called as the reference calls flashinfer.
def _norm(input, residual, weight, eps=1e-6, enable_pdl=None):
    oracle.fused_add_rmsnorm(input, residual, weight.detach(), eps)


def _norm_quant(out, input, residual, weight, scale, eps=1e-6, enable_pdl=None):
    oracle.fused_add_rmsnorm_quant(out, input, residual, weight.detach(), float(scale), eps)


def _silu(input, out=None, enable_pdl=None):
    return oracle.silu_and_mul(input, out)


def _rope(positions, query, key, head_size, cos_sin_cache, is_neox=True):
    assert oracle.apply_rope_with_cos_sin_cache_inplace(positions, query, key, head_size, cos_sin_cache, is_neox) == 0


def _append(append_key, append_value, batch_indices, positions, paged_kv_cache, kv_indices, kv_indptr,
            kv_last_page_len, kv_layout="NHD"):
    assert oracle.append_paged_kv_cache(append_key, append_value, batch_indices, positions, paged_kv_cache,
                                        kv_indices, kv_indptr, kv_layout) == 0


def _pass_query_through(query, out):
    out.copy_(query)


def logged(name, fn):
    def wrapper(*args, **kwargs):
        return LOG.call(name, fn, args, kwargs)
    return wrapper


def logged_attention(name):
    """The attention stand-in: logs the query the forward hands over (its layout and values) and the
    output slice, and ignores the cache, workspace and lengths (not part of this path)."""
    def wrapper(*, query, out, **_):
        return LOG.call(name, _pass_query_through, (), {"query": query, "out": out})
    return wrapper


def config() -> Devstral2Config:
    return Devstral2Config(
        vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
        num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-5, max_position_embeddings=1024, bos_token_id=1,
        eos_token_id=2, pad_token_id=11, rope_theta=1e6, dtype=torch.bfloat16, rope_factor=4.0,
        rope_original_max_position_embeddings=16, rope_beta_fast=32.0, rope_beta_slow=1.0, rope_mscale=1.0,
        rope_mscale_all_dim=1.0, rope_truncate=True, llama_4_scaling_beta=0.1)


def build_model(cfg: Devstral2Config, g: torch.Generator) -> ref.Devstral2Model:
    model = ref.Devstral2Model(cfg)
    with torch.no_grad():
        model.embed_tokens.weight.copy_(torch.randn(model.embed_tokens.weight.shape, generator=g) * 0.5)
        for layer in model.layers:
            layer.input_layernorm.copy_(1 + 0.1 * torch.randn(cfg.hidden_size, generator=g))
            layer.post_attention_layernorm.copy_(1 + 0.1 * torch.randn(cfg.hidden_size, generator=g))
            for lin in (layer.self_attn.qkv_proj, layer.self_attn.o_proj, layer.mlp.gate_up_proj,
                        layer.mlp.down_proj):
                lin.weight.copy_((torch.randn(lin.weight.shape, generator=g) * 4).to(FP8))
                lin.weight_scale_inv.fill_(1.0 / (16 * lin.weight.shape[1] ** 0.5))
                lin.activation_scale.fill_(0.02)
        model.norm.copy_(1 + 0.1 * torch.randn(cfg.hidden_size, generator=g))
    # As from_pretrained leaves it (devstral2.py:330-345): embedding and norm weights in the model
    # dtype; fp8 weights, fp32 scales and the fp32 cos/sin cache untouched.
    for p in [model.embed_tokens.weight, model.norm] + [w for l in model.layers
                                                        for w in (l.input_layernorm, l.post_attention_layernorm)]:
        p.data = p.data.to(cfg.dtype)
    return model.eval()


def step_inputs(cfg: Devstral2Config, g: torch.Generator, block: int = 16):
    """Three decode rows, then two prompt chunks, as ModelRunner builds them (model_runner.py:31-66)."""
    cached = [19, 4, 32, 0, 10]
    new = [1, 1, 1, 6, 9]
    seq_lens = [c + n for c, n in zip(cached, new)]
    blocks = [-(-s // block) for s in seq_lens]
    max_blocks = max(blocks)
    num_blocks = sum(blocks) + 3
    perm = torch.randperm(num_blocks, generator=g)
    table = torch.full((len(new), max_blocks), num_blocks, dtype=torch.int32)  # padding: the sink block
    o = 0
    for b, nb in enumerate(blocks):
        table[b, :nb] = perm[o:o + nb]
        o += nb
    positions = torch.cat([torch.arange(c, c + n) for c, n in zip(cached, new)])
    batch_indices = torch.cat([torch.full((n,), b) for b, n in enumerate(new)]).to(torch.int32)
    cu = torch.tensor([0, 6, 15], dtype=torch.int32)
    T = positions.shape[0]
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g)
    shape = (cfg.num_hidden_layers, num_blocks + 1, block, cfg.num_key_value_heads, cfg.head_dim)
    k_cache = (torch.randn(shape, generator=g) * 0.1).to(torch.bfloat16)
    v_cache = (torch.randn(shape, generator=g) * 0.1).to(torch.bfloat16)
    return dict(input_ids=ids, k_cache=k_cache, v_cache=v_cache, positions=positions.to(torch.int32),
                batch_indices=batch_indices, seq_lens=torch.tensor(seq_lens, dtype=torch.int32), cu_seqlens_q=cu,
                block_tables=table)


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    g = torch.Generator().manual_seed(2024)
    cfg = config()
    model = build_model(cfg, g)
    inputs = step_inputs(cfg, g)

    ref.fused_add_rmsnorm = logged("fused_add_rmsnorm", _norm)
    ref.fused_add_rmsnorm_quant = logged("fused_add_rmsnorm_quant", _norm_quant)
    ref.silu_and_mul = logged("silu_and_mul", _silu)
    ref.apply_rope_with_cos_sin_cache_inplace = logged("apply_rope_with_cos_sin_cache_inplace", _rope)
    ref.append_paged_kv_cache = logged("append_paged_kv_cache", _append)
    ref.quantize_fp8 = logged("quantize_fp8", ref.quantize_fp8)
    ref.trtllm_batch_decode_with_kv_cache = logged_attention("attention_decode")
    ref.trtllm_batch_context_with_kv_cache = logged_attention("attention_prefill")
    embed_forward = model.embed_tokens.forward
    model.embed_tokens.forward = lambda ids: LOG.call("embedding", embed_forward, (ids,), {})

    with torch.no_grad():
        out = model(**inputs)
    meta = {"config": {k: (str(v) if isinstance(v, torch.dtype) else v) for k, v in cfg.__dict__.items()},
            "embedding_weight_blob": LOG.blob(model.embed_tokens.weight.detach()),
            "embedding_weight_shape": list(model.embed_tokens.weight.shape),
            "calls": LOG.calls, "final_hidden_blob": LOG.blob(out.contiguous())}
    arrays = {f"blob_{k}": v for k, v in LOG.blobs.items()}
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT / "reference_layer_calls.npz", **arrays)
    names = [c["name"] for c in LOG.calls]
    print(f"{len(names)} calls: " + ", ".join(f"{n} x{names.count(n)}" for n in dict.fromkeys(names)))
    print(f"{len(LOG.blobs)} storages, {sum(b.nbytes for b in LOG.blobs.values())} bytes")


if __name__ == "__main__":
    main()
