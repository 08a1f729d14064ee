"""Generates golden fixtures from the reference's OWN code (run where mini-agent-serve is importable).

    PYTHONPATH=<mini-agent-serve checkout> python tests/golden/gen_reference_golden.py

Writes, next to this file:
  reference_yarn_cache.npz  rows of Devstral2Model's fp32 cos|sin cache, built by the reference's
                            _yarn_cos_sin_cache (miniagentserve/models/devstral2/devstral2.py:44-90)
                            for three rope configurations (Devstral2Config fields, configs.py:153-162);
  reference_embedding.npz   Devstral2Model.embed_tokens(input_ids) (devstral2.py:260, :282) on a small
                            seeded bf16 table, int64 and int32 ids including 0 and vocab-1.

Only the reference's functions and modules compute the outputs; this script only builds inputs
and saves results. The fixtures are small (tens of KB) and committed; tests never import the
reference.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from miniagentserve.models.devstral2.configs import Devstral2Config
from miniagentserve.models.devstral2.devstral2 import Devstral2Model, _yarn_cos_sin_cache

OUT = Path(__file__).resolve().parent

# Devstral-2-like rope settings (the values a config.json's rope_parameters carries), plus two
# variants that reach the other branches: no truncation and the single-mscale path, and an exact
# low == high collapse guarded by +0.001.
ROPE_CASES = {
    "yarn_a": dict(head_dim=128, rope_theta=1e8, max_position_embeddings=65536, rope_factor=16.0,
                   rope_original_max_position_embeddings=4096, rope_beta_fast=32.0, rope_beta_slow=1.0,
                   rope_mscale=1.0, rope_mscale_all_dim=1.0, rope_truncate=True),
    "yarn_b": dict(head_dim=128, rope_theta=1e6, max_position_embeddings=32768, rope_factor=8.0,
                   rope_original_max_position_embeddings=8192, rope_beta_fast=16.0, rope_beta_slow=2.0,
                   rope_mscale=0.0, rope_mscale_all_dim=0.0, rope_truncate=False),
    "yarn_c": dict(head_dim=64, rope_theta=1e4, max_position_embeddings=8192, rope_factor=4.0,
                   rope_original_max_position_embeddings=2048, rope_beta_fast=32.0, rope_beta_slow=32.0,
                   rope_mscale=0.707, rope_mscale_all_dim=1.0, rope_truncate=True),
}


def tiny_config(**rope) -> Devstral2Config:
    base = dict(vocab_size=1000, hidden_size=72, intermediate_size=64, num_hidden_layers=1, num_attention_heads=2,
                num_key_value_heads=1, head_dim=rope.get("head_dim", 36), rms_norm_eps=1e-5,
                max_position_embeddings=rope.get("max_position_embeddings", 64), bos_token_id=1, eos_token_id=2,
                pad_token_id=11, rope_theta=rope.get("rope_theta", 1e6), dtype=torch.bfloat16,
                rope_factor=rope.get("rope_factor", 4.0),
                rope_original_max_position_embeddings=rope.get("rope_original_max_position_embeddings", 16),
                rope_beta_fast=rope.get("rope_beta_fast", 32.0), rope_beta_slow=rope.get("rope_beta_slow", 1.0),
                rope_mscale=rope.get("rope_mscale", 0.0), rope_mscale_all_dim=rope.get("rope_mscale_all_dim", 0.0),
                rope_truncate=rope.get("rope_truncate", True), llama_4_scaling_beta=0.0)
    return Devstral2Config(**base)


def main() -> None:
    g = torch.Generator().manual_seed(1234)
    arrays = {}
    for name, rope in ROPE_CASES.items():
        cache = _yarn_cos_sin_cache(tiny_config(**rope))
        P = cache.shape[0]
        rows = torch.cat([torch.arange(64), torch.randint(64, P, (64,), generator=g), torch.tensor([P - 1])])
        arrays[f"{name}_rows"] = rows.numpy().astype(np.int64)
        arrays[f"{name}_cache"] = cache[rows].numpy()
        arrays[f"{name}_shape"] = np.array(cache.shape, dtype=np.int64)
        for k, v in rope.items():
            arrays[f"{name}_param_{k}"] = np.array(v)
    np.savez_compressed(OUT / "reference_yarn_cache.npz", **arrays)

    cfg = tiny_config()
    with torch.device("cpu"):
        model = Devstral2Model(cfg)
    with torch.no_grad():
        model.embed_tokens.weight.copy_((torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g) * 0.02))
        model.embed_tokens.weight.data = model.embed_tokens.weight.data.to(torch.bfloat16)
        ids64 = torch.cat([torch.tensor([0, cfg.vocab_size - 1, 7, 7]),
                           torch.randint(0, cfg.vocab_size, (60,), generator=g)])
        out64 = model.embed_tokens(ids64)
        ids32 = ids64.flip(0).to(torch.int32)
        out32 = model.embed_tokens(ids32)
    np.savez_compressed(
        OUT / "reference_embedding.npz",
        table=model.embed_tokens.weight.view(torch.int16).numpy(),
        ids64=ids64.numpy(), out64=out64.view(torch.int16).numpy(),
        ids32=ids32.numpy(), out32=out32.view(torch.int16).numpy(),
    )
    print("wrote", OUT / "reference_yarn_cache.npz", OUT / "reference_embedding.npz")


if __name__ == "__main__":
    main()
