"""mas_b200: B200-native per-token layer ops of mini-agent-serve's Devstral 2 model.

Drop-in replacements for the flashinfer functions and the nn.Embedding that
miniagentserve/models/devstral2/devstral2.py calls on its per-token path (devstral2.py:18-23, :260):

    from mas_b200 import (fused_add_rmsnorm, fused_add_rmsnorm_quant, silu_and_mul,
                          apply_rope_with_cos_sin_cache_inplace, Embedding)

Every op is a hand-written sm_100a CUDA kernel in libmas_b200.so, reached through the C ABI of
include/mas_b200.h and registered as a `mas_b200::*` torch custom op (eager, torch.compile and CUDA
graph capture all work). Importing the package loads the library; if it is missing the import fails.

The package directory is named ``mini-agent-serve_b200``; ``import mas_b200`` resolves to it through
the alias module at the repository root, and the submodules are registered under both names.
"""
from __future__ import annotations

import sys as _sys

from . import _lib, ops, rope_cache, embedding, chain, workloads  # noqa: F401
from ._lib import MasError, prepare_device, read_fault_word, status_string, version
from .embedding import Embedding
from .ops import (
    apply_rope_and_llama4_query_scale_inplace,
    apply_rope_with_cos_sin_cache_inplace,
    append_paged_kv_cache,
    apply_rope_and_append_paged_kv_cache,
    embedding as embedding_gather,
    embedding_fill_placeholders,
    embedding_out,
    fused_add_rmsnorm,
    fused_add_rmsnorm_quant,
    read_status,
    silu_and_mul,
    silu_and_mul_quant,
    status_word,
)
from .rope_cache import plain_cos_sin_cache, yarn_cos_sin_cache

__all__ = [
    "Embedding",
    "MasError",
    "apply_rope_and_llama4_query_scale_inplace",
    "apply_rope_with_cos_sin_cache_inplace",
    "append_paged_kv_cache",
    "apply_rope_and_append_paged_kv_cache",
    "chain",
    "embedding_fill_placeholders",
    "embedding_gather",
    "embedding_out",
    "fused_add_rmsnorm",
    "fused_add_rmsnorm_quant",
    "ops",
    "plain_cos_sin_cache",
    "prepare_device",
    "read_fault_word",
    "read_status",
    "rope_cache",
    "silu_and_mul",
    "silu_and_mul_quant",
    "status_string",
    "status_word",
    "version",
    "workloads",
    "yarn_cos_sin_cache",
]

# One module object per submodule, whichever name imported the package.
for _name in ("_lib", "ops", "rope_cache", "embedding", "chain", "workloads"):
    _mod = _sys.modules[f"{__name__}.{_name}"]
    _sys.modules.setdefault(f"mas_b200.{_name}", _mod)
_sys.modules.setdefault("mas_b200", _sys.modules[__name__])
