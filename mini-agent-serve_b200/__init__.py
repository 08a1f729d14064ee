"""mas_b200: B200-native per-token layer ops of mini-agent-serve's Devstral 2 model.

Drop-in replacements for the flashinfer functions and the nn.Embedding that
miniagentserve/models/devstral2/devstral2.py calls on its per-token path (devstral2.py:18-23, :260):

    from mas_b200 import (fused_add_rmsnorm, fused_add_rmsnorm_quant, silu_and_mul,
                          apply_rope_with_cos_sin_cache_inplace, Embedding)

Every op is a hand-written sm_100a CUDA kernel in libmas_b200.so, reached through the C ABI of
include/mas_b200.h and registered as a `mas_b200::*` torch custom op (eager, torch.compile and CUDA
graph capture all work).

The native libraries are loaded by the first access to an op (or to `ops`, `_lib`, `Embedding`, ...),
and that access raises ImportError if they are missing: there is no fallback. The host-only modules
(`rope_cache`, `chain`, `workloads`) import without them, so a process that only builds inputs or
cos/sin caches never maps the CUDA library.

The package directory is named ``mini-agent-serve_b200``; ``import mas_b200`` loads it under that name
through the alias module at the repository root.
"""
from __future__ import annotations

import importlib

# Names served by the native-library modules, loaded on first access.
_NATIVE = {
    "ops": ("ops", None),
    "_lib": ("_lib", None),
    "embedding": ("embedding", None),
    "MasError": ("_lib", "MasError"),
    "prepare_device": ("_lib", "prepare_device"),
    "read_fault_word": ("_lib", "read_fault_word"),
    "status_string": ("_lib", "status_string"),
    "version": ("_lib", "version"),
    "Embedding": ("embedding", "Embedding"),
    "apply_rope_and_llama4_query_scale_inplace": ("ops", None),
    "apply_rope_with_cos_sin_cache_inplace": ("ops", None),
    "append_paged_kv_cache": ("ops", None),
    "apply_rope_and_append_paged_kv_cache": ("ops", None),
    "embedding_gather": ("ops", "embedding"),
    "embedding_fill_placeholders": ("ops", None),
    "embedding_out": ("ops", None),
    "fused_add_rmsnorm": ("ops", None),
    "fused_add_rmsnorm_quant": ("ops", None),
    "read_status": ("ops", None),
    "silu_and_mul": ("ops", None),
    "silu_and_mul_quant": ("ops", None),
}
# Host-only modules and names (no native library).
_HOST = {
    "rope_cache": ("rope_cache", None),
    "chain": ("chain", None),
    "workloads": ("workloads", None),
    "plain_cos_sin_cache": ("rope_cache", "plain_cos_sin_cache"),
    "yarn_cos_sin_cache": ("rope_cache", "yarn_cos_sin_cache"),
}

__all__ = sorted((set(_NATIVE) | set(_HOST)) - {"_lib"})


def __getattr__(name: str):
    try:
        module, attr = _NATIVE.get(name) or _HOST[name]
    except KeyError:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}") from None
    mod = importlib.import_module(f"{__name__}.{module}")
    value = mod if attr is None and name == module else getattr(mod, attr or name)
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(__all__))
