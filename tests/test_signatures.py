"""The drop-ins keep the signatures of the flashinfer functions the reference imports
(miniagentserve/models/devstral2/devstral2.py:18-23, :170): same parameter names in the same order,
same kinds and defaults. Additions may only follow as trailing keyword parameters with defaults, so
every call the reference makes binds identically. flashinfer is an installed package here (it is
what the reference calls); the test skips where it is absent.
"""
from __future__ import annotations

import inspect

import pytest

import mas_b200

flashinfer = pytest.importorskip("flashinfer")

PAIRS = [
    ("flashinfer.norm", "fused_add_rmsnorm"),
    ("flashinfer.norm", "fused_add_rmsnorm_quant"),
    ("flashinfer.activation", "silu_and_mul"),
    ("flashinfer.rope", "apply_rope_with_cos_sin_cache_inplace"),
    ("flashinfer.page", "append_paged_kv_cache"),
]


@pytest.mark.parametrize("module,name", PAIRS)
def test_signature_is_a_prefix_of_ours(module, name):
    import importlib

    theirs = inspect.signature(getattr(importlib.import_module(module), name)).parameters
    ours = inspect.signature(getattr(mas_b200, name)).parameters
    t, o = list(theirs.values()), list(ours.values())
    assert [p.name for p in o[: len(t)]] == [p.name for p in t], (name, list(ours), list(theirs))
    for a, b in zip(t, o):
        assert a.kind == b.kind, (name, a.name)
        assert a.default == b.default or (a.default is None and b.default is None), (name, a.name)
    for extra in o[len(t):]:
        assert extra.default is not inspect.Parameter.empty, (name, extra.name)
