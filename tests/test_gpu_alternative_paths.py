"""The non-default kernels of each op, through the same parity tests as the defaults.

Each op picks among several kernels by shape and step size (and the choice can be forced from the
environment, read once per process: MAS_NORM_IMPL, MAS_NORM_STAGES, MAS_NORM_KEEP_THREADS, MAS_ROPE_IMPL,
MAS_ROPE_PREFETCH_QK, MAS_SILU_IMPL, MAS_SILU_NOALLOC,
MAS_EMBED_IMPL).
A choice the default shapes never reach would otherwise go untested, so every forced choice reruns
its op's test files in a child process with the variable set.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

TESTS = Path(__file__).resolve().parent

CASES = {
    "norm-loop": ({"MAS_NORM_IMPL": "loop"}, ["test_gpu_norm.py"]),
    "norm-loopreg-3stages": ({"MAS_NORM_IMPL": "loopreg", "MAS_NORM_STAGES": "3"}, ["test_gpu_norm.py"]),
    "norm-row": ({"MAS_NORM_IMPL": "row"}, ["test_gpu_norm.py"]),
    "norm-rowreg": ({"MAS_NORM_IMPL": "rowreg"}, ["test_gpu_norm.py"]),
    "norm-rowreg-256": ({"MAS_NORM_IMPL": "rowreg", "MAS_NORM_KEEP_THREADS": "256"}, ["test_gpu_norm.py"]),
    "norm-rowreg-512": ({"MAS_NORM_IMPL": "rowreg", "MAS_NORM_KEEP_THREADS": "512"}, ["test_gpu_norm.py"]),
    "norm-ring": ({"MAS_NORM_IMPL": "ring", "MAS_NORM_STAGES": "3"}, ["test_gpu_norm.py"]),
    "rope-ring": ({"MAS_ROPE_IMPL": "ring"}, ["test_gpu_rope.py", "test_gpu_llama4.py"]),
    "rope-ring-no-prefetch": ({"MAS_ROPE_IMPL": "ring", "MAS_ROPE_PREFETCH_QK": "0"},
                              ["test_gpu_rope.py", "test_gpu_paged_kv.py"]),
    "rope-vec": ({"MAS_ROPE_IMPL": "vec"}, ["test_gpu_rope.py", "test_gpu_llama4.py"]),
    "silu-ring": ({"MAS_SILU_IMPL": "ring"}, ["test_gpu_silu.py", "test_gpu_silu_quant.py"]),
    "silu-loads-noalloc": ({"MAS_SILU_NOALLOC": "1"}, ["test_gpu_silu.py", "test_gpu_silu_quant.py"]),
    "silu-loads-plain": ({"MAS_SILU_NOALLOC": "0"}, ["test_gpu_silu.py", "test_gpu_silu_quant.py"]),
    "embed-tma": ({"MAS_EMBED_IMPL": "tma"}, ["test_gpu_embed.py"]),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_forced_kernel_passes_its_op_tests(case):
    env_vars, files = CASES[case]
    env = dict(os.environ, **env_vars)
    cmd = [sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
           *[str(TESTS / f) for f in files]]
    r = subprocess.run(cmd, env=env, cwd=TESTS.parent, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, f"{case}: {env_vars}\n{r.stdout[-3000:]}\n{r.stderr[-2000:]}"
