"""The C-ABI library without a GPU: it loads, exports exactly what include/mas_b200.h declares, and
rejects bad arguments before touching CUDA (these calls never launch anything).
"""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import mas_b200
from mas_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mas_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"MAS_API\s+[\w\s\*]+?\b(mas_\w+)\s*\(", text)


def declared_constants() -> dict[str, int]:
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+(MAS_\w+)\s+\(?(-?\d+)\)?", HEADER.read_text())}


def test_header_declares_the_expected_entry_points():
    fns = declared_functions()
    for name in ("mas_fused_add_rmsnorm", "mas_fused_add_rmsnorm_quant", "mas_silu_and_mul",
                 "mas_rope_cos_sin_cache_inplace", "mas_embedding_gather", "mas_prepare_device",
                 "mas_status_string", "mas_version", "mas_read_fault_word", "mas_read_status_word"):
        assert name in fns, name


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert exported == set(declared_functions()), exported ^ set(declared_functions())


def test_ctypes_signatures_cover_the_header():
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_python_constants_match_header():
    c = declared_constants()
    assert c["MAS_DTYPE_BF16"] == _lib.DTYPE_BF16 and c["MAS_DTYPE_FP16"] == _lib.DTYPE_FP16
    assert c["MAS_DTYPE_FP8_E4M3"] == _lib.DTYPE_FP8_E4M3
    assert c["MAS_DTYPE_INT32"] == _lib.DTYPE_INT32 and c["MAS_DTYPE_INT64"] == _lib.DTYPE_INT64
    assert c["MAS_ERR_INVALID_ARGUMENT"] == _lib.ERR_INVALID_ARGUMENT
    assert c["MAS_ERR_UNSUPPORTED_DTYPE"] == _lib.ERR_UNSUPPORTED_DTYPE
    assert c["MAS_ERR_UNSUPPORTED_SHAPE"] == _lib.ERR_UNSUPPORTED_SHAPE
    assert c["MAS_ERR_NO_DEVICE"] == _lib.ERR_NO_DEVICE
    assert c["MAS_STATUS_EMBED_ID_OUT_OF_RANGE"] == _lib.STATUS_EMBED_ID_OUT_OF_RANGE
    assert c["MAS_STATUS_ROPE_POS_OUT_OF_RANGE"] == _lib.STATUS_ROPE_POS_OUT_OF_RANGE
    assert c["MAS_STATUS_COPY_TIMEOUT"] == _lib.STATUS_COPY_TIMEOUT
    assert c["MAS_STATUS_KV_SLOT_OUT_OF_RANGE"] == _lib.STATUS_KV_SLOT_OUT_OF_RANGE


def test_paged_kv_struct_layout_matches_header():
    """struct MasPagedKVCache: two pointers, five int64, pointer, int64, pointer, int64 (88 bytes)."""
    text = HEADER.read_text()
    body = re.search(r"typedef struct MasPagedKVCache \{(.*?)\} MasPagedKVCache;", text, re.S).group(1)
    fields = re.findall(r"(\w+);", body)
    assert fields == [f for f, _ in _lib.PagedKVCache._fields_]
    assert ctypes.sizeof(_lib.PagedKVCache) == 88


def test_version_and_status_strings():
    assert mas_b200.version() == (0, 1)
    assert mas_b200.status_string(0) == "ok"
    for code in (-1, -2, -3, -4):
        assert mas_b200.status_string(code) and "unknown" not in mas_b200.status_string(code)
    assert "unknown" in mas_b200.status_string(-99)


L = _lib.lib
P = 0x1000  # a non-null pointer value; argument checks reject before any dereference or CUDA call


def _kv(page_size=16):
    c = _lib.PagedKVCache(k_cache=P, v_cache=P, num_pages=4, page_size=page_size, stride_page=16 * 64,
                          stride_entry=64, stride_head=64, kv_indices=P, num_indices=4, kv_indptr=P, batch_size=1)
    return ctypes.byref(c)


@pytest.mark.parametrize("call,code", [
    (lambda: L.mas_fused_add_rmsnorm(P, P, P, -1, 8, 8, 8, 1e-5, 0, 0, None), -1),
    (lambda: L.mas_fused_add_rmsnorm(P, P, P, 2, 0, 8, 8, 1e-5, 0, 0, None), -1),
    (lambda: L.mas_fused_add_rmsnorm(P, P, P, 2, 8, 7, 8, 1e-5, 0, 0, None), -1),
    (lambda: L.mas_fused_add_rmsnorm(None, P, P, 2, 8, 8, 8, 1e-5, 0, 0, None), -1),
    (lambda: L.mas_fused_add_rmsnorm(P, P, P, 2, 8, 8, 8, 1e-5, 9, 0, None), -2),
    (lambda: L.mas_fused_add_rmsnorm_quant(P, P, P, P, P, 2, 8, 8, 8, 8, 1e-5, 0, 0, 0, None), -2),
    (lambda: L.mas_fused_add_rmsnorm_quant(P, P, P, P, None, 2, 8, 8, 8, 8, 1e-5, 0, 3, 0, None), -1),
    (lambda: L.mas_selftest_bounded_wait(0, None), -1),
    (lambda: L.mas_selftest_bounded_wait(3_000_000_000, None), -1),
    (lambda: L.mas_silu_and_mul(P, P, 2, 8, 8, 15, 0, 0, None), -1),
    (lambda: L.mas_silu_and_mul(P, P, 2, 8, 7, 16, 0, 0, None), -1),
    (lambda: L.mas_silu_and_mul(P, P, 2, 8, 8, 16, 2, 0, None), -2),
    (lambda: L.mas_rope_cos_sin_cache_inplace(P, 4, P, P, P, 2, 2, 1, 128, 129, 10, 0, 0, 0, 0, 1, 0, None, 0, None), -3),
    (lambda: L.mas_rope_cos_sin_cache_inplace(P, 4, P, P, P, 2, 2, 1, 128, 127, 10, 0, 0, 0, 0, 1, 0, None, 0, None), -3),
    (lambda: L.mas_rope_cos_sin_cache_inplace(P, 7, P, P, P, 2, 2, 1, 128, 128, 10, 0, 0, 0, 0, 1, 0, None, 0, None), -2),
    (lambda: L.mas_rope_cos_sin_cache_inplace(P, 4, None, P, P, 2, 2, 1, 128, 128, 10, 0, 0, 0, 0, 1, 0, None, 0, None), -1),
    (lambda: L.mas_embedding_gather(P, P, P, 4, 2, 8, 10, 8, 8, 3, None, 0, None), -2),
    (lambda: L.mas_embedding_gather(P, P, P, 6, 2, 8, 10, 8, 8, 2, None, 0, None), -2),
    (lambda: L.mas_embedding_gather(P, P, P, 4, 2, 8, 10, 4, 8, 2, None, 0, None), -1),
    (lambda: L.mas_embedding_gather(P, None, P, 4, 2, 8, 10, 8, 8, 2, None, 0, None), -1),
    (lambda: L.mas_append_paged_kv_cache(P, P, P, P, 4, None, 2, 1, 64, 64, 64, 64, 64, 0, None, 0, None), -1),
    (lambda: L.mas_append_paged_kv_cache(P, P, P, P, 4, _kv(page_size=0), 2, 1, 64, 64, 64, 64, 64, 0, None, 0,
                                         None), -1),
    (lambda: L.mas_append_paged_kv_cache(P, P, P, P, 4, _kv(), 2, 1, 64, 64, 64, 64, 64, 3, None, 0, None), -2),
    (lambda: L.mas_append_paged_kv_cache(P, P, P, P, 9, _kv(), 2, 1, 64, 64, 64, 64, 64, 0, None, 0, None), -2),
    (lambda: L.mas_append_paged_kv_cache(P, P, None, P, 4, _kv(), 2, 1, 64, 64, 64, 64, 64, 0, None, 0, None), -1),
    (lambda: L.mas_rope_append_paged_kv_cache(P, 4, P, P, P, P, P, None, 2, 2, 1, 64, 64, 10, 0, 0, 0, 0, 0, 0, 1,
                                              0.0, 1, 0, None, 0, None), -1),
    (lambda: L.mas_rope_append_paged_kv_cache(P, 4, P, P, None, P, P, _kv(), 2, 2, 1, 64, 64, 10, 0, 0, 0, 0, 0, 0,
                                              1, 0.0, 1, 0, None, 0, None), -1),
    (lambda: L.mas_rope_append_paged_kv_cache(P, 4, P, P, P, P, P, _kv(), 2, 2, 1, 64, 65, 10, 0, 0, 0, 0, 0, 0, 1,
                                              0.0, 1, 0, None, 0, None), -3),
    (lambda: L.mas_rope_append_paged_kv_cache(P, 4, P, P, P, P, P, _kv(), 2, 2, 1, 64, 64, 10, 0, 0, 0, 0, 0, 0, 1,
                                              0.5, 0, 0, None, 0, None), -1),
])
def test_argument_checks_reject_before_launch(call, code):
    assert call() == code


def test_empty_batches_are_no_ops_without_a_device():
    # zero tokens returns success before any device query, even with no GPU present
    assert L.mas_fused_add_rmsnorm(None, None, None, 0, 8, 8, 8, 1e-5, 0, 0, None) == 0
    assert L.mas_silu_and_mul(None, None, 0, 8, 8, 16, 0, 0, None) == 0
    assert L.mas_embedding_gather(None, None, None, 4, 0, 8, 10, 8, 8, 2, None, 0, None) == 0
    assert L.mas_rope_cos_sin_cache_inplace(None, 4, None, None, None, 0, 2, 1, 128, 128, 10, 0, 0, 0, 0, 1, 0,
                                            None, 0, None) == 0
    assert L.mas_append_paged_kv_cache(None, None, None, None, 4, _kv(), 0, 1, 64, 64, 64, 64, 64, 0, None, 0,
                                       None) == 0
    assert L.mas_rope_append_paged_kv_cache(None, 4, None, None, None, None, None, _kv(), 0, 2, 1, 64, 64, 10, 0, 0,
                                            0, 0, 0, 0, 1, 0.0, 1, 0, None, 0, None) == 0


def test_valid_call_without_gpu_reports_no_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert L.mas_silu_and_mul(P, P, 2, 8, 8, 16, 0, 0, None) == _lib.ERR_NO_DEVICE
    with pytest.raises(mas_b200.MasError):
        _lib.check("mas_silu_and_mul", L.mas_silu_and_mul(P, P, 2, 8, 8, 16, 0, 0, None))
