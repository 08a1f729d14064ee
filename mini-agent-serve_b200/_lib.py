"""ctypes binding of libmas_b200.so (the C ABI declared in include/mas_b200.h).

The library is loaded once per process. A missing library is an ImportError that says how to build
it: there is no fallback implementation, by design.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("MAS_B200_LIB", str(_PKG / "libmas_b200.so")))
TORCH_LIB_PATH = _PKG / "libmas_b200_torch.so"

# Dtype codes (MAS_DTYPE_*).
DTYPE_BF16 = 0
DTYPE_FP16 = 1
DTYPE_FP32 = 2
DTYPE_FP8_E4M3 = 3
DTYPE_INT32 = 4
DTYPE_INT64 = 5

# Return codes (MAS_OK / MAS_ERR_*).
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED_DTYPE = -2
ERR_UNSUPPORTED_SHAPE = -3
ERR_NO_DEVICE = -4

# Device status bits (MAS_STATUS_*).
STATUS_EMBED_ID_OUT_OF_RANGE = 1
STATUS_ROPE_POS_OUT_OF_RANGE = 2
STATUS_COPY_TIMEOUT = 4
STATUS_KV_SLOT_OUT_OF_RANGE = 8

_i32, _i64, _f32, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class PagedKVCache(ctypes.Structure):
    """struct MasPagedKVCache (include/mas_b200.h): one layer's paged k/v cache and page table."""

    _fields_ = [("k_cache", _vp), ("v_cache", _vp), ("num_pages", _i64), ("page_size", _i64),
                ("stride_page", _i64), ("stride_entry", _i64), ("stride_head", _i64), ("kv_indices", _vp),
                ("num_indices", _i64), ("kv_indptr", _vp), ("batch_size", _i64)]


_kvp = ctypes.POINTER(PagedKVCache)

# Every exported function with its argument types, in header order.
SIGNATURES: dict[str, tuple[type, list[type]]] = {
    "mas_version": (_i32, []),
    "mas_status_string": (ctypes.c_char_p, [_i32]),
    "mas_prepare_device": (_i32, [_i32]),
    "mas_read_fault_word": (_i32, [_i32, ctypes.POINTER(ctypes.c_int32), _i32]),
    "mas_read_status_word": (_i32, [_i32, ctypes.POINTER(ctypes.c_int32), _i32]),
    "mas_selftest_bounded_wait": (_i32, [_i64, _vp]),
    "mas_fused_add_rmsnorm": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _vp]),
    "mas_fused_add_rmsnorm_quant": (
        _i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _vp]),
    "mas_silu_and_mul": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "mas_silu_and_mul_quant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _vp]),
    "mas_rope_cos_sin_cache_inplace": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
               _i32, _i32, _vp, _i32, _vp]),
    "mas_rope_cos_sin_cache_q_scale_inplace": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
               _i32, _f32, _i64, _i32, _vp, _i32, _vp]),
    "mas_embedding_gather": (
        _i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _i32, _vp]),
    "mas_embedding_gather_fill_placeholders": (
        _i32, [_vp, _vp, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _i32, _vp]),
    "mas_append_paged_kv_cache": (
        _i32, [_vp, _vp, _vp, _vp, _i32, _kvp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _i32, _vp]),
    "mas_rope_append_paged_kv_cache": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _kvp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
               _i64, _i64, _i64, _i32, _f32, _i64, _i32, _vp, _i32, _vp]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"mas_b200: CUDA library {LIB_PATH} is missing. Build it with "
            f"`python {_PKG / 'build.py'}` (nvcc, sm_100a) or `python -c 'import __graft_entry__ as g; g.build()'`."
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _load_torch_ops() -> None:
    """Registers the `mas_b200::*` operators (C++, over the C ABI) with the torch dispatcher."""
    import torch

    if not TORCH_LIB_PATH.exists():
        raise ImportError(f"mas_b200: operator library {TORCH_LIB_PATH} is missing. Build it with "
                          f"`python {_PKG / 'build.py'}`.")
    torch.ops.load_library(str(TORCH_LIB_PATH))


_load_torch_ops()


class MasError(RuntimeError):
    """A nonzero return code of a C-ABI entry point."""

    def __init__(self, fn: str, code: int):
        self.code = code
        super().__init__(f"{fn} failed with status {code}: {status_string(code)}")


def status_string(code: int) -> str:
    return lib.mas_status_string(code).decode()


def check(fn: str, code: int) -> None:
    if code != OK:
        raise MasError(fn, code)


def version() -> tuple[int, int]:
    v = lib.mas_version()
    return v >> 16, v & 0xFFFF


def prepare_device(device: int) -> None:
    check("mas_prepare_device", lib.mas_prepare_device(device))


def read_fault_word(device: int, clear: bool = False) -> int:
    """The library fault word of `device` (host-synchronising diagnostic)."""
    out = ctypes.c_int32(0)
    check("mas_read_fault_word", lib.mas_read_fault_word(device, ctypes.byref(out), int(clear)))
    return out.value


def read_status_word(device: int, clear: bool = False) -> int:
    """The library status word of `device`: the MAS_STATUS_* data-error bits (host-synchronising)."""
    out = ctypes.c_int32(0)
    check("mas_read_status_word", lib.mas_read_status_word(device, ctypes.byref(out), int(clear)))
    return out.value
