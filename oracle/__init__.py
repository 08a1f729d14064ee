"""CPU oracle of the per-token layer ops -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import this package, and
only as the checker (or the timed CPU baseline). The product package never imports it.

The arithmetic lives in oracle.c (a C restatement of flashinfer 0.6.11.post2's kernels, each function
citing the source it follows), compiled by `build()` with gcc into liborc.so next to this file. This
module exposes it with the call style of the product ops (CPU tensors instead of CUDA tensors), so
parity tests read like the reference's own call sites.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
SRC = HERE / "oracle.c"
LIB_PATH = HERE / "liborc.so"

BF16, FP16, INT32, INT64 = 0, 1, 4, 5
_ACT = {torch.bfloat16: BF16, torch.float16: FP16}
_IDS = {torch.int32: INT32, torch.int64: INT64}


def _compilers() -> list[str]:
    cands = [os.environ.get("CC"), "/usr/bin/gcc", shutil.which("gcc"), shutil.which("cc")]
    return [c for i, c in enumerate(cands) if c and Path(c).exists() and c not in cands[:i]]


def build(force: bool = False) -> Path:
    """gcc -O2 -fopenmp -ffp-contract=off oracle.c -> liborc.so (skipped when up to date).

    Falls back to a single-threaded build when no compiler on this machine has OpenMP.
    """
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    base = ["-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"]
    errors = []
    for omp in (["-fopenmp"], []):
        for cc in _compilers():
            r = subprocess.run([cc, *omp, *base], capture_output=True, text=True)
            if r.returncode == 0:
                os.replace(tmp, LIB_PATH)
                return LIB_PATH
            errors.append(f"{cc} {' '.join(omp)}: {r.stderr.strip()[:300]}")
    raise RuntimeError("oracle build failed:\n" + "\n".join(errors))


_lib = None
_i32, _i64, _f32, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
_SIGS = {
    "orc_fused_add_rmsnorm": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32]),
    "orc_fused_add_rmsnorm_quant": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32]),
    "orc_silu_and_mul": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i32]),
    "orc_silu_and_mul_quant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32]),
    "orc_rope_cos_sin_cache_inplace": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp]),
    "orc_rope_cos_sin_cache_q_scale_inplace": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _f32, _i64,
               _i32, _vp]),
    "orc_append_paged_kv_cache": (
        _i32, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i64, _i64,
               _i64, _i64, _i64, _i64, _i64, _vp]),
    "orc_rope_append_paged_kv_cache": (
        _i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _i64,
               _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _f32, _i64, _i32, _vp]),
    "orc_embedding_gather": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "orc_embedding_gather_fill_placeholders": (
        _i32, [_vp, _vp, _vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "orc_f32_to_e4m3": (ctypes.c_uint8, [_f32]),
    "orc_e4m3_to_f32": (_f32, [ctypes.c_uint8]),
    "orc_f32_to_bf16": (ctypes.c_uint16, [_f32]),
    "orc_bf16_to_f32": (_f32, [ctypes.c_uint16]),
    "orc_f32_to_f16": (ctypes.c_uint16, [_f32]),
    "orc_set_num_threads": (None, [_i32]),
    "orc_get_num_threads": (_i32, []),
}


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return lib().orc_get_num_threads()


def _cpu(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cpu":
        raise ValueError(f"oracle: {name} must be a CPU tensor")


def _rows(t: torch.Tensor) -> torch.Tensor:
    return t.view(1, -1) if t.dim() == 1 else t.view(-1, t.shape[-1])


def _ok(rc: int, fn: str) -> None:
    if rc != 0:
        raise ValueError(f"oracle {fn}: invalid arguments")


def fused_add_rmsnorm(input: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> None:
    for n, t in (("input", input), ("residual", residual), ("weight", weight)):
        _cpu(t, n)
    x, r = _rows(input), _rows(residual)
    _ok(lib().orc_fused_add_rmsnorm(x.data_ptr(), r.data_ptr(), weight.data_ptr(), x.shape[0], x.shape[1],
                                    x.stride(0), r.stride(0), float(eps), _ACT[x.dtype]), "fused_add_rmsnorm")


def fused_add_rmsnorm_quant(out: torch.Tensor, input: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                            scale: float, eps: float = 1e-6) -> None:
    for n, t in (("out", out), ("input", input), ("residual", residual), ("weight", weight)):
        _cpu(t, n)
    o, x, r = _rows(out), _rows(input), _rows(residual)
    s = torch.tensor([float(scale)], dtype=torch.float32)
    _ok(lib().orc_fused_add_rmsnorm_quant(o.data_ptr(), x.data_ptr(), r.data_ptr(), weight.data_ptr(), s.data_ptr(),
                                          x.shape[0], x.shape[1], o.stride(0), x.stride(0), r.stride(0), float(eps),
                                          _ACT[x.dtype]), "fused_add_rmsnorm_quant")


def silu_and_mul(input: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _cpu(input, "input")
    d = input.shape[-1] // 2
    if out is None:
        out = torch.empty(input.shape[:-1] + (d,), dtype=input.dtype)
    x, o = _rows(input), _rows(out)
    _ok(lib().orc_silu_and_mul(o.data_ptr(), x.data_ptr(), x.shape[0], d, o.stride(0), x.stride(0), _ACT[x.dtype]),
        "silu_and_mul")
    return out


def silu_and_mul_quant(input: torch.Tensor, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu_and_mul then quantize_fp8 with `scale`: e4m3 bytes as a torch.float8_e4m3fn tensor."""
    _cpu(input, "input")
    d = input.shape[-1] // 2
    if out is None:
        out = torch.empty(input.shape[:-1] + (d,), dtype=torch.float8_e4m3fn)
    x, o = _rows(input), _rows(out)
    s = torch.tensor([float(scale)], dtype=torch.float32)
    _ok(lib().orc_silu_and_mul_quant(o.data_ptr(), x.data_ptr(), s.data_ptr(), x.shape[0], d, o.stride(0),
                                     x.stride(0), _ACT[x.dtype]), "silu_and_mul_quant")
    return out


def apply_rope_with_cos_sin_cache_inplace(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                                          head_size: int, cos_sin_cache: torch.Tensor, is_neox: bool = True) -> int:
    """In place on CPU q/k; returns the status bits (2 = a position out of range)."""
    for n, t in (("positions", positions), ("query", query), ("key", key), ("cos_sin_cache", cos_sin_cache)):
        _cpu(t, n)
    cache = cos_sin_cache.contiguous()
    q = query.view(query.shape[0], -1, head_size)
    k = key.view(key.shape[0], -1, head_size)
    st = ctypes.c_int32(0)
    _ok(lib().orc_rope_cos_sin_cache_inplace(
        positions.data_ptr(), _IDS[positions.dtype], q.data_ptr(), k.data_ptr(), cache.data_ptr(), q.shape[0],
        q.shape[1], k.shape[1], head_size, cache.shape[1], cache.shape[0], q.stride(0), q.stride(1), k.stride(0),
        k.stride(1), int(bool(is_neox)), _ACT[q.dtype], ctypes.byref(st)), "rope")
    return st.value


def apply_rope_and_llama4_query_scale_inplace(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                                              head_size: int, cos_sin_cache: torch.Tensor, beta: float,
                                              original_max_position_embeddings: int, is_neox: bool = True) -> int:
    """Rope then the llama-4 query scale, in place on CPU q/k; returns the status bits."""
    for n, t in (("positions", positions), ("query", query), ("key", key), ("cos_sin_cache", cos_sin_cache)):
        _cpu(t, n)
    cache = cos_sin_cache.contiguous()
    q = query.view(query.shape[0], -1, head_size)
    k = key.view(key.shape[0], -1, head_size)
    st = ctypes.c_int32(0)
    _ok(lib().orc_rope_cos_sin_cache_q_scale_inplace(
        positions.data_ptr(), _IDS[positions.dtype], q.data_ptr(), k.data_ptr(), cache.data_ptr(), q.shape[0],
        q.shape[1], k.shape[1], head_size, cache.shape[1], cache.shape[0], q.stride(0), q.stride(1), k.stride(0),
        k.stride(1), int(bool(is_neox)), float(beta), int(original_max_position_embeddings), _ACT[q.dtype],
        ctypes.byref(st)), "rope_q_scale")
    return st.value


def _paged(k_cache: torch.Tensor, v_cache: torch.Tensor, kv_layout: str):
    """(num_pages, page_size, stride_page, stride_entry, stride_head) of a 4-D NHD / HND cache."""
    if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("oracle: k and v caches must share shape and strides")
    if kv_layout == "NHD":
        return k_cache.shape[0], k_cache.shape[1], k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
    return k_cache.shape[0], k_cache.shape[2], k_cache.stride(0), k_cache.stride(2), k_cache.stride(1)


def append_paged_kv_cache(append_key: torch.Tensor, append_value: torch.Tensor, batch_indices: torch.Tensor,
                          positions: torch.Tensor, paged_kv_cache, kv_indices: torch.Tensor,
                          kv_indptr: torch.Tensor, kv_layout: str = "NHD") -> int:
    """Appends (T, Hkv, D) k/v rows to the CPU caches in place; returns the status bits (8 = a slot
    out of range)."""
    k_cache, v_cache = paged_kv_cache
    for n, t in (("append_key", append_key), ("append_value", append_value), ("batch_indices", batch_indices),
                 ("positions", positions), ("k_cache", k_cache), ("v_cache", v_cache),
                 ("kv_indices", kv_indices), ("kv_indptr", kv_indptr)):
        _cpu(t, n)
    bi, ki, kp = (x.to(torch.int32).contiguous() for x in (batch_indices, kv_indices, kv_indptr))
    pos = positions.contiguous()
    P, S, sp, se, sh = _paged(k_cache, v_cache, kv_layout)
    st = ctypes.c_int32(0)
    _ok(lib().orc_append_paged_kv_cache(
        append_key.data_ptr(), append_value.data_ptr(), bi.data_ptr(), pos.data_ptr(), _IDS[pos.dtype],
        k_cache.data_ptr(), v_cache.data_ptr(), P, S, sp, se, sh, ki.data_ptr(), ki.numel(), kp.data_ptr(),
        kp.numel() - 1, append_key.shape[0], append_key.shape[1], append_key.shape[2], append_key.stride(0),
        append_key.stride(1), append_value.stride(0), append_value.stride(1), ctypes.byref(st)), "append")
    return st.value


def rope_append_paged_kv_cache(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                               value: torch.Tensor, head_size: int, cos_sin_cache: torch.Tensor,
                               batch_indices: torch.Tensor, paged_kv_cache, kv_indices: torch.Tensor,
                               kv_indptr: torch.Tensor, is_neox: bool = True, kv_layout: str = "NHD",
                               beta: float = 0.0, original_max_position_embeddings: int = 1) -> int:
    """Rope on CPU q/k in place, the paged append of k and v, then (beta != 0) the llama-4 query scale.
    query/key: (T, H*D) or (T, H, D) views; value (T, Hkv, D). Returns the status bits."""
    k_cache, v_cache = paged_kv_cache
    cache = cos_sin_cache.contiguous()
    T = query.shape[0]
    q = query.view(T, -1, head_size)
    k = key.view(T, -1, head_size)
    v = value.view(T, -1, head_size)
    bi, ki, kp = (x.to(torch.int32).contiguous() for x in (batch_indices, kv_indices, kv_indptr))
    pos = positions.contiguous()
    P, S, sp, se, sh = _paged(k_cache, v_cache, kv_layout)
    st = ctypes.c_int32(0)
    _ok(lib().orc_rope_append_paged_kv_cache(
        pos.data_ptr(), _IDS[pos.dtype], q.data_ptr(), k.data_ptr(), v.data_ptr(), cache.data_ptr(), bi.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), P, S, sp, se, sh, ki.data_ptr(), ki.numel(), kp.data_ptr(),
        kp.numel() - 1, T, q.shape[1], k.shape[1], head_size, cache.shape[1], cache.shape[0], q.stride(0),
        q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1), int(bool(is_neox)), float(beta),
        int(original_max_position_embeddings), _ACT[q.dtype], ctypes.byref(st)), "rope_append")
    return st.value


def embedding(input_ids: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, int]:
    """(weight[input_ids] with zero rows for out-of-range ids, status bits (1 = an id out of range))."""
    _cpu(input_ids, "input_ids")
    _cpu(weight, "weight")
    ids = input_ids.reshape(-1).contiguous()
    out = torch.empty(tuple(input_ids.shape) + (weight.shape[1],), dtype=weight.dtype)
    st = ctypes.c_int32(0)
    _ok(lib().orc_embedding_gather(out.data_ptr(), weight.data_ptr(), ids.data_ptr(), _IDS[ids.dtype], ids.shape[0],
                                   weight.shape[1], weight.shape[0], weight.shape[1], weight.stride(0),
                                   weight.element_size(), ctypes.byref(st)), "embedding")
    return out, st.value


def embedding_fill_placeholders(input_ids: torch.Tensor, weight: torch.Tensor,
                                last_tokens: torch.Tensor) -> tuple[torch.Tensor, int]:
    """fill_placeholders (in place on CPU input_ids) then the gather; returns (rows, status bits)."""
    for n, t in (("input_ids", input_ids), ("weight", weight), ("last_tokens", last_tokens)):
        _cpu(t, n)
    assert input_ids.is_contiguous() and last_tokens.is_contiguous()
    out = torch.empty(tuple(input_ids.shape) + (weight.shape[1],), dtype=weight.dtype)
    st = ctypes.c_int32(0)
    _ok(lib().orc_embedding_gather_fill_placeholders(
        out.data_ptr(), weight.data_ptr(), input_ids.data_ptr(), _IDS[input_ids.dtype], last_tokens.data_ptr(),
        _IDS[last_tokens.dtype], last_tokens.numel(), input_ids.numel(), weight.shape[1], weight.shape[0],
        weight.shape[1], weight.stride(0), weight.element_size(), ctypes.byref(st)), "embedding_fill")
    return out, st.value


def f32_to_e4m3(x: float) -> int:
    return lib().orc_f32_to_e4m3(float(x))


def e4m3_to_f32(b: int) -> float:
    return lib().orc_e4m3_to_f32(int(b))


def f32_to_bf16_bits(x: float) -> int:
    return lib().orc_f32_to_bf16(float(x))


def f32_to_f16_bits(x: float) -> int:
    return lib().orc_f32_to_f16(float(x))
