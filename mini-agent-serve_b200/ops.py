"""Drop-in per-token layer ops for mini-agent-serve's Devstral 2 model, on the B200 CUDA kernels.

The public functions keep the names, signatures, argument meaning and error behaviour of the
flashinfer 0.6.11.post2 functions that miniagentserve/models/devstral2/devstral2.py imports
(devstral2.py:18-23), so the module forwards call them unchanged:

    fused_add_rmsnorm          FI/norm/__init__.py:236-274         devstral2.py:305-307
    fused_add_rmsnorm_quant    FI/norm/__init__.py:288-344         devstral2.py:241-252
    silu_and_mul               FI/activation.py:77-118             devstral2.py:223-224
    apply_rope_with_cos_sin_cache_inplace  FI/rope.py:1223-1272    devstral2.py:163-166
    append_paged_kv_cache      FI/page.py:280-406                  devstral2.py:170-173

plus the token-embedding gather behind nn.Embedding (devstral2.py:260, :282), as `embedding` and the
`Embedding` module (embedding.py). Four fused forms, each one launch where the reference makes
several, are additions: silu_and_mul_quant (SiLU-mul then FP8Linear's quantisation),
apply_rope_and_llama4_query_scale_inplace, apply_rope_and_append_paged_kv_cache (rope, the paged
append and optionally the query scale) and embedding_fill_placeholders (the runner's placeholder
substitution then the gather).

Each function is a thin Python check layer (raising flashinfer's exception types) over a
`mas_b200::*` torch operator. The operators are defined and implemented in C++
(csrc/torch_ops.cpp, loaded by _lib) over the C ABI of libmas_b200.so (include/mas_b200.h) and launch
on the current stream; their fake kernels, registered here, make them opaque nodes under
torch.compile (mirroring flashinfer's register_custom_op/register_fake_op, FI/activation.py:48-58).
There is no CPU implementation: the operators are registered for CUDA only, and the libraries must
be present.
"""
from __future__ import annotations

import warnings
from typing import Optional, Union

import torch

from . import _lib

__all__ = [
    "fused_add_rmsnorm",
    "fused_add_rmsnorm_quant",
    "silu_and_mul",
    "silu_and_mul_quant",
    "apply_rope_with_cos_sin_cache_inplace",
    "apply_rope_and_llama4_query_scale_inplace",
    "append_paged_kv_cache",
    "apply_rope_and_append_paged_kv_cache",
    "embedding",
    "embedding_out",
    "embedding_fill_placeholders",
    "read_status",
]

FP8 = torch.float8_e4m3fn

_ACT_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_FP16}
_ID_DTYPES = {torch.int32: _lib.DTYPE_INT32, torch.int64: _lib.DTYPE_INT64}


def _check_device(ref: torch.Tensor, **tensors: Optional[torch.Tensor]) -> None:
    """Every tensor argument on `ref`'s device, as aten and flashinfer require: a kernel handed a host
    tensor would be given a host pointer. Raises RuntimeError, as torch does for the same mistake."""
    for name, t in tensors.items():
        if t is not None and t.device != ref.device:
            raise RuntimeError(f"Expected all tensors to be on the same device, but {name} is on {t.device} "
                               f"and the other operands on {ref.device}")


def _act_code(t: torch.Tensor) -> int:
    try:
        return _ACT_DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected bfloat16 or float16") from None


# ------------------------------------------------------------------------------------------------
# Device status word (out-of-range ids, positions and paged-KV slots), one int32 per device.
# ------------------------------------------------------------------------------------------------
def read_status(device: Union[int, torch.device, None] = None, clear: bool = True) -> int:
    """The MAS_STATUS_* bits the gather, rope and paged-append kernels have raised on `device` since it
    was last cleared, then (by default) clears them. This synchronises the host with the device.

    The word lives in the library (one per device), so every launch reports into it: eager calls,
    calls traced by torch.compile and launches replayed from a CUDA graph alike.
    """
    if device is None:
        idx = torch.cuda.current_device()
    else:
        dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
    return _lib.read_status_word(idx, clear)


# ------------------------------------------------------------------------------------------------
# Fused add RMSNorm.
# ------------------------------------------------------------------------------------------------
@torch.library.register_fake("mas_b200::fused_add_rmsnorm")
def _(input, residual, weight, eps, enable_pdl) -> None:
    return None


_OP_NORM = torch.ops.mas_b200.fused_add_rmsnorm.default
_OP_NORM_QUANT = torch.ops.mas_b200.fused_add_rmsnorm_quant.default
_OP_SILU = torch.ops.mas_b200.silu_and_mul.default
_OP_SILU_QUANT = torch.ops.mas_b200.silu_and_mul_quant.default
_OP_ROPE = torch.ops.mas_b200.apply_rope_pos_ids_cos_sin_cache.default
_OP_ROPE_QS = torch.ops.mas_b200.apply_rope_q_scale.default
_OP_APPEND = torch.ops.mas_b200.append_paged_kv_cache.default
_OP_ROPE_APPEND = torch.ops.mas_b200.rope_append_paged_kv_cache.default
_OP_EMBED = torch.ops.mas_b200.embedding.default
_OP_EMBED_OUT = torch.ops.mas_b200.embedding_out.default
_OP_EMBED_FILL = torch.ops.mas_b200.embedding_fill.default


def _check_norm(input: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor) -> None:
    if input.shape != residual.shape:
        raise ValueError(f"input {tuple(input.shape)} and residual {tuple(residual.shape)} differ")
    if input.dtype != residual.dtype or weight.dtype != input.dtype:
        raise ValueError("input, residual and weight must share one dtype")
    if weight.dim() != 1 or weight.shape[0] != input.shape[-1] or not weight.is_contiguous():
        raise ValueError(f"weight must be a contiguous ({input.shape[-1]},) tensor")
    _act_code(input)


def fused_add_rmsnorm(input: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                      enable_pdl: Optional[bool] = None) -> None:
    r"""Fused add root mean square normalization, in place.

    ``residual[i] += input[i]`` then ``input[i] = (residual[i] / RMS(residual)) * weight[i]``, with the
    sum kept in fp32 and the norm taken over the unrounded sum (as flashinfer does).
    Same signature and meaning as flashinfer.norm.fused_add_rmsnorm (FI/norm/__init__.py:236-274).
    """
    _check_norm(input, residual, weight)
    _check_device(input, residual=residual, weight=weight)
    _OP_NORM(input, residual, weight, float(eps), True if enable_pdl is None else bool(enable_pdl))


def _normalize_scale(scale: Union[float, torch.Tensor], ref: torch.Tensor) -> torch.Tensor:
    """Scale as a (1,) fp32 tensor on `ref`'s device (FI/norm/__init__.py:84-108)."""
    if not isinstance(scale, torch.Tensor):
        warnings.warn("Passing scale as a float is deprecated; pass a torch.Tensor of shape (1,)",
                      FutureWarning, stacklevel=3)
        scale = torch.tensor([scale], dtype=torch.float32, device=ref.device)
    if scale.device != ref.device:
        scale = scale.to(ref.device)
    if scale.dtype != torch.float32:
        scale = scale.to(torch.float32)
    if scale.ndim == 0:
        scale = scale.view(1)
    elif not (scale.ndim == 1 and scale.numel() == 1):
        raise ValueError(f"scale must be a scalar tensor or shape (1,), got shape {tuple(scale.shape)}")
    return scale.contiguous()


@torch.library.register_fake("mas_b200::fused_add_rmsnorm_quant")
def _(out, input, residual, weight, scale, eps, enable_pdl) -> None:
    return None


def fused_add_rmsnorm_quant(out: torch.Tensor, input: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                            scale: Union[float, torch.Tensor], eps: float = 1e-6,
                            enable_pdl: Optional[bool] = None) -> None:
    r"""Fused add root mean square normalization + fp8 (e4m3) quantisation.

    ``residual[i] += input[i]`` then ``out[i] = fp8(clamp(residual[i] / RMS(residual) * weight[i] / scale,
    -448, 448))``; `input` is left unchanged. Same signature and meaning as
    flashinfer.norm.fused_add_rmsnorm_quant (FI/norm/__init__.py:288-344).
    """
    _check_norm(input, residual, weight)
    if out.dtype != FP8:
        raise ValueError(f"out must be {FP8}, got {out.dtype}")
    if out.shape != input.shape:
        raise ValueError(f"out {tuple(out.shape)} and input {tuple(input.shape)} differ")
    _check_device(input, out=out, residual=residual, weight=weight)
    scale = _normalize_scale(scale, input)
    _OP_NORM_QUANT(out, input, residual, weight, scale, float(eps), True if enable_pdl is None else bool(enable_pdl))


# ------------------------------------------------------------------------------------------------
# SiLU and mul.
# ------------------------------------------------------------------------------------------------
@torch.library.register_fake("mas_b200::silu_and_mul")
def _(out, input, enable_pdl) -> None:
    return None


def _check_shape(input: torch.Tensor, output: torch.Tensor) -> None:
    """Shape agreement of input and out (FI/activation.py:65-74)."""
    assert input.ndim == output.ndim, f"{input.ndim} != {output.ndim}"
    assert input.shape[:-1] == output.shape[:-1], f"{input.shape[:-1]} != {output.shape[:-1]}"
    assert input.shape[-1] == 2 * output.shape[-1], f"{input.shape[-1]} != {2 * output.shape[-1]}"


def silu_and_mul(input: torch.Tensor, out: Optional[torch.Tensor] = None,
                 enable_pdl: Optional[bool] = None) -> torch.Tensor:
    r"""Fused SiLU and mul: ``silu(input[..., :d]) * input[..., d:]``.

    Same signature, checks and allocation behaviour as flashinfer.activation.silu_and_mul
    (FI/activation.py:77-118): the last dimension must span a multiple of 16 bytes, and `out` is
    allocated with torch.empty when not given.
    """
    if input.shape[-1] * input.dtype.itemsize % 16 != 0:
        raise ValueError("The pointers must be multiple of 16 bytes.")
    if out is not None:
        _check_shape(input, out)
        if out.dtype != input.dtype:
            raise ValueError("out must have the dtype of input")
        _check_device(input, out=out)
    else:
        out = torch.empty(input.shape[:-1] + (input.shape[-1] // 2,), device=input.device, dtype=input.dtype)
    _act_code(input)
    _OP_SILU(out, input, True if enable_pdl is None else bool(enable_pdl))
    return out


@torch.library.register_fake("mas_b200::silu_and_mul_quant")
def _(out, input, scale, enable_pdl) -> None:
    return None


def silu_and_mul_quant(input: torch.Tensor, scale: Union[float, torch.Tensor], out: Optional[torch.Tensor] = None,
                       enable_pdl: Optional[bool] = None) -> torch.Tensor:
    r"""SiLU-and-mul fused with the fp8 (e4m3) activation quantisation of the layer that consumes it.

    Equal, bit for bit, to ``quantize_fp8(silu_and_mul(input), scale)`` -- the pair
    Devstral2MLP.forward -> FP8Linear.forward runs (devstral2.py:224, :110-111, quantize_fp8 at
    :93-95: ``(x / scale).clamp(-448, 448).to(float8_e4m3fn)``) -- in one pass, so the bf16/fp16
    activation is never written. `scale` is FP8Linear's ``activation_scale`` (a 0-dim or (1,) fp32
    tensor). Returns `out`, allocated as float8_e4m3fn when not given.
    """
    if input.shape[-1] * input.dtype.itemsize % 16 != 0:
        raise ValueError("The pointers must be multiple of 16 bytes.")
    if out is not None:
        _check_shape(input, out)
        if out.dtype != FP8:
            raise ValueError(f"out must be {FP8}, got {out.dtype}")
        _check_device(input, out=out)
    else:
        out = torch.empty(input.shape[:-1] + (input.shape[-1] // 2,), device=input.device, dtype=FP8)
    _act_code(input)
    scale = _normalize_scale(scale, input)
    _OP_SILU_QUANT(out, input, scale, True if enable_pdl is None else bool(enable_pdl))
    return out


# ------------------------------------------------------------------------------------------------
# Rotary embedding from the fp32 cos|sin cache.
# ------------------------------------------------------------------------------------------------
def _check_rope(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor, head_size: int,
                cos_sin_cache: torch.Tensor) -> None:
    """flashinfer's checks (FI/rope.py:1260-1261) plus the layout the kernels assume."""
    if cos_sin_cache.dtype != torch.float32:
        raise ValueError("cos_sin_cache should be float32")
    if cos_sin_cache.dim() != 2 or not cos_sin_cache.is_contiguous():
        raise ValueError("cos_sin_cache must be a contiguous (max_seq_len, rotary_dim) tensor")
    if positions.dtype not in _ID_DTYPES:
        raise ValueError(f"positions must be int32 or int64, got {positions.dtype}")
    if query.dtype != key.dtype:
        raise ValueError("query and key must share one dtype")
    rotary_dim = cos_sin_cache.shape[1]
    if rotary_dim % 2 != 0 or rotary_dim > head_size:
        raise ValueError(f"rotary_dim {rotary_dim} must be even and <= head_size {head_size}")
    if query.shape[0] != positions.shape[0] or key.shape[0] != positions.shape[0]:
        raise ValueError("positions, query and key must have the same number of tokens")
    _check_device(query, positions=positions, key=key, cos_sin_cache=cos_sin_cache)


@torch.library.register_fake("mas_b200::apply_rope_pos_ids_cos_sin_cache")
def _(q, k, cos_sin_cache, pos_ids, interleave, enable_pdl) -> None:
    return None


def apply_rope_with_cos_sin_cache_inplace(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                                          head_size: int, cos_sin_cache: torch.Tensor, is_neox: bool = True,
                                          enable_pdl: Optional[bool] = None) -> None:
    r"""Applies rotary embedding to `query` and `key` in place, with cos/sin from `cos_sin_cache`.

    Same signature and meaning as flashinfer.rope.apply_rope_with_cos_sin_cache_inplace
    (FI/rope.py:1223-1272): `query` is ``(nnz, num_q_heads * head_size)`` and `key`
    ``(nnz, num_k_heads * head_size)`` (views of one fused qkv row are fine); `cos_sin_cache` is fp32
    ``(max_seq_len, rotary_dim)``, cos in the first half, sin in the second; ``is_neox`` selects the
    half-rotation (True) or the interleaved pairs (False). A ValueError is raised for a non-fp32
    cache. `enable_pdl` (an addition; the kernels are PDL-safe) defaults to True.
    """
    _check_rope(positions, query, key, head_size, cos_sin_cache)
    if positions.shape[0] == 0:
        return
    q = query.view(query.shape[0], -1, head_size)
    k = key.view(key.shape[0], -1, head_size)
    _OP_ROPE(q, k, cos_sin_cache, positions.contiguous(), not is_neox,
             True if enable_pdl is None else bool(enable_pdl))


@torch.library.register_fake("mas_b200::apply_rope_q_scale")
def _(q, k, cos_sin_cache, pos_ids, interleave, beta, original_max, enable_pdl) -> None:
    return None


def apply_rope_and_llama4_query_scale_inplace(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                                              head_size: int, cos_sin_cache: torch.Tensor, beta: float,
                                              original_max_position_embeddings: int, is_neox: bool = True,
                                              enable_pdl: Optional[bool] = None) -> None:
    r"""Rotary embedding of q and k fused with Devstral 2's llama-4 query scale, in place.

    Equivalent to the two steps of Devstral2Attention.forward (devstral2.py:163-166 and :175-179)::

        apply_rope_with_cos_sin_cache_inplace(positions, query, key, head_size, cos_sin_cache, is_neox)
        scale = 1 + beta * torch.log1p(torch.floor(positions.float() / original_max_position_embeddings))
        query *= scale[:, None].to(query.dtype)

    with the difference that q is scaled in place instead of into a new tensor (the reference does not
    use the unscaled q afterwards). One pass over q instead of three (rope, scale, multiply).
    """
    if original_max_position_embeddings <= 0:
        raise ValueError("original_max_position_embeddings must be positive")
    _check_rope(positions, query, key, head_size, cos_sin_cache)
    if positions.shape[0] == 0:
        return
    q = query.view(query.shape[0], -1, head_size)
    k = key.view(key.shape[0], -1, head_size)
    _OP_ROPE_QS(q, k, cos_sin_cache, positions.contiguous(), not is_neox, float(beta),
                int(original_max_position_embeddings), True if enable_pdl is None else bool(enable_pdl))


# ------------------------------------------------------------------------------------------------
# Paged KV cache append (alone, and fused with rope).
# ------------------------------------------------------------------------------------------------
@torch.library.register_fake("mas_b200::append_paged_kv_cache")
def _(k, v, batch_indices, positions, k_cache, v_cache, kv_indices, kv_indptr, hnd, enable_pdl) -> None:
    return None


@torch.library.register_fake("mas_b200::rope_append_paged_kv_cache")
def _(q, k, v, cos_sin_cache, pos_ids, batch_indices, k_cache, v_cache, kv_indices, kv_indptr, interleave, hnd,
      beta, original_max, enable_pdl) -> None:
    return None


def _unpack_paged_kv_cache(paged_kv_cache, kv_layout: str) -> tuple[torch.Tensor, torch.Tensor]:
    """(k_cache, v_cache) from a tuple of 4-D tensors or one 5-D tensor with k/v on dimension 1
    (FI/page.py:_unpack_paged_kv_cache)."""
    if kv_layout not in ("NHD", "HND"):
        raise KeyError(f"Invalid kv_layout {kv_layout}")
    if isinstance(paged_kv_cache, tuple):
        k_cache, v_cache = paged_kv_cache
    elif torch.is_tensor(paged_kv_cache) and paged_kv_cache.dim() == 5:
        k_cache, v_cache = paged_kv_cache[:, 0], paged_kv_cache[:, 1]
    else:
        raise KeyError("Unrecognized paged_kv_cache type or shape")
    return k_cache, v_cache


def _heads(t: torch.Tensor, head_size: int) -> torch.Tensor:
    """(tokens, heads, head_size) view of a (tokens, heads * head_size) or 3-D tensor."""
    if t.dim() == 3:
        return t
    if t.dim() != 2 or t.shape[-1] % head_size != 0:
        raise ValueError(f"expected (tokens, heads * {head_size}) or (tokens, heads, {head_size}), got {tuple(t.shape)}")
    return t.view(t.shape[0], t.shape[-1] // head_size, head_size)


def _int32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 and t.is_contiguous() else t.int().contiguous()


def _check_paged(k_cache: torch.Tensor, v_cache: torch.Tensor, kv_indptr: torch.Tensor,
                 kv_last_page_len: torch.Tensor, heads: int, head_size: int, kv_layout: str, dtype) -> None:
    if k_cache.dim() != 4 or k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("k/v caches must be 4-D with identical shapes and strides")
    if k_cache.dtype != dtype or v_cache.dtype != dtype:
        raise ValueError(f"k/v caches must be {dtype}")
    cache_heads = k_cache.shape[1] if kv_layout == "HND" else k_cache.shape[2]
    if cache_heads != heads or k_cache.shape[3] != head_size:
        raise ValueError(f"cache heads/head_dim {(cache_heads, k_cache.shape[3])} differ from {(heads, head_size)}")
    if kv_indptr.dim() != 1 or kv_last_page_len.dim() != 1 or kv_indptr.shape[0] != kv_last_page_len.shape[0] + 1:
        raise ValueError("kv_indptr must have batch_size + 1 entries, kv_last_page_len batch_size")


def append_paged_kv_cache(append_key: torch.Tensor, append_value: torch.Tensor, batch_indices: torch.Tensor,
                          positions: torch.Tensor, paged_kv_cache, kv_indices: torch.Tensor, kv_indptr: torch.Tensor,
                          kv_last_page_len: torch.Tensor, kv_layout: str = "NHD",
                          enable_pdl: Optional[bool] = None) -> None:
    r"""Appends each token's k and v rows to the paged KV cache.

    Same signature and meaning as flashinfer.page.append_paged_kv_cache (FI/page.py:280-406), as
    Devstral2Attention.forward calls it (devstral2.py:170-173): token ``i`` of sequence
    ``b = batch_indices[i]`` at ``positions[i]`` is written to entry ``p % page_size`` of page
    ``kv_indices[kv_indptr[b] + p // page_size]`` of `paged_kv_cache` (a ``(k_cache, v_cache)`` tuple or
    one 5-D tensor; layout NHD or HND). `append_key`/`append_value` are ``(nnz, num_kv_heads, head_dim)``
    (strided views of a qkv row are fine). An out-of-range index skips that token and sets
    STATUS_KV_SLOT_OUT_OF_RANGE in the device status word instead of writing out of bounds.
    `enable_pdl` (an addition) defaults to True.
    """
    k_cache, v_cache = _unpack_paged_kv_cache(paged_kv_cache, kv_layout)
    if append_key.dim() != 3 or append_value.shape != append_key.shape:
        raise ValueError("append_key and append_value must be (nnz, num_kv_heads, head_dim) and equal in shape")
    if append_key.dtype != append_value.dtype:
        raise ValueError("append_key and append_value must share one dtype")
    _act_code(append_key)
    nnz, heads, head_size = append_key.shape
    if batch_indices.shape != (nnz,) or positions.shape != (nnz,):
        raise ValueError("batch_indices and positions must have one entry per appended token")
    if positions.dtype not in _ID_DTYPES:
        positions = positions.int()
    _check_paged(k_cache, v_cache, kv_indptr, kv_last_page_len, heads, head_size, kv_layout, append_key.dtype)
    _check_device(append_key, append_value=append_value, batch_indices=batch_indices, positions=positions,
                  k_cache=k_cache, v_cache=v_cache, kv_indices=kv_indices, kv_indptr=kv_indptr)
    if nnz == 0:
        return
    _OP_APPEND(append_key, append_value, _int32(batch_indices), positions.contiguous(), k_cache, v_cache,
               _int32(kv_indices), _int32(kv_indptr), kv_layout == "HND",
               True if enable_pdl is None else bool(enable_pdl))


def apply_rope_and_append_paged_kv_cache(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                                         value: torch.Tensor, head_size: int, cos_sin_cache: torch.Tensor,
                                         batch_indices: torch.Tensor, paged_kv_cache, kv_indices: torch.Tensor,
                                         kv_indptr: torch.Tensor, kv_last_page_len: torch.Tensor,
                                         is_neox: bool = True, kv_layout: str = "NHD",
                                         llama_4_scaling_beta: float = 0.0,
                                         original_max_position_embeddings: int = 1,
                                         enable_pdl: Optional[bool] = None) -> None:
    r"""Rope on q and k, the paged KV append of the rotated k and of v, and (when
    `llama_4_scaling_beta` is nonzero) the llama-4 query scale, in one pass where the layout allows.

    Equivalent to Devstral2Attention.forward's sequence (devstral2.py:163-179)::

        apply_rope_with_cos_sin_cache_inplace(positions, query, key, head_size, cos_sin_cache, is_neox)
        append_paged_kv_cache(key_heads, value_heads, batch_indices, positions, paged_kv_cache,
                              kv_indices, kv_indptr, kv_last_page_len, kv_layout)
        query *= (1 + beta * log1p(floor(positions.float() / original_max))).to(query.dtype)

    with q scaled in place. k and v are read once; the rotated k is written back to `key` as well as
    to the cache. A token whose position lies outside the cos/sin cache is neither rotated nor
    appended (STATUS_ROPE_POS_OUT_OF_RANGE). `query`/`key` are ``(nnz, heads * head_size)`` or
    ``(nnz, heads, head_size)`` views; `value` ``(nnz, num_kv_heads, head_size)`` or flat.
    """
    k_cache, v_cache = _unpack_paged_kv_cache(paged_kv_cache, kv_layout)
    _check_rope(positions, query, key, head_size, cos_sin_cache)
    if value.dtype != query.dtype:
        raise ValueError("query, key and value must share one dtype")
    _act_code(query)
    nnz = positions.shape[0]
    if value.shape[0] != nnz or batch_indices.shape != (nnz,):
        raise ValueError("positions, batch_indices, query, key and value must have the same number of tokens")
    if llama_4_scaling_beta and original_max_position_embeddings <= 0:
        raise ValueError("original_max_position_embeddings must be positive")
    q, k, v = (_heads(t, head_size) for t in (query, key, value))
    if v.shape != k.shape:
        raise ValueError("key and value must have the same heads")
    _check_paged(k_cache, v_cache, kv_indptr, kv_last_page_len, k.shape[1], head_size, kv_layout, query.dtype)
    _check_device(query, value=value, batch_indices=batch_indices, k_cache=k_cache, v_cache=v_cache,
                  kv_indices=kv_indices, kv_indptr=kv_indptr)
    if nnz == 0:
        return
    _OP_ROPE_APPEND(q, k, v, cos_sin_cache, positions.contiguous(), _int32(batch_indices), k_cache, v_cache,
                    _int32(kv_indices), _int32(kv_indptr), not is_neox, kv_layout == "HND",
                    float(llama_4_scaling_beta or 0.0), int(original_max_position_embeddings),
                    True if enable_pdl is None else bool(enable_pdl))


# ------------------------------------------------------------------------------------------------
# Token-embedding gather.
# ------------------------------------------------------------------------------------------------
@torch.library.register_fake("mas_b200::embedding")
def _(input_ids, weight, enable_pdl):
    return weight.new_empty(tuple(input_ids.shape) + (weight.shape[1],))


@torch.library.register_fake("mas_b200::embedding_out")
def _(out, input_ids, weight, enable_pdl) -> None:
    return None


def _check_embedding(input_ids: torch.Tensor, weight: torch.Tensor) -> None:
    if input_ids.dtype not in _ID_DTYPES:
        raise ValueError(f"input_ids must be int32 or int64, got {input_ids.dtype}")
    if weight.dim() != 2 or weight.stride(1) != 1:
        raise ValueError("weight must be a (num_embeddings, embedding_dim) tensor, contiguous in its last dimension")
    _check_device(weight, input_ids=input_ids)


def embedding(input_ids: torch.Tensor, weight: torch.Tensor, enable_pdl: Optional[bool] = None) -> torch.Tensor:
    """``weight[input_ids]``: the row gather nn.Embedding performs (devstral2.py:260, :282), bit-exact.

    An id outside ``[0, num_embeddings)`` yields a zero row and sets MAS_STATUS_EMBED_ID_OUT_OF_RANGE
    in the device status word (`read_status`), where aten would raise a device-side assert.
    """
    _check_embedding(input_ids, weight)
    return _OP_EMBED(input_ids, weight, True if enable_pdl is None else bool(enable_pdl))


def embedding_out(out: torch.Tensor, input_ids: torch.Tensor, weight: torch.Tensor,
                  enable_pdl: Optional[bool] = None) -> torch.Tensor:
    """`embedding` into a caller-owned ``(*input_ids.shape, embedding_dim)`` tensor."""
    _check_embedding(input_ids, weight)
    if out.shape != tuple(input_ids.shape) + (weight.shape[1],) or out.dtype != weight.dtype:
        raise ValueError("out must be (*input_ids.shape, embedding_dim) with weight's dtype")
    if not out.is_contiguous():
        raise ValueError("out must be contiguous")
    _check_device(weight, out=out)
    _OP_EMBED_OUT(out, input_ids.contiguous(), weight, True if enable_pdl is None else bool(enable_pdl))
    return out


@torch.library.register_fake("mas_b200::embedding_fill")
def _(input_ids, weight, last_tokens, enable_pdl):
    return weight.new_empty(tuple(input_ids.shape) + (weight.shape[1],))


def embedding_fill_placeholders(input_ids: torch.Tensor, weight: torch.Tensor, last_tokens: torch.Tensor,
                                enable_pdl: Optional[bool] = None) -> torch.Tensor:
    """ModelRunner.fill_placeholders then the embedding gather, in one launch.

    Equivalent to (miniagentserve/engine/model_runner.py:149-154, then devstral2.py:282)::

        is_placeholder = input_ids < 0
        rows = (-1 - input_ids).clamp(min=0)
        input_ids.copy_(torch.where(is_placeholder, last_tokens[rows], input_ids))
        return embed_tokens(input_ids)

    `input_ids` is updated in place. A placeholder naming a row past the end of `last_tokens` gives a
    zero row and sets MAS_STATUS_EMBED_ID_OUT_OF_RANGE (torch would raise a device-side assert).
    """
    _check_embedding(input_ids, weight)
    if last_tokens.dtype not in _ID_DTYPES:
        raise ValueError(f"last_tokens must be int32 or int64, got {last_tokens.dtype}")
    _check_device(weight, last_tokens=last_tokens)
    if not input_ids.is_contiguous():
        raise ValueError("input_ids must be contiguous (it is updated in place)")
    return _OP_EMBED_FILL(input_ids, weight, last_tokens.contiguous(),
                          True if enable_pdl is None else bool(enable_pdl))
