"""The per-layer op chain of Devstral2DecoderLayer, minus its GEMMs and attention.

Devstral2Model.forward (miniagentserve/models/devstral2/devstral2.py:267-308) runs, per step:

    hidden = embed_tokens(input_ids)                                   # :282
    residual = zeros_like(hidden)                                      # :302
    for each layer (Devstral2DecoderLayer.forward, :237-253):
        fused_add_rmsnorm[_quant](x, hidden, residual, w_in, ...)      # :242-246  input norm
        qkv = qkv_proj(x); rope(positions, q, k, head_dim, cache)      # :158-166  q, k views of qkv
        ... attention, o_proj -> attn_out
        fused_add_rmsnorm[_quant](x, attn_out, residual, w_post, ...)  # :248-252  post-attn norm
        hidden = down_proj(silu_and_mul(gate_up_proj(x)))              # :223-224
    fused_add_rmsnorm(hidden, residual, norm, eps)                     # :305-307

`LayerChain` runs exactly the per-token ops of that sequence, on buffers that stand in for the GEMM
and attention outputs (attn_out, qkv, gate_up, and hidden as the previous MLP output). Every op is
the drop-in function the model would call, so a step through `LayerChain` exercises the same calls,
arguments and tensor layouts as the model: q and k are strided views of one fused qkv row.
`ChainShape` carries the ModelConfig / Devstral2Config fields the ops consume
(miniagentserve/models/model_config.py:68-86, devstral2/configs.py:153-162).
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass
from typing import Any, Optional

import torch

__all__ = ["ChainShape", "ChainBuffers", "LayerChain"]


@dataclass(frozen=True)
class ChainShape:
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    num_hidden_layers: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 1e9
    max_position_embeddings: int = 131072

    @classmethod
    def from_model_config(cls, config: Any) -> "ChainShape":
        """From a ModelConfig / Devstral2Config (same attribute names)."""
        return cls(**{f: getattr(config, f) for f in cls.__dataclass_fields__})

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    def bytes_per_layer(self, tokens: int, quant: bool = False) -> int:
        """Algorithmic HBM bytes of one layer's four ops at `tokens` tokens (each byte once).

        norm: read x, r; write r and y (bf16: 8 B/elem; fp8 out: 7 B/elem) + the weight once;
        rope: read+write q and k, one fp32 cos|sin row and one int32 position per token;
        silu: read gate and up, write out (6 B per output element; 5 B with the fp8 output).
        """
        H, I, D = self.hidden_size, self.intermediate_size, self.head_dim
        norm = (7 if quant else 8) * tokens * H + 2 * H
        rope = tokens * (2 * 2 * (self.q_size + self.kv_size) + 4 * D + 4)
        silu = (5 if quant else 6) * tokens * I
        return 2 * norm + rope + silu

    def embed_bytes(self, tokens: int, id_bytes: int = 8) -> int:
        return 2 * 2 * tokens * self.hidden_size + id_bytes * tokens


@dataclass
class ChainBuffers:
    """Device tensors one step of the chain reads and writes."""

    ids: torch.Tensor          # (T,) int64 token ids
    positions: torch.Tensor    # (T,) int32
    table: torch.Tensor        # (V, H) embedding table
    hidden: torch.Tensor       # (T, H): embedding output, then each layer's MLP-output stand-in
    residual: torch.Tensor     # (T, H)
    attn_out: torch.Tensor     # (T, H) attention-output stand-in
    qkv: torch.Tensor          # (T, qkv_size) qkv_proj-output stand-in
    gate_up: torch.Tensor      # (T, 2I) gate_up_proj-output stand-in
    act: torch.Tensor          # (T, I) silu_and_mul output
    cos_sin_cache: torch.Tensor  # (P, D) fp32
    w_in: torch.Tensor         # (L, H) input_layernorm weights
    w_post: torch.Tensor       # (L, H) post_attention_layernorm weights
    x_fp8: Optional[torch.Tensor] = None    # (T, H) e4m3, quantised form only
    act_fp8: Optional[torch.Tensor] = None  # (T, I) e4m3 down_proj input, quantised form only
    act_scale: Optional[torch.Tensor] = None  # (3,) fp32 activation scales (qkv, gate_up, down proj)


class LayerChain:
    """One model step's per-token ops over `ChainBuffers` (see the module docstring).

    quant=False uses the bf16 fused_add_rmsnorm for both per-layer norms (in place on hidden and
    attn_out) and the bf16 silu_and_mul; quant=True uses fused_add_rmsnorm_quant into x_fp8, as the
    decoder layers do, and -- when act_fp8 is given -- silu_and_mul_quant into act_fp8, which is
    down_proj's quantize_fp8 (devstral2.py:110-111) fused into the activation.
    """

    def __init__(self, shape: ChainShape, quant: bool = False, layers: Optional[int] = None, ops: Any = None):
        self.shape = shape
        self.quant = quant
        self.layers = shape.num_hidden_layers if layers is None else layers
        self._ops = ops  # an op namespace (this package's ops module unless given)

    @property
    def ops(self):
        if self._ops is None:
            self._ops = importlib.import_module(f"{__package__}.ops")
        return self._ops

    def embed(self, b: ChainBuffers) -> None:
        self.ops.embedding_out(b.hidden, b.ids, b.table)

    def layer(self, b: ChainBuffers, l: int) -> None:
        s = self.shape
        ops = self.ops
        eps = s.rms_norm_eps
        if self.quant:
            ops.fused_add_rmsnorm_quant(b.x_fp8, b.hidden, b.residual, b.w_in[l], b.act_scale[0:1], eps)
        else:
            ops.fused_add_rmsnorm(b.hidden, b.residual, b.w_in[l], eps)
        q = b.qkv[:, : s.q_size]
        k = b.qkv[:, s.q_size: s.q_size + s.kv_size]
        ops.apply_rope_with_cos_sin_cache_inplace(b.positions, q, k, s.head_dim, b.cos_sin_cache, is_neox=True)
        if self.quant:
            ops.fused_add_rmsnorm_quant(b.x_fp8, b.attn_out, b.residual, b.w_post[l], b.act_scale[1:2], eps)
        else:
            ops.fused_add_rmsnorm(b.attn_out, b.residual, b.w_post[l], eps)
        if self.quant and b.act_fp8 is not None:
            ops.silu_and_mul_quant(b.gate_up, b.act_scale[2:3], out=b.act_fp8)
        else:
            ops.silu_and_mul(b.gate_up, out=b.act)

    def step(self, b: ChainBuffers) -> None:
        """embed -> residual = 0 -> layers x (norm, rope, norm, silu)."""
        self.embed(b)
        b.residual.zero_()
        for l in range(self.layers):
            self.layer(b, l)

    def kernel_launches(self) -> int:
        """Kernels of this package per step (the residual memset is torch's)."""
        return 1 + 4 * self.layers

    def step_bytes(self, tokens: int) -> int:
        return self.shape.embed_bytes(tokens) + self.layers * self.shape.bytes_per_layer(tokens, self.quant)
