"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configurations.

There is no dataset on this path: every input is synthetic, drawn from a seeded torch.Generator on
the target device (so multi-GB inputs never cross PCIe), with the distributions the configurations
name. Host-side integer inputs (token ids, positions, ragged sequence lengths) come from a CPU
generator so the same seed gives the same batch on every machine.

    1 norm   x, r ~ N(0,1) bf16 [4096, 5120]; w = 1 + 0.1 N(0,1); eps 1e-5               seed 0
    2 silu   gate_up ~ N(0,1) bf16 [8192, 65536] -> out [8192, 32768]                      seed 1
    3 rope   64 seqs, len U[1,1024], offset U[0,65536), pos = offset + arange(len) int32;
             q [T,32,128], k [T,8,128] ~ N(0,1) bf16; fp32 cache [131072,128], theta 1e9   seed 2
    4 embed  table N(0,0.02) bf16 [131072, 5120]; ids int32 U[0,131072), T = 16384          seed 3
    5 chain  H 12288, 96/8 heads, D 128, I 28672, V 131072, theta 1e9, 88 layers;
             T = 256 decode + 2 x 2048 prefill = 4352                                       seed 4
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .chain import ChainBuffers, ChainShape
from .rope_cache import plain_cos_sin_cache

__all__ = ["CHAIN_SHAPE", "norm_inputs", "silu_inputs", "rope_batch", "rope_inputs", "embed_inputs",
           "paged_batch", "paged_batch_from_lengths", "PagedBatch", "rope_append_inputs",
           "chain_host_inputs", "chain_buffers", "RopeBatch"]

CHAIN_SHAPE = ChainShape(hidden_size=12288, intermediate_size=28672, num_attention_heads=96,
                         num_key_value_heads=8, head_dim=128, vocab_size=131072, num_hidden_layers=88,
                         rms_norm_eps=1e-5, rope_theta=1e9, max_position_embeddings=131072)
CHAIN_DECODE, CHAIN_PREFILL_CHUNKS, CHAIN_CHUNK = 256, 2, 2048


def _gen(device: torch.device | str, seed: int) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def _normal(shape, gen, device, dtype=torch.bfloat16, std: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(dtype)


def norm_inputs(device="cuda", seed: int = 0, tokens: int = 4096, hidden: int = 5120, dtype=torch.bfloat16):
    g = _gen(device, seed)
    x = _normal((tokens, hidden), g, device, dtype)
    r = _normal((tokens, hidden), g, device, dtype)
    w = _normal((hidden,), g, device, dtype, std=0.1, mean=1.0)
    return x, r, w, 1e-5


def silu_inputs(device="cuda", seed: int = 1, tokens: int = 8192, d: int = 32768, dtype=torch.bfloat16):
    return _normal((tokens, 2 * d), _gen(device, seed), device, dtype)


@dataclass
class RopeBatch:
    positions: torch.Tensor  # (T,) int32, CPU
    seq_lens: torch.Tensor   # (num_seqs,) int64, CPU


def rope_batch(seed: int = 2, num_seqs: int = 64, max_len: int = 1024, max_offset: int = 65536) -> RopeBatch:
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, max_len + 1, (num_seqs,), generator=g)
    offs = torch.randint(0, max_offset, (num_seqs,), generator=g)
    pos = torch.cat([o + torch.arange(int(n)) for o, n in zip(offs.tolist(), lens.tolist())]).to(torch.int32)
    return RopeBatch(positions=pos, seq_lens=lens)


def rope_inputs(device="cuda", seed: int = 2, num_q_heads: int = 32, num_kv_heads: int = 8, head_dim: int = 128,
                max_positions: int = 131072, theta: float = 1e9, dtype=torch.bfloat16, batch: RopeBatch | None = None):
    """(positions int32 [T] on device, q [T, Hq*D], k [T, Hkv*D], cache fp32 [P, D]) for config 3."""
    b = rope_batch(seed) if batch is None else batch
    T = b.positions.shape[0]
    g = _gen(device, seed)
    q = _normal((T, num_q_heads * head_dim), g, device, dtype)
    k = _normal((T, num_kv_heads * head_dim), g, device, dtype)
    cache = plain_cos_sin_cache(head_dim, max_positions, theta).to(device)
    return b.positions.to(device), q, k, cache


@dataclass
class PagedBatch:
    """One step's paged-KV metadata as ModelRunner / Devstral2Model.forward build it
    (miniagentserve/engine/model_runner.py:31-66, models/devstral2/devstral2.py:283-290): decode rows
    first (one new token each), then prompt chunks; every sequence's cache blocks come from a shared
    pool, listed row by row in block_tables (batch, max_blocks) whose flattening is kv_indices."""

    positions: torch.Tensor        # (T,) int32: each new token's position in its sequence
    batch_indices: torch.Tensor    # (T,) int32
    seq_lens: torch.Tensor         # (batch,) int32: cached + new tokens
    block_tables: torch.Tensor     # (batch, max_blocks) int32
    kv_indptr: torch.Tensor        # (batch + 1,) int32 = arange(batch + 1) * max_blocks
    kv_last_page_len: torch.Tensor  # (batch,) int32 = (seq_lens - 1) % page_size + 1
    num_pages: int
    page_size: int

    @property
    def kv_indices(self) -> torch.Tensor:
        return self.block_tables.flatten()

    def to(self, device) -> "PagedBatch":
        f = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in self.__dict__.items()}
        return PagedBatch(**f)


def paged_batch(seed: int = 6, num_decodes: int = 8, prompt_lens=(37, 64), max_cached: int = 300,
                page_size: int = 16, spare_pages: int = 5) -> PagedBatch:
    """A mixed step on the CPU: `num_decodes` decode rows with random cached lengths in
    [1, max_cached], then prompt rows of `prompt_lens` new tokens after random cached prefixes.
    Pages are a random permutation of a pool with `spare_pages` unused pages (plus the runner's
    padding sink, page num_pages - 1); unused block-table slots point at the sink."""
    g = torch.Generator().manual_seed(seed)
    new = [1] * num_decodes + list(prompt_lens)
    cached = torch.randint(1, max_cached + 1, (len(new),), generator=g).tolist()
    if num_decodes < len(new):
        for i in range(num_decodes, len(new)):
            cached[i] = int(torch.randint(0, max_cached + 1, (1,), generator=g))
    return paged_batch_from_lengths(cached, new, page_size, spare_pages, g)


def paged_batch_from_lengths(cached, new, page_size: int = 16, spare_pages: int = 5,
                             gen: torch.Generator | None = None) -> PagedBatch:
    """Sequences of cached[b] tokens already in the cache and new[b] tokens this step, their blocks
    a random permutation of the pool (see `paged_batch`)."""
    g = torch.Generator().manual_seed(0) if gen is None else gen
    cached, new = [int(c) for c in cached], [int(n) for n in new]
    seq_lens = [c + n for c, n in zip(cached, new)]
    blocks = [-(-L // page_size) for L in seq_lens]
    max_blocks = max(blocks)
    used = sum(blocks)
    num_pages = used + spare_pages + 1
    sink = num_pages - 1
    perm = torch.randperm(num_pages - 1, generator=g)[:used].to(torch.int32)
    table = torch.full((len(new), max_blocks), sink, dtype=torch.int32)
    o = 0
    for b, nb in enumerate(blocks):
        table[b, :nb] = perm[o:o + nb]
        o += nb
    positions = torch.cat([torch.arange(c, c + n) for c, n in zip(cached, new)]).to(torch.int32)
    batch_indices = torch.cat([torch.full((n,), b) for b, n in enumerate(new)]).to(torch.int32)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    return PagedBatch(positions=positions, batch_indices=batch_indices, seq_lens=sl, block_tables=table,
                      kv_indptr=torch.arange(len(new) + 1, dtype=torch.int32) * max_blocks,
                      kv_last_page_len=(sl - 1) % page_size + 1, num_pages=num_pages, page_size=page_size)


def rope_append_inputs(device="cuda", seed: int = 2, num_q_heads: int = 32, num_kv_heads: int = 8,
                       head_dim: int = 128, page_size: int = 16, max_positions: int = 131072, theta: float = 1e9,
                       dtype=torch.bfloat16, max_offset: int = 65536):
    """Configuration 3's ragged batch (64 sequences of U[1, 1024] new tokens after random cached
    prefixes below `max_offset`) as one prefill step over a paged cache: (PagedBatch on device,
    qkv [T, (Hq+2Hkv)*D], cos|sin cache, k_cache, v_cache [pages, page_size, Hkv, D])."""
    rb = rope_batch(seed, max_offset=max_offset)
    starts = torch.cumsum(rb.seq_lens, 0) - rb.seq_lens
    cached = rb.positions[starts.long()].tolist()
    b = paged_batch_from_lengths(cached, rb.seq_lens.tolist(), page_size, 5, torch.Generator().manual_seed(seed))
    assert torch.equal(b.positions, rb.positions)
    T = b.positions.shape[0]
    g = _gen(device, seed)
    qkv = _normal((T, (num_q_heads + 2 * num_kv_heads) * head_dim), g, device, dtype)
    cache = plain_cos_sin_cache(head_dim, max_positions, theta).to(device)
    shape = (b.num_pages, page_size, num_kv_heads, head_dim)
    k_cache = torch.zeros(shape, dtype=dtype, device=device)
    v_cache = torch.zeros(shape, dtype=dtype, device=device)
    return b.to(device), qkv, cache, k_cache, v_cache


def embed_inputs(device="cuda", seed: int = 3, vocab: int = 131072, hidden: int = 5120, tokens: int = 16384,
                 id_dtype=torch.int32, dtype=torch.bfloat16):
    table = _normal((vocab, hidden), _gen(device, seed), device, dtype, std=0.02)
    ids = torch.randint(0, vocab, (tokens,), generator=torch.Generator().manual_seed(seed), dtype=torch.int64)
    return table, ids.to(id_dtype).to(device)


def chain_host_inputs(seed: int = 4, shape: ChainShape = CHAIN_SHAPE, replicas: int = 1,
                      decode: int = CHAIN_DECODE, chunks: int = CHAIN_PREFILL_CHUNKS, chunk: int = CHAIN_CHUNK):
    """Token ids (int64) and positions (int32) of `replicas` back-to-back mixed steps, on the CPU.

    Each mixed step is `decode` decode tokens (one per sequence, at a random position) followed by
    `chunks` prefill chunks of `chunk` consecutive positions. Rank r of an N-GPU run takes the r-th
    step: a contiguous slice of the ragged global batch.
    """
    g = torch.Generator().manual_seed(seed)
    P = shape.max_position_embeddings
    ids, pos = [], []
    for _ in range(replicas):
        ids.append(torch.randint(0, shape.vocab_size, (decode + chunks * chunk,), generator=g, dtype=torch.int64))
        p = [torch.randint(1, P, (decode,), generator=g)]
        for _c in range(chunks):
            off = int(torch.randint(0, P - chunk, (1,), generator=g))
            p.append(off + torch.arange(chunk))
        pos.append(torch.cat(p).to(torch.int32))
    return torch.cat(ids), torch.cat(pos)


def chain_buffers(ids: torch.Tensor, positions: torch.Tensor, device="cuda", seed: int = 4,
                  shape: ChainShape = CHAIN_SHAPE, quant: bool = False, layers: int | None = None) -> ChainBuffers:
    """Device buffers for `LayerChain` over the given (host or device) ids and positions."""
    s = shape
    L = s.num_hidden_layers if layers is None else layers
    T = ids.shape[0]
    g = _gen(device, seed)
    b = ChainBuffers(
        ids=ids.to(device),
        positions=positions.to(device),
        table=_normal((s.vocab_size, s.hidden_size), g, device, std=0.02),
        hidden=torch.empty((T, s.hidden_size), dtype=torch.bfloat16, device=device),
        residual=torch.zeros((T, s.hidden_size), dtype=torch.bfloat16, device=device),
        attn_out=_normal((T, s.hidden_size), g, device),
        qkv=_normal((T, s.qkv_size), g, device),
        gate_up=_normal((T, 2 * s.intermediate_size), g, device),
        act=torch.empty((T, s.intermediate_size), dtype=torch.bfloat16, device=device),
        cos_sin_cache=plain_cos_sin_cache(s.head_dim, s.max_position_embeddings, s.rope_theta).to(device),
        w_in=_normal((L, s.hidden_size), g, device, std=0.1, mean=1.0),
        w_post=_normal((L, s.hidden_size), g, device, std=0.1, mean=1.0),
    )
    if quant:
        b.x_fp8 = torch.empty((T, s.hidden_size), dtype=torch.float8_e4m3fn, device=device)
        b.act_fp8 = torch.empty((T, s.intermediate_size), dtype=torch.float8_e4m3fn, device=device)
        b.act_scale = torch.tensor([0.05, 0.05, 0.0137], dtype=torch.float32, device=device)
    return b
