"""Benchmark of the B200 per-token layer ops (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mas|reference|flashinfer]
                    [--workload chain|chain_fp8|norm|norm_fp8|silu|silu_fp8|rope|rope_append|embed|
                                embed_fill|norm_chain|norm_fp8_chain|silu_chain|silu_fp8_chain|rope_chain|
                                rope_qscale_chain]

Default workload: configuration 5, the per-layer op chain at 123B-class shapes (H 12288, 96/8 heads,
D 128, I 28672, V 131072): one step = embed + 88 x (input RMSNorm+residual, rope on q/k, post-attn
RMSNorm+residual, SiLU-mul on [T, 57344]) over T = 256 decode + 2 x 2048 prefill tokens, with seeded
random bf16 activations standing in for the attention and GEMM outputs (mas_b200.chain). `chain_fp8`
is the same step with the calls the decoder layers actually make (e4m3-out norms, and SiLU-mul with
the down projection's activation quantisation). The other workloads time one op per launch:
configurations 1-4, their fp8 and paged-append forms, and the chain's shapes.

Metric: tokens/s of the whole job (all ranks), plus the chain's algorithmic HBM GB/s and its fraction
of the measured HBM peak. Multi-GPU (torchrun, one rank per GPU): the headline is weak scaling (the
global batch is N mixed steps and rank r takes the r-th, a contiguous slice); no collective touches
the data path. NCCL only carries barriers, the max over ranks of the timings and, after the timed
regions, the gather of every rank's sampled outputs for the oracle check.

Reported alongside the device-resident `value` (chain workloads, this package's kernels):
  e2e             the same step through the public API with the step's host inputs (token ids,
                  positions) copied from pinned memory and the result (the residual stream) copied
                  back to pinned memory on a second stream, overlapping the next step, all inside the
                  timed region;
  roofline        the dominant kernel's algorithmic bytes / its CUDA-event time, against the measured
                  HBM copy peak (MEASURED_PEAKS.json); events bracket its launches in every 16th layer
                  (both norms); `traffic` is that kernel's DRAM bytes from an ncu capture, and
                  `ncu_in_chain_us` its mean in-chain time from an ncu launch list (profiles/);
  flashinfer      the reference's own GPU kernels (flashinfer 0.6.11.post2 and aten's gather) on the
                  same inputs in the same process: value, e2e, clocks;
  chain_fp8       the other chain form, both kernel sets;
  strong_scaling  one fixed 4352-token step split into N contiguous token ranges, both kernel sets;
  small_steps     steps of 64, 256 and 512 tokens replayed from a CUDA graph, both kernel sets;
  cpu_baseline    the reference's CPU path timed on this host's cores on a token sample of the same
                  workload (rank 0, N = 1): torch's CPU embedding, and the C oracle for the ops whose
                  reference kernels are CUDA-only;
  fault_word, status_word  the library's words after the timed regions (must be 0);
  gathered_outputs  every rank's digest, and an oracle check of 8 sampled tokens per rank through a
                  whole step (the run fails if a word is nonzero or the check fails);
  clocks          SM clock and throttle reasons sampled by nvidia-smi during the timed region.

--impl reference times the reference's CPU path alone (rank 0; nothing of this package's CUDA code
is loaded). --impl flashinfer times the reference's GPU kernels alone on any workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Fused-op HBM GB/s (% of B200 peak) and tokens/s at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0  # the B200 data-sheet figure, for context beside the measured copy peak
L2_BYTES = 126 * 1024 * 1024
SLEEP_CYCLES = 100_000_000  # ~50 ms at 1.9 GHz


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of each workload's dominant
# kernel, from one ncu capture of that workload (summaries and commands in profiles/). Reads equal the
# algorithmic bytes; writes come out lower because dirty lines still in the 126 MB L2 when the kernel
# ends are not counted.
NCU_TRAFFIC = {
    "chain": (214_000_896 + 157_683_968, "profiles/norm_row_keep_chain_shape.md"),
    "norm_chain": (214_000_896 + 157_683_968, "profiles/norm_row_keep_chain_shape.md"),
    "chain_fp8": (213_974_272 + 105_492_480, "profiles/norm_row_keep_chain_shape.md"),
    "norm_fp8_chain": (213_974_272 + 105_492_480, "profiles/norm_row_keep_chain_shape.md"),
    "norm": (83_919_616 + 24_468_480, "profiles/norm_loop_keep_config1.md"),
    "norm_fp8": (83_921_152 + 10_962_688, "profiles/norm_loop_keep_config1.md"),
    "silu": (1_073_837_568 + 498_061_312, "profiles/ops_dram_traffic.md"),
    "silu_fp8": (1_073_865_728 + 253_526_784, "profiles/ops_dram_traffic.md"),
    "silu_chain": (499_155_200 + 219_000_064, "profiles/ops_dram_traffic.md"),
    "embed": (160_659_200 + 115_822_848, "profiles/ops_dram_traffic.md"),
    "rope": (327_856_384 + 256_022_016, "profiles/ops_dram_traffic.md"),
    "rope_chain": (118_173_952 + 59_143_424, "profiles/rope_ring_chain_shape.md"),
    "silu_fp8_chain": (499_176_448 + 109_594_624, "profiles/ops_dram_traffic.md"),
    "rope_append_small": (383_225_088 + 380_423_424, "profiles/ops_dram_traffic.md"),
}


# Mean device time of the dominant kernel inside the chain, from an ncu launch list of the bench's
# own default command (gpu__time_duration.sum only, --clock-control none): an unperturbed in-chain
# figure beside the event-bracketed one, which cancels the programmatic-launch overlap around it.
NCU_IN_CHAIN = {"chain": (62.24, "profiles/chain_launches.md")}

# Bound on the end-to-end oracle check of sampled tokens (bf16 ulps / e4m3 steps after 88 layers).
CHECK_BOUND_ULP = 8


# --------------------------------------------------------------------------------------------------
# Process group.
# --------------------------------------------------------------------------------------------------
class Dist:
    def __init__(self, backend: str = "nccl"):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False
        if self.world > 1 and backend != "none":
            import datetime

            import torch.distributed as dist

            if backend == "nccl":
                torch.cuda.set_device(self.local_rank)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local_rank) if backend == "nccl" else None)
            self.pg = True

    def barrier(self) -> None:
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def max(self, x: float, device) -> float:
        if not self.pg:
            return x
        import torch.distributed as dist

        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_objects(self, obj) -> list:
        if not self.pg:
            return [obj]
        import torch.distributed as dist

        out = [None] * self.world
        dist.all_gather_object(out, obj)
        return out

    def close(self) -> None:
        if self.pg:
            import torch.distributed as dist

            dist.destroy_process_group()


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) slice of `total` units for `rank` (sizes differ by at most one)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


# --------------------------------------------------------------------------------------------------
# Clock sampling during the timed region.
# --------------------------------------------------------------------------------------------------
class Clocks:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, names = [], [], set()
        reason_names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(reason_names, f[5:9]):
                if v.lower() == "active":
                    names.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(names), "samples": len(sm)}


# --------------------------------------------------------------------------------------------------
# Implementations of the ops (the chain calls whichever namespace it is given).
# --------------------------------------------------------------------------------------------------
class FlashinferOps:
    """The reference's own GPU path: flashinfer kernels and the aten gather behind nn.Embedding."""

    def __init__(self):
        from flashinfer.activation import silu_and_mul
        from flashinfer.norm import fused_add_rmsnorm, fused_add_rmsnorm_quant
        from flashinfer.rope import apply_rope_with_cos_sin_cache_inplace

        self.fused_add_rmsnorm = fused_add_rmsnorm
        self.fused_add_rmsnorm_quant = fused_add_rmsnorm_quant
        self.silu_and_mul = silu_and_mul
        self.apply_rope_with_cos_sin_cache_inplace = apply_rope_with_cos_sin_cache_inplace

    @staticmethod
    def embedding_out(out, ids, table):
        return torch.index_select(table, 0, ids, out=out.view(-1, table.shape[1]))

    @staticmethod
    def apply_rope_and_append_paged_kv_cache(positions, q, k, v, head_size, cache, batch_indices, paged_kv_cache,
                                             kv_indices, kv_indptr, kv_last_page_len, **_):
        """The reference's unfused pair: flashinfer rope, then flashinfer append_paged_kv_cache
        (devstral2.py:163-173)."""
        from flashinfer.page import append_paged_kv_cache
        from flashinfer.rope import apply_rope_with_cos_sin_cache_inplace

        T = q.shape[0]
        apply_rope_with_cos_sin_cache_inplace(positions, q, k, head_size, cache, is_neox=True)
        append_paged_kv_cache(k.view(T, -1, head_size), v.view(T, -1, head_size), batch_indices, positions,
                              paged_kv_cache, kv_indices, kv_indptr, kv_last_page_len, kv_layout="NHD")

    def apply_rope_and_llama4_query_scale_inplace(self, positions, q, k, head_size, cache, beta, orig, is_neox=True):
        """The reference's sequence: flashinfer rope, then the eager llama-4 query scale into a new
        tensor (devstral2.py:163-166, :175-179)."""
        self.apply_rope_with_cos_sin_cache_inplace(positions, q, k, head_size, cache, is_neox=is_neox)
        attn_scale = 1 + beta * torch.log1p(torch.floor(positions.float() / orig))
        q3 = q.unflatten(-1, (-1, head_size))
        return q3 * attn_scale[:, None, None].to(q.dtype)

    @staticmethod
    def embedding_fill_placeholders(ids, table, last):
        """The reference's pair: ModelRunner.fill_placeholders (model_runner.py:149-154) then the
        embedding gather."""
        is_placeholder = ids < 0
        rows = (-1 - ids).clamp(min=0)
        ids.copy_(torch.where(is_placeholder, last[rows], ids))
        return torch.index_select(table, 0, ids)

    _quantize = None

    def silu_and_mul_quant(self, x, scale, out=None, enable_pdl=True):
        """The reference's unfused pair: flashinfer silu_and_mul, then FP8Linear's compiled
        quantize_fp8 (devstral2.py:93-95, :110-111)."""
        if FlashinferOps._quantize is None:
            fp8 = torch.float8_e4m3fn
            fp8_max = torch.finfo(fp8).max

            @torch.compile(dynamic=True)
            def quantize_fp8(a, s):
                return (a / s).clamp(-fp8_max, fp8_max).to(fp8)

            FlashinferOps._quantize = quantize_fp8
        # `out` is ignored: the reference allocates the quantised activation (no extra copy timed)
        return FlashinferOps._quantize(self.silu_and_mul(x, enable_pdl=enable_pdl), scale)


# --------------------------------------------------------------------------------------------------
# Workloads: each builds device state and returns closures for one step.
# --------------------------------------------------------------------------------------------------
def chain_config(layers: int, tokens_per_gpu: int, global_tokens: int) -> dict:
    """The chain workload's config, identical for every arm (mas, flashinfer, reference) at one N."""
    from mas_b200 import workloads as wl

    s = wl.CHAIN_SHAPE
    return {"workload": "chain (config 5): embed + 88 x [RMSNorm+res, rope q/k, RMSNorm+res, SiLU-mul]",
            "hidden": s.hidden_size, "q_heads": s.num_attention_heads, "kv_heads": s.num_key_value_heads,
            "head_dim": s.head_dim, "intermediate": s.intermediate_size, "vocab": s.vocab_size, "layers": layers,
            "tokens_per_gpu": tokens_per_gpu, "global_tokens": global_tokens,
            "step_mix": "256 decode + 2 x 2048 prefill tokens per GPU", "norm": "bf16 fused_add_rmsnorm",
            "l2": "inputs larger than L2 (per-layer working set 1.84 GB)", "parallelism": "token-sharded dp"}


def chain_fp8_config(layers: int, tokens_per_gpu: int, global_tokens: int) -> dict:
    cfg = chain_config(layers, tokens_per_gpu, global_tokens)
    cfg["workload"] = ("chain, fp8 form (the decoder layers' own calls): embed + 88 x [RMSNorm+res -> e4m3, "
                       "rope q/k, RMSNorm+res -> e4m3, SiLU-mul -> e4m3]")
    cfg["norm"] = "fused_add_rmsnorm_quant"
    return cfg


class ChainWorkload:
    """Configuration 5's step on this rank's tokens, through a pluggable op namespace.

    The buffers hold this rank's `tokens` tokens; `view(n, ids, pos)` gives a workload over the first n
    rows of the same buffers with other ids and positions (the strong-scaling slice, the small steps).
    The fp8 outputs are always allocated, so one set of inputs serves both forms (`quant`).
    """

    name = "chain"
    EVENT_EVERY = 16  # layers 8, 24, 40, 56, 72 carry events around both of their norms
    per_launch_value = False

    def __init__(self, device, ops, layers: int, host_ids, host_pos, seed: int, quant: bool = False,
                 buffers=None):
        from mas_b200 import workloads as wl
        from mas_b200.chain import LayerChain

        self.wl = wl
        self.shape = wl.CHAIN_SHAPE
        self.device = device
        self.host_ids = host_ids.clone().pin_memory()
        self.host_pos = host_pos.clone().pin_memory()
        self.tokens = host_ids.shape[0]
        self.layers = layers
        self.seed = seed
        self.b = buffers if buffers is not None else wl.chain_buffers(
            self.host_ids, self.host_pos, device=device, seed=seed, layers=layers, quant=True)
        self.chain_ops = ops
        self.set_quant(quant)

    def set_quant(self, quant: bool) -> None:
        from mas_b200.chain import LayerChain

        self.quant = quant
        self.name = "chain_fp8" if quant else "chain"
        self.dominant = "fused_add_rmsnorm_quant" if quant else "fused_add_rmsnorm"
        self.chain = LayerChain(self.shape, quant=quant, layers=self.layers)

    def view(self, n: int, host_ids, host_pos) -> "ChainWorkload":
        """A workload over the first n rows of these buffers, with the given ids and positions."""
        from mas_b200.chain import ChainBuffers

        b = self.b
        v = ChainBuffers(ids=host_ids.to(self.device), positions=host_pos.to(self.device), table=b.table,
                         hidden=b.hidden[:n], residual=b.residual[:n], attn_out=b.attn_out[:n], qkv=b.qkv[:n],
                         gate_up=b.gate_up[:n], act=b.act[:n], cos_sin_cache=b.cos_sin_cache, w_in=b.w_in,
                         w_post=b.w_post, x_fp8=b.x_fp8[:n], act_fp8=b.act_fp8[:n], act_scale=b.act_scale)
        return ChainWorkload(self.device, self.chain_ops, self.layers, host_ids, host_pos, self.seed,
                             quant=self.quant, buffers=v)

    # the chain with a pluggable op namespace, optionally bracketing the dominant kernel with events
    def step(self, dom_events=None):
        b, s, o = self.b, self.shape, self.chain_ops
        eps = s.rms_norm_eps
        o.embedding_out(b.hidden, b.ids, b.table)
        b.residual.zero_()
        q = b.qkv[:, : s.q_size]
        k = b.qkv[:, s.q_size: s.q_size + s.kv_size]
        st = torch.cuda.current_stream()
        for l in range(self.layers):
            # Events bracket the dominant kernel's launches in a sample of layers only: an event
            # between two kernels cancels their programmatic-launch overlap, so bracketing every
            # launch would slow the timed region itself.
            timed = dom_events is not None and l % self.EVENT_EVERY == self.EVENT_EVERY // 2
            if timed:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
            if self.quant:
                o.fused_add_rmsnorm_quant(b.x_fp8, b.hidden, b.residual, b.w_in[l], b.act_scale[0:1], eps,
                                          enable_pdl=True)
            else:
                o.fused_add_rmsnorm(b.hidden, b.residual, b.w_in[l], eps, enable_pdl=True)
            if timed:
                e1.record(st)
                dom_events.append((e0, e1))
            o.apply_rope_with_cos_sin_cache_inplace(b.positions, q, k, s.head_dim, b.cos_sin_cache, is_neox=True)
            if timed:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
            if self.quant:
                o.fused_add_rmsnorm_quant(b.x_fp8, b.attn_out, b.residual, b.w_post[l], b.act_scale[1:2], eps,
                                          enable_pdl=True)
            else:
                o.fused_add_rmsnorm(b.attn_out, b.residual, b.w_post[l], eps, enable_pdl=True)
            if timed:
                e1.record(st)
                dom_events.append((e0, e1))
            if self.quant:
                o.silu_and_mul_quant(b.gate_up, b.act_scale[2:3], out=b.act_fp8, enable_pdl=True)
            else:
                o.silu_and_mul(b.gate_up, out=b.act, enable_pdl=True)

    def e2e_setup(self):
        """Two residual buffers and two pinned host outputs, alternating by step, and a copy stream."""
        b = self.b
        self._res0 = b.residual
        self._res = [b.residual, torch.empty_like(b.residual)]
        self._host_out = [torch.empty(b.residual.shape, dtype=b.residual.dtype).pin_memory() for _ in range(2)]
        self._copy_stream = torch.cuda.Stream(device=b.residual.device)
        self._d2h_done = [None, None]
        self._i = 0

    def e2e_step(self):
        """One step through the public API, as a serving loop runs it: the step's ids and positions in
        from pinned memory, the chain, then the step's residual out to pinned memory on a copy stream,
        which overlaps the next step's kernels. The residual buffers alternate, so a step never writes
        a buffer whose copy to the host is still in flight."""
        b = self.b
        main = torch.cuda.current_stream()
        k = self._i & 1
        if self._d2h_done[k] is not None:
            main.wait_event(self._d2h_done[k])
        b.residual = self._res[k]
        b.ids.copy_(self.host_ids, non_blocking=True)
        b.positions.copy_(self.host_pos, non_blocking=True)
        self.step(None)
        done = torch.cuda.Event()
        done.record(main)
        cs = self._copy_stream
        cs.wait_event(done)
        with torch.cuda.stream(cs):
            self._host_out[k].copy_(self._res[k], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(cs)
        self._d2h_done[k] = ev
        self._i += 1

    def e2e_finish(self):
        """Makes the current stream wait for the last copy to the host (inside the timed region), and
        puts the first residual buffer back."""
        torch.cuda.current_stream().wait_stream(self._copy_stream)
        self.b.residual = self._res0

    def digest(self) -> dict:
        """This rank's output fingerprint (outside the timed region): its token count and the integer
        sums of the final residual and hidden bit patterns."""
        b = self.b
        return {"tokens": int(self.tokens),
                "residual_bits_sum": int(b.residual.view(torch.int16).to(torch.int64).sum().item()),
                "hidden_bits_sum": int(b.hidden.view(torch.int16).to(torch.int64).sum().item())}

    def sample_step(self, n: int = 8) -> dict:
        """One more step, with the inputs and outputs of `n` evenly spaced tokens copied to the host for
        an oracle check. Every op is per token, so the sampled tokens' outputs depend only on their own
        inputs (the layer weights are shared). Inputs carried from step to step (attn_out and qkv are
        updated in place) are captured just before the step."""
        b, s = self.b, self.shape
        sel = torch.linspace(0, self.tokens - 1, n, device=self.device).long()
        ids = b.ids[sel]
        inp = {"ids": ids.cpu(), "table_rows": b.table[ids].cpu(), "attn_out": b.attn_out[sel].cpu(),
               "qkv": b.qkv[sel].cpu(), "gate_up": b.gate_up[sel].cpu(), "cache_rows": b.cos_sin_cache[
                   b.positions[sel].long()].cpu(), "w_in": b.w_in.cpu(), "w_post": b.w_post.cpu(),
               "act_scale": b.act_scale.cpu()}
        self.step()
        out = {"residual": b.residual[sel].cpu(), "qkv": b.qkv[sel].cpu()}
        if self.quant:
            out.update(x_fp8=b.x_fp8[sel].cpu(), act_fp8=b.act_fp8[sel].cpu())
        else:
            out.update(hidden=b.hidden[sel].cpu(), attn_out=b.attn_out[sel].cpu(), act=b.act[sel].cpu())
        return {"tokens": sel.cpu(), "quant": self.quant, "layers": self.layers, "inputs": inp, "outputs": out}

    def e2e_bytes(self) -> tuple[int, int]:
        return (self.host_ids.numel() * 8 + self.host_pos.numel() * 4,
                self.b.residual.numel() * self.b.residual.element_size())

    def launches_per_step(self) -> int:
        return 1 + 4 * self.layers

    def step_bytes(self) -> int:
        return self.chain.step_bytes(self.tokens)

    def dominant_bytes_per_launch(self) -> int:
        return (7 if self.quant else 8) * self.tokens * self.shape.hidden_size + 2 * self.shape.hidden_size


def oracle_check(sample: dict, eps: float) -> dict:
    """Runs the oracle over a `ChainWorkload.sample_step` sample and compares: max distance in units
    of the output format's last place (bf16 ulps, e4m3 steps) per output.

    The oracle follows the reference's kernels to within one ulp per op; over 88 chained layers such
    last-place differences feed later layers (the residual stream carries them), so an end-to-end
    comparison allows a few ulps where the op-by-op tests allow one."""
    import oracle
    from mas_b200 import workloads as wl

    s = wl.CHAIN_SHAPE
    inp, L = sample["inputs"], sample["layers"]
    n = inp["ids"].shape[0]
    hidden = inp["table_rows"].clone()
    residual = torch.zeros_like(hidden)
    attn, qkv, gate_up = inp["attn_out"].clone(), inp["qkv"].clone(), inp["gate_up"]
    pos = torch.arange(n, dtype=torch.int32)
    cache = inp["cache_rows"].contiguous()
    act = torch.empty(n, s.intermediate_size, dtype=torch.bfloat16)
    x8 = torch.empty(n, s.hidden_size, dtype=torch.float8_e4m3fn)
    act8 = torch.empty(n, s.intermediate_size, dtype=torch.float8_e4m3fn)
    sc = inp["act_scale"].tolist()
    q = qkv[:, : s.q_size]
    k = qkv[:, s.q_size: s.q_size + s.kv_size]
    for l in range(L):
        if sample["quant"]:
            oracle.fused_add_rmsnorm_quant(x8, hidden, residual, inp["w_in"][l], sc[0], eps)
        else:
            oracle.fused_add_rmsnorm(hidden, residual, inp["w_in"][l], eps)
        oracle.apply_rope_with_cos_sin_cache_inplace(pos, q, k, s.head_dim, cache)
        if sample["quant"]:
            oracle.fused_add_rmsnorm_quant(x8, attn, residual, inp["w_post"][l], sc[1], eps)
            oracle.silu_and_mul_quant(gate_up, sc[2], out=act8)
        else:
            oracle.fused_add_rmsnorm(attn, residual, inp["w_post"][l], eps)
            oracle.silu_and_mul(gate_up, out=act)
    want = {"residual": residual, "qkv": qkv}
    if sample["quant"]:
        want.update(x_fp8=x8, act_fp8=act8)
    else:
        want.update(hidden=hidden, attn_out=attn, act=act)

    def ordered(t):
        if t.dtype == torch.float8_e4m3fn:
            i = t.view(torch.uint8).to(torch.int32)
            return torch.where(i >= 128, -(i & 127), i)
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)

    return {name: int((ordered(sample["outputs"][name]) - ordered(w)).abs().max()) for name, w in want.items()}


class OpWorkload:
    """One op of configurations 1-4 per step (for per-kernel measurements)."""

    def __init__(self, name: str, device, dist: Dist, ops):
        from mas_b200 import workloads as wl

        self.name, self.o, self.dominant = name, ops, name
        self.workload = name
        self.dev = device
        cs = wl.CHAIN_SHAPE
        if name in ("norm", "norm_fp8", "norm_chain", "norm_fp8_chain"):
            chain = name.endswith("_chain")
            quant = name.startswith("norm_fp8")
            if chain:
                self.x, self.r, self.w, self.eps = wl.norm_inputs(device, seed=4, tokens=4352, hidden=cs.hidden_size)
            else:
                self.x, self.r, self.w, self.eps = wl.norm_inputs(device)
            self.T, H = self.x.shape
            self.out = torch.empty(self.x.shape, dtype=torch.float8_e4m3fn, device=device)
            self.scale = torch.tensor([0.05], device=device)
            self.bytes = (7 if quant else 8) * self.T * H + 2 * H
            self.cfg = {"workload": f"{'chain-shape' if chain else 'config 1'} "
                                    f"{'fp8-out ' if quant else ''}RMSNorm+residual",
                        "tokens": self.T, "hidden": H,
                        "l2": f"inputs {2 * self.x.numel() * self.x.element_size() / 1e6:.0f} MB "
                              f"{'>' if 2 * self.x.numel() * self.x.element_size() > L2_BYTES else '<'} L2"}
            self.name = "norm_fp8" if quant else "norm"
        elif name in ("silu", "silu_chain", "silu_fp8", "silu_fp8_chain"):
            chain = name.endswith("_chain")
            quant = name.startswith("silu_fp8")
            self.x = (wl.silu_inputs(device, seed=4, tokens=4352, d=cs.intermediate_size) if chain
                      else wl.silu_inputs(device))
            self.T = self.x.shape[0]
            self.out = torch.empty(self.T, self.x.shape[1] // 2,
                                   dtype=torch.float8_e4m3fn if quant else self.x.dtype, device=device)
            self.scale = torch.tensor(0.0137, device=device)
            # read gate + up (4 B), write the activation (2 B) or its e4m3 byte (1 B)
            self.bytes = (5 if quant else 6) * self.T * self.out.shape[1]
            self.cfg = {"workload": f"{'chain-shape' if chain else 'config 2'} SiLU-mul"
                                    f"{' + fp8 activation quant' if quant else ''}",
                        "tokens": self.T, "d": self.out.shape[1], "l2": "inputs larger than L2"}
            self.name = "silu_fp8" if quant else "silu"
        elif name in ("rope_chain", "rope_qscale_chain"):
            ids, pos = wl.chain_host_inputs()
            b = wl.chain_buffers(ids, pos, device=device, layers=1)
            self.pos, self.cache = b.positions, b.cos_sin_cache
            self.q, self.k = b.qkv[:, : cs.q_size], b.qkv[:, cs.q_size: cs.q_size + cs.kv_size]
            self._keep = b
            self.T = self.pos.shape[0]
            self.bytes = self.T * (2 * 2 * (cs.q_size + cs.kv_size) + 4 * 128 + 4)
            self.cfg = {"workload": "chain-shape rope: q/k strided views of qkv [4352, 14336], 96+8 heads",
                        "tokens": self.T, "l2": "inputs larger than L2"}
            self.name = "rope"
            if name == "rope_qscale_chain":
                # Devstral2Attention's llama-4 query scale (devstral2.py:175-179) fused into rope (f1)
                self.beta, self.orig = 0.1, 8192
                self.cfg["workload"] = "chain-shape rope + llama-4 query scale (beta 0.1, original max 8192)"
                self.name = "rope_qscale"
        elif name == "rope":
            self.pos, self.q, self.k, self.cache = wl.rope_inputs(device)
            self.T = self.pos.shape[0]
            self.bytes = self.T * (2 * 2 * (self.q.shape[1] + self.k.shape[1]) + 4 * 128 + 4)
            self.cfg = {"workload": "config 3 rope q[T,32,128] k[T,8,128]", "tokens": self.T,
                        "l2": "inputs larger than L2 (689 MB)"}
        elif name in ("rope_append", "rope_append_small"):
            # _small: the same tokens with cached prefixes below 4096 positions, so the page pool (and the
            # device memory an ncu capture saves and restores) is about 20 times smaller
            self.pb, self.qkv, self.cache, self.kc, self.vc = wl.rope_append_inputs(
                device, max_offset=4096 if name == "rope_append_small" else 65536)
            Hq, Hkv, D = 32, 8, 128
            self.q = self.qkv[:, : Hq * D]
            self.k = self.qkv[:, Hq * D: (Hq + Hkv) * D]
            self.v = self.qkv[:, (Hq + Hkv) * D:]
            self.kv_indices = self.pb.kv_indices.contiguous()
            self.T = self.qkv.shape[0]
            # q read+write, k read + write back + cache write, v read + cache write, cos|sin row,
            # position, batch index, page-table entry
            self.bytes = self.T * (2 * 2 * Hq * D + 3 * 2 * Hkv * D + 2 * 2 * Hkv * D + 4 * D + 12)
            self.cfg = {"workload": "config 3 rope q[T,32,128] k[T,8,128] + paged KV append (NHD, 16-token pages)"
                        + (", cached prefixes < 4096" if name == "rope_append_small" else ""),
                        "tokens": self.T, "pages": self.pb.num_pages, "l2": "inputs larger than L2"}
            self.name = self.dominant = "rope_append"
        elif name == "embed_fill":
            # A configuration-5 step's ids (int64, as the runner keeps them): the 256 decode rows hold
            # placeholders -1 - r for the previous step's samples (model_runner.py:149-154).
            ids, _ = wl.chain_host_inputs()
            ids[:256] = -1 - torch.arange(256)
            self.ids_init = ids.to(device)
            self.ids = self.ids_init.clone()
            self.last = torch.randint(0, cs.vocab_size, (256,), generator=torch.Generator().manual_seed(8),
                                      dtype=torch.int64).to(device)
            self.table = wl._normal((cs.vocab_size, cs.hidden_size), wl._gen(device, 3), device, torch.bfloat16,
                                    std=0.02)
            self.T = self.ids.shape[0]
            self.out = torch.empty(self.T, self.table.shape[1], dtype=self.table.dtype, device=device)
            # gather rows in and out, ids read and written back, the placeholders' samples
            self.bytes = 2 * 2 * self.T * self.table.shape[1] + 2 * 8 * self.T + 8 * 256
            self.cfg = {"workload": "chain-shape embedding gather with the runner's placeholder substitution (f4)",
                        "tokens": self.T, "hidden": self.table.shape[1], "placeholders": 256,
                        "l2": "table 3.2 GB > L2; output 107 MB"}
        elif name == "embed":
            self.table, self.ids = wl.embed_inputs(device)
            self.T = self.ids.shape[0]
            self.out = torch.empty(self.T, self.table.shape[1], dtype=self.table.dtype, device=device)
            self.bytes = 2 * 2 * self.T * self.table.shape[1] + 4 * self.T
            self.cfg = {"workload": "config 4 embedding gather", "tokens": self.T, "hidden": self.table.shape[1],
                        "l2": "table 1.34 GB > L2; output 168 MB > L2"}
        else:
            raise ValueError(name)
        self.tokens = self.T
        self.global_tokens = self.T * dist.world
        self.layers = 1
        self.cfg["l2"] = "flushed between launches (write, then read, of 2x L2; outside the events); " + self.cfg["l2"]
        self.flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)
        self.per_launch_value = True  # tokens / mean launch time (the flush between launches is not timed)

    def step(self, dom_events=None):
        st = torch.cuda.current_stream()
        # Evict the previous launch's data from L2 outside the launch's events: a 256 MB write, then a
        # read of the same buffer so that the lines L2 is left holding are clean (no write-back of the
        # flush itself lands inside the timed launch). Each launch then reads its inputs from HBM.
        self.flush.zero_()
        self.flush_sum = self.flush.sum(dtype=torch.int32)
        if self.name == "embed_fill":
            self.ids.copy_(self.ids_init)  # the placeholders again (the op resolves them in place)
        if dom_events is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
        o, n = self.o, self.name
        if n == "norm":
            o.fused_add_rmsnorm(self.x, self.r, self.w, self.eps, enable_pdl=True)
        elif n == "norm_fp8":
            o.fused_add_rmsnorm_quant(self.out, self.x, self.r, self.w, self.scale, self.eps, enable_pdl=True)
        elif n == "silu":
            o.silu_and_mul(self.x, out=self.out, enable_pdl=True)
        elif n == "silu_fp8":
            o.silu_and_mul_quant(self.x, self.scale, out=self.out, enable_pdl=True)
        elif n == "rope":
            o.apply_rope_with_cos_sin_cache_inplace(self.pos, self.q, self.k, 128, self.cache, is_neox=True)
        elif n == "rope_qscale":
            self.q_scaled = o.apply_rope_and_llama4_query_scale_inplace(
                self.pos, self.q, self.k, 128, self.cache, self.beta, self.orig, is_neox=True)
        elif n == "rope_append":
            pb = self.pb
            o.apply_rope_and_append_paged_kv_cache(pb.positions, self.q, self.k, self.v, 128, self.cache,
                                                   pb.batch_indices, (self.kc, self.vc), self.kv_indices,
                                                   pb.kv_indptr, pb.kv_last_page_len)
        elif n == "embed":
            o.embedding_out(self.out, self.ids, self.table)
        elif n == "embed_fill":
            self.out = o.embedding_fill_placeholders(self.ids, self.table, self.last)
        if dom_events is not None:
            e1.record(st)
            dom_events.append((e0, e1))

    def launches_per_step(self) -> int:
        return 1

    def step_bytes(self) -> int:
        return self.bytes

    def dominant_bytes_per_launch(self) -> int:
        return self.bytes

    def config(self) -> dict:
        return dict(self.cfg, parallelism="token-sharded dp")


# --------------------------------------------------------------------------------------------------
# CPU arm: the reference's CPU path on a token sample of the chain.
# --------------------------------------------------------------------------------------------------
class CpuChainSample:
    """The chain on `tokens` sampled tokens (all layers), inputs on the host: the embedding through
    torch's own CPU embedding (the reference's nn.Embedding path, devstral2.py:260, :282), and the
    norms, rope and SiLU-mul through the C oracle (the reference has no CPU implementation of those:
    its kernels are flashinfer's, CUDA-only)."""

    def __init__(self, tokens: int, layers: int, seed: int = 4):
        import oracle
        from mas_b200 import workloads as wl

        s = wl.CHAIN_SHAPE
        self.s, self.oracle, self.layers, self.tokens = s, oracle, layers, tokens
        ids, pos = wl.chain_host_inputs(seed=seed)
        sel = torch.linspace(0, ids.shape[0] - 1, tokens).long()
        self.ids, self.pos = ids[sel].contiguous(), pos[sel].contiguous()
        g = torch.Generator().manual_seed(seed)
        # only the table rows the sample touches are materialised (the rest are never read)
        uniq, inv = torch.unique(self.ids, return_inverse=True)
        self.table = (torch.randn(uniq.shape[0], s.hidden_size, generator=g) * 0.02).to(torch.bfloat16)
        self.local_ids = inv.to(torch.int64)
        self.attn = torch.randn(tokens, s.hidden_size, generator=g).to(torch.bfloat16)
        self.qkv = torch.randn(tokens, s.qkv_size, generator=g).to(torch.bfloat16)
        self.gate_up = torch.randn(tokens, 2 * s.intermediate_size, generator=g).to(torch.bfloat16)
        self.act = torch.empty(tokens, s.intermediate_size, dtype=torch.bfloat16)
        self.w_in = (1 + 0.1 * torch.randn(layers, s.hidden_size, generator=g)).to(torch.bfloat16)
        self.w_post = (1 + 0.1 * torch.randn(layers, s.hidden_size, generator=g)).to(torch.bfloat16)
        from mas_b200.rope_cache import plain_cos_sin_cache

        self.cache = plain_cos_sin_cache(s.head_dim, s.max_position_embeddings, s.rope_theta)

    def step(self):
        o, s = self.oracle, self.s
        hidden = torch.nn.functional.embedding(self.local_ids, self.table)
        residual = torch.zeros_like(hidden)
        q = self.qkv[:, : s.q_size]
        k = self.qkv[:, s.q_size: s.q_size + s.kv_size]
        for l in range(self.layers):
            o.fused_add_rmsnorm(hidden, residual, self.w_in[l], s.rms_norm_eps)
            o.apply_rope_with_cos_sin_cache_inplace(self.pos, q, k, s.head_dim, self.cache)
            o.fused_add_rmsnorm(self.attn, residual, self.w_post[l], s.rms_norm_eps)
            o.silu_and_mul(self.gate_up, out=self.act)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def calibrate_cpu_tokens(layers: int, target_s: float) -> int:
    """Tokens whose step takes about target_s on this host (the probe's first step, which pays for
    thread start-up and first-touch page faults, is not used)."""
    probe = CpuChainSample(64, layers)
    probe.step()
    t0 = time.perf_counter()
    probe.step()
    per_token = (time.perf_counter() - t0) / 64
    return int(max(16, min(4352, target_s / max(per_token, 1e-9))))


def time_cpu_chain(tokens: int, layers: int, reps: int) -> tuple[float, list[float]]:
    w = CpuChainSample(tokens, layers)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        w.step()
        times.append(time.perf_counter() - t0)
    return tokens / statistics.median(times), times


# --------------------------------------------------------------------------------------------------
# Arms.
# --------------------------------------------------------------------------------------------------
def run_reference_arm(args, world: int, rank: int) -> None:
    """The reference's CPU path on this host (all threads), rank 0 only, on the GPU arms' config.

    Nothing here loads this package's CUDA libraries: workloads, chain shapes and the cos/sin cache
    are host-only modules, and the arithmetic is the C oracle's and torch's."""
    if rank != 0:
        return
    if args.workload != "chain":
        print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm is defined for the chain workload"}))
        return
    import oracle

    cores = host_cores()
    oracle.set_num_threads(cores)
    layers = args.layers or 88
    per_step_budget = max(0.5, min(4.0, 150.0 / max(1, args.steps + args.warmup)))
    tokens = calibrate_cpu_tokens(layers, per_step_budget)
    w = CpuChainSample(tokens, layers)
    for _ in range(args.warmup):
        w.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        w.step()
    dt = (time.perf_counter() - t0) / args.steps
    value = tokens / dt
    from mas_b200.chain import LayerChain

    chain = LayerChain(w.s, layers=layers)
    sample = (f"{tokens} of the 4352 tokens of a step, all {layers} layers, per step; embedding by torch's CPU "
              f"embedding, norms/rope/SiLU-mul by the C oracle (OpenMP, {cores} threads)")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": chain_config(layers, 4352, 4352 * world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "hbm_gbs_equivalent": chain.step_bytes(tokens) / dt / 1e9,
    }
    print(json.dumps(line))


def _flush_queue_then(fn):
    """Runs fn() with a spin kernel ahead of it in the stream, so that the host queues the launches of
    fn() while the GPU is still busy: the events then time the device, not the Python launch rate."""
    torch.cuda._sleep(SLEEP_CYCLES)
    return fn()


def time_steps(step, steps: int, warmup: int, dist: Dist, device, dom=None, clocks: bool = False):
    """Device time per step (ms), max over ranks, of `steps` calls of step() after `warmup` calls;
    barrier + synchronize on both sides. Returns (ms, clocks summary or None)."""
    st = torch.cuda.current_stream()
    for _ in range(warmup):
        step(None)
    torch.cuda.synchronize()
    clk = Clocks(device.index) if clocks else None
    if clk is not None:
        clk.__enter__()
        time.sleep(0.25)
    try:
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def region():
            e0.record(st)
            for _ in range(steps):
                step(dom)
            e1.record(st)

        _flush_queue_then(region)
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        if clk is not None:
            clk.__exit__(None, None, None)
    ms = dist.max(e0.elapsed_time(e1) / steps, device)
    return ms, (clk.summary() if clk is not None else None)


def time_e2e(w: ChainWorkload, steps: int, warmup: int, dist: Dist, device) -> float:
    """ms per step through the public API with host inputs and outputs (ChainWorkload.e2e_step)."""
    st = torch.cuda.current_stream()
    w.e2e_setup()
    for _ in range(max(1, warmup // 2)):
        w.e2e_step()
    w.e2e_finish()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def region():
        a.record(st)
        for _ in range(steps):
            w.e2e_step()
        w.e2e_finish()
        b.record(st)

    _flush_queue_then(region)
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(a.elapsed_time(b) / steps, device)


def time_graph(w: ChainWorkload, steps: int, warmup: int, dist: Dist, device) -> float:
    """ms per step of the chain captured once into a CUDA graph and replayed, as the reference's
    runner replays steps of up to 512 tokens (model_runner.py:20, :87-119); max over ranks."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            w.step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        w.step()
    try:
        return time_steps(lambda _d: graph.replay(), steps, warmup, dist, device)[0]
    finally:
        torch.cuda.synchronize()
        del graph


def check_words(impl: str, device) -> dict:
    """The library's fault and status words after a timed region (mas arm), read and cleared."""
    if impl != "mas":
        return {}
    import mas_b200

    return {"fault_word": mas_b200.read_fault_word(device.index, clear=True),
            "status_word": mas_b200.read_status(device)}


def arm_record(w: ChainWorkload, args, dist: Dist, device, impl: str, e2e: bool = True) -> dict:
    """value, ms per step, e2e and clocks of one arm on the workload's current inputs."""
    ms, clk = time_steps(w.step, args.steps, args.warmup, dist, device, clocks=True)
    rec = {"value": w.tokens * dist.world / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "clocks": clk}
    if e2e and not args.no_e2e:
        e_ms = time_e2e(w, args.steps, args.warmup, dist, device)
        h2d, d2h = w.e2e_bytes()
        rec["e2e"] = {"value": w.tokens * dist.world / (e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e_ms,
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    rec.update(check_words(impl, device))
    return rec


def strong_and_small(w: ChainWorkload, args, dist: Dist, device, arms: dict) -> tuple[dict, dict]:
    """Strong scaling (one fixed 4352-token step split into N contiguous token ranges, positions
    alongside) and small steps (T = 64, 256, 512 tokens, replayed from a CUDA graph), per arm."""
    from mas_b200 import workloads as wl

    ids, pos = wl.chain_host_inputs(replicas=1)
    T = ids.shape[0]
    s, e = shard(T, dist.world, dist.rank)
    strong = {"global_tokens": T, "tokens_per_gpu": [shard(T, dist.world, r)[1] - shard(T, dist.world, r)[0]
                                                      for r in range(dist.world)],
              "timing": "eager launches, max over ranks"}
    small = {"timing": "one step captured into a CUDA graph and replayed, max over ranks",
             "tokens": [64, 256, 512]}
    for name, ops in arms.items():
        w.chain_ops = ops
        v = w.view(e - s, ids[s:e], pos[s:e])
        ms, _ = time_steps(v.step, args.steps, args.warmup, dist, device)
        strong[name] = {"value": T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms}
        for n in small["tokens"]:
            v = w.view(n, ids[:n], pos[:n])
            ms = time_graph(v, args.steps, args.warmup, dist, device)
            small.setdefault(name, {})[str(n)] = {"value": n * dist.world / (ms / 1e3), "unit": "tokens/s",
                                                  "ms_per_step": ms}
    return strong, small


def run_gpu_arm(args, dist: Dist) -> None:
    device = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(device)
    mas = None
    if args.impl == "flashinfer":
        ops = FlashinferOps()
    else:
        import mas_b200

        mas = ops = mas_b200.ops
        mas_b200.prepare_device(device.index)
        mas_b200.read_fault_word(device.index, clear=True)
        mas_b200.read_status(device)
    layers = args.layers or 88
    chain = args.workload in ("chain", "chain_fp8")
    if chain:
        from mas_b200 import workloads as wl

        ids, pos = wl.chain_host_inputs(replicas=dist.world)
        per = ids.shape[0] // dist.world
        s, e = dist.rank * per, (dist.rank + 1) * per
        w = ChainWorkload(device, ops, layers, ids[s:e], pos[s:e], seed=4 + dist.rank,
                          quant=args.workload == "chain_fp8")
        w.global_tokens = per * dist.world
    else:
        w = OpWorkload(args.workload, device, dist, ops)

    # ---- device-resident timed region -----------------------------------------------------------
    dom = [] if not args.no_kernel_events else None
    ms, clocks = time_steps(w.step, args.steps, args.warmup, dist, device, dom=dom, clocks=True)
    words = check_words(args.impl, device)
    dom_ms = statistics.fmean(a.elapsed_time(b) for a, b in dom) if dom else None
    if dom_ms is not None:
        dom_ms = dist.max(dom_ms, device)

    # ---- end-to-end through the public API with host inputs/outputs --------------------------------
    e2e = None
    if chain and not args.no_e2e:
        e2e_ms = time_e2e(w, args.steps, args.warmup, dist, device)
        h2d, d2h = w.e2e_bytes()
        e2e = {"value": w.global_tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "path": "public API (mas_b200 ops), pinned host ids+positions in, residual stream out "
                       "(copy stream, double-buffered: step i's copy out overlaps step i+1's kernels)"}
        for k, v in check_words(args.impl, device).items():
            words[k] = words.get(k, 0) | v

    # ---- the reference's GPU kernels on the same inputs, the other chain form, strong/small steps ----
    subs = {}
    if chain and args.impl == "mas" and not args.no_compare:
        fi = FlashinferOps()
        w.chain_ops = fi
        subs["flashinfer"] = dict(arm_record(w, args, dist, device, "flashinfer"),
                                  kernels="flashinfer 0.6.11.post2 (norm, rope, silu) + aten index_select (gather)")
        other = not w.quant
        w.set_quant(other)
        rec = {"config": (chain_fp8_config if other else chain_config)(layers, w.tokens, w.global_tokens)}
        w.chain_ops = mas
        rec["mas"] = arm_record(w, args, dist, device, "mas")
        w.chain_ops = fi
        rec["flashinfer"] = arm_record(w, args, dist, device, "flashinfer")
        subs["chain_fp8" if other else "chain_bf16"] = rec
        w.set_quant(not other)
        subs["strong_scaling"], subs["small_steps"] = strong_and_small(w, args, dist, device,
                                                                       {"mas": mas, "flashinfer": fi})
        w.chain_ops = mas
        for k in ("fault_word", "status_word"):
            words[k] = words.get(k, 0) | rec["mas"].get(k, 0)

    # ---- CPU baseline (rank 0, N = 1) ----------------------------------------------------------------
    cpu = None
    if args.workload == "chain" and dist.world == 1 and not args.no_cpu_baseline and args.impl != "flashinfer":
        import oracle

        cores = host_cores()
        oracle.set_num_threads(cores)
        tokens = calibrate_cpu_tokens(layers, 4.0)
        value_cpu, times = time_cpu_chain(tokens, layers, reps=3)
        cpu = {"value": value_cpu, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{tokens} of {w.tokens} tokens, all {layers} layers, median of 3 steps "
                         f"({sum(times):.1f} s of CPU work); embedding by torch's CPU embedding, the rest by "
                         f"the C oracle"}

    # ---- outputs gathered for checking (NCCL, outside every timed region) ------------------------
    gathered = None
    if chain:
        sample = w.sample_step()
        per_rank = dist.gather_objects({"rank": dist.rank, "digest": w.digest(), "sample": sample})
        if dist.rank == 0:
            checks = []
            for r in per_rank:
                ulps = oracle_check(r["sample"], w.shape.rms_norm_eps)
                checks.append({"rank": r["rank"], "tokens_checked": int(r["sample"]["tokens"].numel()),
                               "max_ulp": ulps})
            worst = max(max(c["max_ulp"].values()) for c in checks)
            gathered = {"ranks": dist.world, "digests": [r["digest"] for r in per_rank],
                        "tokens_total": sum(r["digest"]["tokens"] for r in per_rank),
                        "oracle_check": {"per_rank": checks, "worst_ulp": worst, "bound_ulp": CHECK_BOUND_ULP,
                                         "ok": worst <= CHECK_BOUND_ULP,
                                         "how": "8 evenly spaced tokens per rank, one full step (all layers) "
                                                "after the timed regions, gathered to rank 0 over NCCL and "
                                                "replayed by the C oracle"}}
        for k, v in check_words(args.impl, device).items():
            words[k] = words.get(k, 0) | v

    if dist.rank != 0:
        return
    peak, peak_kind = measured_peak()
    if w.per_launch_value and dom_ms is not None:
        ms = dom_ms  # per-op workloads: the launch itself (the L2 flush between launches is untimed)
    step_s = ms / 1e3
    value = w.global_tokens / step_s
    gbs = w.step_bytes() / step_s / 1e9  # per GPU
    roof = None
    if dom_ms is not None:
        achieved = w.dominant_bytes_per_launch() / (dom_ms / 1e3) / 1e9
        traffic, traffic_src = args.traffic, "--traffic" if args.traffic is not None else None
        if traffic is None and args.impl == "mas" and args.workload in NCU_TRAFFIC:
            traffic, traffic_src = NCU_TRAFFIC[args.workload]
        roof = {"bound": "hbm", "kernel": w.dominant, "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
                "traffic": traffic, "traffic_source": traffic_src, "bytes_per_launch": w.dominant_bytes_per_launch(),
                "avg_launch_us": dom_ms * 1e3, "launches_timed": len(dom)}
        if chain and args.impl == "mas" and args.workload in NCU_IN_CHAIN:
            us, src = NCU_IN_CHAIN[args.workload]
            roof["ncu_in_chain_us"] = us
            roof["ncu_in_chain_frac"] = w.dominant_bytes_per_launch() / (us / 1e6) / 1e9 / peak
            roof["ncu_in_chain_source"] = src
    if chain:
        cfg = (chain_fp8_config if w.quant else chain_config)(layers, w.tokens, w.global_tokens)
    else:
        cfg = w.config()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, random ids/positions)",
        "config": cfg,
        "hbm_gbs_per_gpu": gbs, "hbm_frac_of_peak": gbs / peak, "hbm_peak_kind": peak_kind,
        "hbm_frac_of_nominal_8tbs": gbs / NOMINAL_HBM_GBS,
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": (w.launches_per_step() * args.steps) if args.impl == "mas" else 0,
        "clocks": clocks,
    }
    line.update(words)
    line.update(subs)
    if gathered is not None:
        line["gathered_outputs"] = gathered
    if args.impl != "mas":
        line["impl"] = args.impl
    print(json.dumps(line), flush=True)
    bad = [k for k in ("fault_word", "status_word") if line.get(k)]
    if bad or (gathered is not None and not gathered["oracle_check"]["ok"]):
        print(f"bench: check failed: {bad or 'oracle check'}", file=sys.stderr)
        raise SystemExit(1)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["mas", "reference", "flashinfer"], default="mas")
    ap.add_argument("--workload", choices=["chain", "norm", "norm_fp8", "silu", "rope", "embed", "norm_chain",
                                           "silu_chain", "rope_chain", "silu_fp8", "silu_fp8_chain", "rope_append",
                                           "chain_fp8", "norm_fp8_chain", "embed_fill", "rope_qscale_chain",
                                           "rope_append_small"],
                    default="chain")
    ap.add_argument("--layers", type=int, default=0, help="chain layers (default 88)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-compare", action="store_true",
                    help="chain: skip the flashinfer, other-form, strong-scaling and small-step sub-records")
    ap.add_argument("--no-kernel-events", action="store_true", help="time the region without per-launch events")
    ap.add_argument("--traffic", type=float, default=None, help="ncu DRAM bytes per dominant launch, if known")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        # CPU only: no process group; under torchrun rank 0 runs and the other ranks exit at once.
        run_reference_arm(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    dist = Dist()
    try:
        run_gpu_arm(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
