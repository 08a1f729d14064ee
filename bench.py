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
of the measured HBM peak. Multi-GPU (torchrun, one rank per GPU) is weak scaling: the global batch is
N mixed steps and rank r takes the r-th, a contiguous slice; no collective touches the data path.
NCCL only carries the barrier, the max-over-ranks of the timings and, after the timed regions, the
gather of each rank's output digest (parity of the chain itself is checked by
tests/test_gpu_chain.py against the oracle).

Reported alongside the device-resident `value`:
  e2e            the same step through the public API with the step's host inputs (token ids,
                 positions) copied from pinned memory and the result (the residual stream) copied
                 back to pinned memory on a second stream, overlapping the next step, all inside the
                 timed region;
  roofline       the dominant kernel's algorithmic bytes / its CUDA-event time, against the measured
                 HBM copy peak (MEASURED_PEAKS.json); in the timed region, events bracket its
                 launches in every 16th layer (both norms), so they barely perturb the step; `traffic`
                 is that kernel's DRAM bytes from an ncu capture (NCU_TRAFFIC, profiles/);
  cpu_baseline   the C oracle (tests' checker, a restatement of the reference's arithmetic) timed
                 on this host's cores on a token sample of the same workload (rank 0, N = 1);
  clocks         SM clock and throttle reasons sampled by nvidia-smi during the timed region;
  gathered_outputs  each rank's token count and output digest.

--impl reference times the reference's CPU path: the reference has no CPU implementation of norm,
silu or rope (its kernels are flashinfer's, CUDA-only), so this arm runs the C oracle port with all
host threads on a token sample (embedding included), rank 0 only. --impl flashinfer times the
reference's actual GPU kernels (flashinfer 0.6.11.post2, aten gather, the compiled quantize_fp8)
on the same workload.
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
    "chain": (214_014_208 + 156_158_976, "profiles/norm_row_chain_shape.md"),
    "norm_chain": (214_014_208 + 156_158_976, "profiles/norm_row_chain_shape.md"),
    "norm": (83_929_344 + 25_862_656, "profiles/norm_loop_config1.md"),
    "norm_fp8": (83_932_416 + 11_052_544, "profiles/ops_dram_traffic.md"),
    "silu": (1_073_793_792 + 484_039_168, "profiles/ops_dram_traffic.md"),
    "silu_fp8": (1_073_966_592 + 214_110_720, "profiles/ops_dram_traffic.md"),
    "embed": (163_652_608 + 116_655_104, "profiles/ops_dram_traffic.md"),
    "rope": (328_030_464 + 254_389_504, "profiles/ops_dram_traffic.md"),
    "rope_chain": (118_129_152 + 59_046_912, "profiles/rope_ring_chain_shape.md"),
    "silu_fp8_chain": (499_136_256 + 73_464_832, "profiles/silu_fp8_chain_shape.md"),
    "rope_append_small": (383_577_088 + 381_649_152, "profiles/rope_append_config3_small.md"),
}


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
def mas_ops():
    import mas_b200

    return mas_b200.ops


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
    from mas_b200 import workloads as wl

    s = wl.CHAIN_SHAPE
    return {"workload": "chain (config 5): embed + 88 x [RMSNorm+res, rope q/k, RMSNorm+res, SiLU-mul]",
            "hidden": s.hidden_size, "q_heads": s.num_attention_heads, "kv_heads": s.num_key_value_heads,
            "head_dim": s.head_dim, "intermediate": s.intermediate_size, "vocab": s.vocab_size, "layers": layers,
            "tokens_per_gpu": tokens_per_gpu, "global_tokens": global_tokens,
            "step_mix": "256 decode + 2 x 2048 prefill tokens per GPU", "norm": "bf16 fused_add_rmsnorm",
            "l2": "inputs larger than L2 (per-layer working set 1.84 GB)", "parallelism": "token-sharded dp"}


class ChainWorkload:
    name = "chain"
    dominant = "fused_add_rmsnorm"
    EVENT_EVERY = 16  # layers 8, 24, 40, 56, 72 carry events around both of their norms
    per_launch_value = False

    def __init__(self, device, dist: Dist, ops, layers: int, quant: bool = False):
        from mas_b200 import workloads as wl
        from mas_b200.chain import LayerChain

        self.quant = quant
        if quant:
            self.name, self.dominant = "chain_fp8", "fused_add_rmsnorm_quant"
        self.wl = wl
        self.shape = wl.CHAIN_SHAPE
        ids, pos = wl.chain_host_inputs(replicas=dist.world)
        per = ids.shape[0] // dist.world
        s, e = dist.rank * per, (dist.rank + 1) * per
        self.host_ids = ids[s:e].clone().pin_memory()
        self.host_pos = pos[s:e].clone().pin_memory()
        self.tokens = per
        self.global_tokens = ids.shape[0]
        self.b = wl.chain_buffers(self.host_ids, self.host_pos, device=device, seed=4 + dist.rank, layers=layers,
                                  quant=quant)
        self.chain = LayerChain(self.shape, quant=quant, layers=layers)
        self.chain_ops = ops
        self.layers = self.chain.layers
        self.host_out = torch.empty(self.b.residual.shape, dtype=self.b.residual.dtype).pin_memory()
        self._dom_events = None

    # the chain with a pluggable op namespace, optionally bracketing the dominant kernel with events
    def _step(self, dom_events=None):
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

    def step(self, dom_events=None):
        self._step(dom_events)

    def e2e_setup(self):
        """Two residual buffers and two pinned host outputs, alternating by step, and a copy stream."""
        b = self.b
        self._res = [b.residual, torch.empty_like(b.residual)]
        self._host_out = [self.host_out, torch.empty(self.host_out.shape, dtype=self.host_out.dtype).pin_memory()]
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
        self._step(None)
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
        """Makes the current stream wait for the last copy to the host (inside the timed region)."""
        torch.cuda.current_stream().wait_stream(self._copy_stream)

    def digest(self) -> dict:
        """This rank's output fingerprint (outside the timed region): its token count and the integer
        sums of the final residual and hidden bit patterns. Rank 0 of an N-GPU run processes the
        same step as a 1-GPU run, so with equal --steps/--warmup its digest equals the 1-GPU one."""
        b = self.b
        return {"tokens": int(self.tokens),
                "residual_bits_sum": int(b.residual.view(torch.int16).to(torch.int64).sum().item()),
                "hidden_bits_sum": int(b.hidden.view(torch.int16).to(torch.int64).sum().item())}

    def e2e_bytes(self) -> tuple[int, int]:
        return (self.host_ids.numel() * 8 + self.host_pos.numel() * 4,
                self.b.residual.numel() * self.b.residual.element_size())

    def launches_per_step(self) -> int:
        return 1 + 4 * self.layers

    def step_bytes(self) -> int:
        return self.chain.step_bytes(self.tokens)

    def dominant_bytes_per_launch(self) -> int:
        return (7 if self.quant else 8) * self.tokens * self.shape.hidden_size + 2 * self.shape.hidden_size

    def config(self) -> dict:
        cfg = chain_config(self.layers, self.tokens, self.global_tokens)
        if self.quant:
            cfg["workload"] = ("chain, fp8 form (the decoder layers' own calls): embed + 88 x [RMSNorm+res -> e4m3, "
                               "rope q/k, RMSNorm+res -> e4m3, SiLU-mul -> e4m3]")
            cfg["norm"] = "fused_add_rmsnorm_quant"
        return cfg


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
                        "tokens": self.T, "hidden": H, "l2": "inputs larger than L2"}
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
# CPU arm: the C oracle on a token sample of the chain.
# --------------------------------------------------------------------------------------------------
class CpuChainSample:
    """The oracle running the chain on `tokens` sampled tokens (all layers), inputs on the host."""

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
        hidden, _ = o.embedding(self.local_ids, self.table)
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
    probe = CpuChainSample(16, layers)
    t0 = time.perf_counter()
    probe.step()
    per_token = (time.perf_counter() - t0) / 16
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
def run_reference_arm(args, dist: Dist) -> None:
    """The reference's CPU path on this host (C oracle port, all threads), rank 0 only."""
    if dist.rank != 0:
        return
    import oracle

    cores = host_cores()
    oracle.set_num_threads(cores)
    layers = args.layers or 88
    if args.workload != "chain":
        print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm is defined for the chain workload"}))
        return
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
    s = w.s
    from mas_b200.chain import LayerChain

    chain = LayerChain(s, layers=layers)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": dict(chain_config(layers, 4352, 4352), tokens_sampled_per_step=tokens),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{tokens} of 4352 tokens per step, all {layers} layers, C oracle (OpenMP)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "hbm_gbs_equivalent": chain.step_bytes(tokens) / dt / 1e9,
    }
    print(json.dumps(line))


def run_gpu_arm(args, dist: Dist) -> None:
    device = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(device)
    if args.impl == "flashinfer":
        ops = FlashinferOps()
    else:
        ops = mas_ops()
        import mas_b200

        mas_b200.prepare_device(device.index)
    layers = args.layers or 88
    if args.workload in ("chain", "chain_fp8"):
        w = ChainWorkload(device, dist, ops, layers, quant=args.workload == "chain_fp8")
    else:
        w = OpWorkload(args.workload, device, dist, ops)

    st = torch.cuda.current_stream()
    for _ in range(args.warmup):
        w.step()
    torch.cuda.synchronize()

    # ---- device-resident timed region -----------------------------------------------------------
    dom = []
    with Clocks(device.index) as clocks:
        time.sleep(0.25)
        dist.barrier()
        torch.cuda.synchronize()
        # A spin kernel holds the GPU while the host queues the whole timed region, so the region
        # measures the device, not the Python launch rate.
        torch.cuda._sleep(SLEEP_CYCLES)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(st)
        for _ in range(args.steps):
            w.step(dom_events=dom if not args.no_kernel_events else None)
        e_end.record(st)
        torch.cuda.synchronize()
        dist.barrier()
    ms = e_start.elapsed_time(e_end) / args.steps
    ms = dist.max(ms, device)
    dom_ms = statistics.fmean(a.elapsed_time(b) for a, b in dom) if dom else None
    if dom_ms is not None:
        dom_ms = dist.max(dom_ms, device)

    # ---- end-to-end through the public API with host inputs/outputs --------------------------------
    e2e = None
    if args.workload in ("chain", "chain_fp8") and not args.no_e2e:
        w.e2e_setup()
        for _ in range(max(1, args.warmup // 2)):
            w.e2e_step()
        w.e2e_finish()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(SLEEP_CYCLES)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(args.steps):
            w.e2e_step()
        w.e2e_finish()
        b.record(st)
        torch.cuda.synchronize()
        dist.barrier()
        e2e_ms = dist.max(a.elapsed_time(b) / args.steps, device)
        h2d, d2h = w.e2e_bytes()
        e2e = {"value": w.global_tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
               "path": "public API (mas_b200 ops), pinned host ids+positions in, residual stream out "
                       "(copy stream, double-buffered: step i's copy out overlaps step i+1's kernels)"}

    # ---- CPU baseline (rank 0, N = 1) ----------------------------------------------------------------
    cpu = None
    if args.workload == "chain" and dist.world == 1 and not args.no_cpu_baseline and args.impl != "flashinfer":
        import oracle

        cores = host_cores()
        oracle.set_num_threads(cores)
        tokens = calibrate_cpu_tokens(layers, 3.0)
        value_cpu, times = time_cpu_chain(tokens, layers, reps=3)
        cpu = {"value": value_cpu, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{tokens} of {w.tokens} tokens, all {layers} layers, C oracle, median of 3 steps "
                         f"({sum(times):.1f} s of CPU work)"}

    # ---- outputs gathered for checking (NCCL, outside every timed region) ------------------------
    gathered = None
    if hasattr(w, "digest"):
        per_rank = dist.gather_objects(w.digest())
        gathered = {"ranks": dist.world, "per_rank": per_rank,
                    "tokens_total": sum(d["tokens"] for d in per_rank)}

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
                "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
                "traffic": traffic, "traffic_source": traffic_src, "bytes_per_launch": w.dominant_bytes_per_launch(),
                "avg_launch_us": dom_ms * 1e3, "launches_timed": len(dom)}
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations, random ids/positions)",
        "config": w.config(),
        "hbm_gbs_per_gpu": gbs, "hbm_frac_of_peak": gbs / peak, "hbm_peak_kind": peak_kind,
        "hbm_frac_of_nominal_8tbs": gbs / NOMINAL_HBM_GBS,
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": (w.launches_per_step() * args.steps) if args.impl == "mas" else 0,
        "clocks": clocks.summary(),
    }
    if gathered is not None:
        line["gathered_outputs"] = gathered
    if args.impl != "mas":
        line["impl"] = args.impl
    print(json.dumps(line))


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
    ap.add_argument("--no-kernel-events", action="store_true", help="time the region without per-launch events")
    ap.add_argument("--traffic", type=float, default=None, help="ncu DRAM bytes per dominant launch, if known")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        # CPU only: no process group; under torchrun rank 0 runs and the other ranks exit at once.
        run_reference_arm(args, Dist(backend="none"))
        return
    dist = Dist()
    try:
        run_gpu_arm(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
