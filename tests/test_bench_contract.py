"""The benchmark's static contract, checked without a GPU.

* every DRAM-traffic figure bench.py reports as `roofline.traffic` comes from a committed ncu
  summary under profiles/ that holds the read and write counts it adds up;
* every profile summary gives the command that produced it, with ncu's clock control off;
* the HBM peak is read from MEASURED_PEAKS.json when present and labelled as the fallback otherwise.
"""
from __future__ import annotations

import itertools
import json
import re
from pathlib import Path

import pytest

import bench

ROOT = Path(__file__).resolve().parent.parent
PROFILES = sorted((ROOT / "profiles").glob("*.md"))


@pytest.mark.parametrize("workload", sorted(bench.NCU_TRAFFIC))
def test_traffic_figure_is_backed_by_a_profile(workload):
    traffic, source = bench.NCU_TRAFFIC[workload]
    text = (ROOT / source).read_text()
    exact = {int(m.replace(",", "")) for m in re.findall(r"\b\d{1,3}(?:,\d{3}){2,}\b", text)}
    mb = [float(m) for m in re.findall(r"(\d+\.\d) MB", text)]
    by_bytes = any(a + b == traffic for a, b in itertools.combinations(exact, 2))
    by_mb = any(abs((a + b) * 1e6 - traffic) <= 0.11e6 for a, b in itertools.permutations(mb, 2))
    assert by_bytes or by_mb, (workload, traffic, source)


def test_traffic_workloads_are_bench_workloads():
    src = (ROOT / "bench.py").read_text()
    arg = src[src.index('"--workload"'):]
    choices = arg[: arg.index("]")]  # the literal list of --workload choices
    for w in bench.NCU_TRAFFIC:
        assert f'"{w}"' in choices, w


@pytest.mark.parametrize("path", PROFILES, ids=lambda p: p.name)
def test_profile_names_its_command(path):
    text = path.read_text()
    assert "--clock-control none" in text, path.name
    assert "bench.py" in text, path.name
    assert len(text) < 8192, path.name  # short summaries, not raw reports


def test_measured_peak_source(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.measured_peak() == (bench.FALLBACK_HBM_GBS, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6500.5}))
    assert bench.measured_peak() == (6500.5, "measured")


def _oracle_sample(quant: bool, layers: int = 2, n: int = 2) -> dict:
    """A sample in the layout of ChainWorkload.sample_step, its outputs made by the oracle itself."""
    import torch

    import oracle
    from mas_b200 import workloads as wl

    s = wl.CHAIN_SHAPE
    g = torch.Generator().manual_seed(11)
    bf = torch.bfloat16
    inp = {"ids": torch.tensor([3, 9]), "table_rows": (torch.randn(n, s.hidden_size, generator=g) * 0.02).to(bf),
           "attn_out": torch.randn(n, s.hidden_size, generator=g).to(bf),
           "qkv": torch.randn(n, s.qkv_size, generator=g).to(bf),
           "gate_up": torch.randn(n, 2 * s.intermediate_size, generator=g).to(bf),
           "cache_rows": torch.rand(n, s.head_dim, generator=g),
           "w_in": (1 + 0.1 * torch.randn(layers, s.hidden_size, generator=g)).to(bf),
           "w_post": (1 + 0.1 * torch.randn(layers, s.hidden_size, generator=g)).to(bf),
           "act_scale": torch.tensor([0.05, 0.05, 0.0137])}
    hidden, residual = inp["table_rows"].clone(), torch.zeros(n, s.hidden_size, dtype=bf)
    attn, qkv = inp["attn_out"].clone(), inp["qkv"].clone()
    act = torch.empty(n, s.intermediate_size, dtype=bf)
    x8 = torch.empty(n, s.hidden_size, dtype=torch.float8_e4m3fn)
    act8 = torch.empty(n, s.intermediate_size, dtype=torch.float8_e4m3fn)
    pos = torch.arange(n, dtype=torch.int32)
    for l in range(layers):
        if quant:
            oracle.fused_add_rmsnorm_quant(x8, hidden, residual, inp["w_in"][l], 0.05, s.rms_norm_eps)
        else:
            oracle.fused_add_rmsnorm(hidden, residual, inp["w_in"][l], s.rms_norm_eps)
        oracle.apply_rope_with_cos_sin_cache_inplace(pos, qkv[:, : s.q_size], qkv[:, s.q_size: s.q_size + s.kv_size],
                                                     s.head_dim, inp["cache_rows"])
        if quant:
            oracle.fused_add_rmsnorm_quant(x8, attn, residual, inp["w_post"][l], 0.05, s.rms_norm_eps)
            oracle.silu_and_mul_quant(inp["gate_up"], float(inp["act_scale"][2]), out=act8)
        else:
            oracle.fused_add_rmsnorm(attn, residual, inp["w_post"][l], s.rms_norm_eps)
            oracle.silu_and_mul(inp["gate_up"], out=act)
    out = {"residual": residual, "qkv": qkv}
    out.update({"x_fp8": x8, "act_fp8": act8} if quant else {"hidden": hidden, "attn_out": attn, "act": act})
    return {"tokens": torch.arange(n), "quant": quant, "layers": layers, "inputs": inp, "outputs": out}


@pytest.mark.parametrize("quant", [False, True])
def test_oracle_check_of_sampled_rows(quant):
    """bench.oracle_check replays a gathered sample through the oracle: zero distance for the oracle's
    own outputs, and a planted one-step error in one output element is reported as exactly that."""
    import torch

    sample = _oracle_sample(quant)
    got = bench.oracle_check(sample, 1e-5)
    assert set(got) == set(sample["outputs"]) and max(got.values()) == 0, got
    name = "x_fp8" if quant else "act"
    t = sample["outputs"][name]
    bits = t.view(torch.uint8 if quant else torch.int16)
    bits[1, 5] += 1
    got = bench.oracle_check(sample, 1e-5)
    assert got[name] == 1 and max(v for k, v in got.items() if k != name) == 0, got


@pytest.mark.parametrize("workload", sorted(bench.NCU_IN_CHAIN))
def test_in_chain_time_is_backed_by_a_profile(workload):
    """The dominant kernel's in-chain mean (roofline.ncu_in_chain_us) is the mean of a committed
    ncu launch list of the bench's own command."""
    us, source = bench.NCU_IN_CHAIN[workload]
    text = (ROOT / source).read_text()
    assert f"{us:.2f}" in text, (workload, us, source)
    assert "gpu__time_duration.sum" in text and "--clock-control none" in text


def _maps_after(code: str) -> str:
    """/proc/self/maps of a fresh interpreter after running `code` (the repo root on sys.path)."""
    import subprocess
    import sys

    prog = f"import sys; sys.path.insert(0, {str(ROOT)!r})\n{code}\nprint(open('/proc/self/maps').read())"
    r = subprocess.run([sys.executable, "-c", prog], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_host_modules_do_not_map_the_cuda_library():
    maps = _maps_after("import mas_b200\nfrom mas_b200 import workloads, chain, rope_cache\n"
                       "rope_cache.plain_cos_sin_cache(128, 64, 1e6)")
    assert "libmas_b200" not in maps


def test_reference_arm_maps_only_the_oracle():
    """bench.py --impl reference times the reference's CPU path: the oracle and torch, nothing of
    this repository's CUDA code."""
    maps = _maps_after("import runpy, sys\n"
                       "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3', '--layers', '1']\n"
                       "runpy.run_path('bench.py', run_name='__main__')")
    assert "libmas_b200" not in maps and "liborc" in maps
    line = json.loads([l for l in maps.splitlines() if l.startswith("{")][-1])
    assert line["impl"] == "reference" and line["config"] == bench.chain_config(1, 4352, 4352)
