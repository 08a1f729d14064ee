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
