"""Pins the oracle against outputs of the reference's actual kernels (flashinfer 0.6.11.post2 on a B200).

tests/golden/flashinfer_golden.npz was produced by tests/golden/gen_flashinfer_golden.py, which calls
flashinfer with the arguments of the reference's call sites (devstral2.py:163-166, :224, :241-252,
:305-307) on small seeded inputs. The oracle, run here on the CPU on the same inputs, must agree with
flashinfer: bit-exact for the residual and the untouched parts of qkv, <= 1 ulp (bf16/fp16) or one
e4m3 step for the normalised, activated and rotated outputs. The near-cancellation rope cases fix
the fp32 evaluation order of the rotation (one fused multiply-add after a rounded product).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from parity import assert_bits_equal, assert_ulp

Z = np.load(Path(__file__).resolve().parent / "golden" / "flashinfer_golden.npz")


def _t(a: np.ndarray, dtype) -> torch.Tensor:
    if dtype == torch.float8_e4m3fn:
        return torch.from_numpy(a.astype(np.uint8)).view(dtype)
    return torch.from_numpy(a.astype(np.int16)).view(dtype)


def _cases(prefix: str) -> list[str]:
    return sorted({k.split("_")[1] for k in Z.files if k.startswith(prefix + "_")})


def test_fixture_provenance():
    assert str(Z["flashinfer_version"]) == "0.6.11.post2"
    assert "B200" in str(Z["gpu"])


@pytest.mark.parametrize("name", _cases("norm"))
def test_norm_matches_flashinfer(name):
    dtype = torch.float16 if str(Z[f"norm_{name}_dtype"]) == "torch.float16" else torch.bfloat16
    x, r, w = (_t(Z[f"norm_{name}_{k}"], dtype) for k in ("x", "r", "w"))
    H = int(Z[f"norm_{name}_H"])
    xo, ro = x.clone(), r.clone()
    oracle.fused_add_rmsnorm(xo[:, :H], ro[:, :H], w, 1e-5)
    assert_bits_equal(ro, _t(Z[f"norm_{name}_rout"], dtype), f"{name} residual")
    assert_ulp(xo, _t(Z[f"norm_{name}_xout"], dtype), what=f"{name} output")


@pytest.mark.parametrize("name", _cases("siluq"))
def test_silu_quant_matches_reference_pair(name):
    """silu_and_mul -> the reference's compiled quantize_fp8 (devstral2.py:93-95) on a B200: the
    oracle's activation within 1 ulp and its e4m3 bytes within one step (bit-exact where the
    activations agree)."""
    xin = _t(Z[f"siluq_{name}_in"], torch.bfloat16)
    scale = float(Z[f"siluq_{name}_scale"])
    act = _t(Z[f"siluq_{name}_act"], torch.bfloat16)
    want = _t(Z[f"siluq_{name}_out"], torch.float8_e4m3fn)
    got = oracle.silu_and_mul_quant(xin, scale)
    assert_ulp(oracle.silu_and_mul(xin), act, what=f"siluq {name} activation")
    assert_ulp(got, want, what=f"siluq {name} e4m3")
    # from the reference's own activation the oracle's quantisation is exact
    same = (oracle.silu_and_mul(xin).view(torch.int16) == act.view(torch.int16))
    assert torch.equal(got.view(torch.uint8)[same], want.view(torch.uint8)[same])


@pytest.mark.parametrize("name", _cases("quant"))
def test_norm_quant_matches_flashinfer(name):
    x, r, w = (_t(Z[f"quant_{name}_{k}"], torch.bfloat16) for k in ("x", "r", "w"))
    out = torch.empty(x.shape, dtype=torch.float8_e4m3fn)
    xo, ro = x.clone(), r.clone()
    oracle.fused_add_rmsnorm_quant(out, xo, ro, w, float(Z[f"quant_{name}_scale"]), 1e-5)
    assert_bits_equal(ro, _t(Z[f"quant_{name}_rout"], torch.bfloat16), f"{name} residual")
    assert_bits_equal(xo, _t(Z[f"quant_{name}_xafter"], torch.bfloat16), f"{name} input unchanged")
    assert_ulp(out, _t(Z[f"quant_{name}_out"], torch.float8_e4m3fn), what=f"{name} e4m3")


@pytest.mark.parametrize("name", _cases("silu"))
def test_silu_matches_flashinfer(name):
    dtype = torch.float16 if name == "sfp16" else torch.bfloat16
    xin = _t(Z[f"silu_{name}_in"], dtype)
    assert_ulp(oracle.silu_and_mul(xin), _t(Z[f"silu_{name}_out"], dtype), what=f"silu {name}")


@pytest.mark.parametrize("name", sorted({k[len("rope_"):-len("_qkv")] for k in Z.files
                                         if k.startswith("rope_") and k.endswith("_qkv")}))
def test_rope_matches_flashinfer(name):
    qkv = _t(Z[f"rope_{name}_qkv"], torch.bfloat16)
    cache = torch.from_numpy(Z[f"rope_{name}_cache"])
    pos = torch.from_numpy(Z[f"rope_{name}_pos"])
    Hq, Hkv, D, neox = (int(v) for v in Z[f"rope_{name}_dims"])
    qo = qkv.clone()
    oracle.apply_rope_with_cos_sin_cache_inplace(pos, qo[:, : Hq * D], qo[:, Hq * D: (Hq + Hkv) * D], D, cache,
                                                 is_neox=bool(neox))
    want = _t(Z[f"rope_{name}_out"], torch.bfloat16)
    assert_bits_equal(qo[:, (Hq + Hkv) * D:], want[:, (Hq + Hkv) * D:], f"{name} v")
    stats = assert_ulp(qo, want, what=f"rope {name}")
    if name.startswith("rcancel"):
        # the evaluation order is pinned: every element, cancelling ones included, is identical
        assert stats["max_ulp"] == 0, stats


def _i(a) -> torch.Tensor:
    return torch.from_numpy(np.asarray(a))


@pytest.mark.parametrize("name", _cases("append"))
def test_append_matches_flashinfer(name):
    """flashinfer.page.append_paged_kv_cache with the runner's metadata: the oracle's copy is exact."""
    g = lambda k: Z[f"append_{name}_{k}"]  # noqa: E731
    k, v = _t(g("k"), torch.bfloat16), _t(g("v"), torch.bfloat16)
    kc, vc = _t(g("kc"), torch.bfloat16).clone(), _t(g("vc"), torch.bfloat16).clone()
    st = oracle.append_paged_kv_cache(k, v, _i(g("bi")), _i(g("pos")), (kc, vc), _i(g("table")).flatten(),
                                      _i(g("indptr")), kv_layout="HND" if int(g("hnd")) else "NHD")
    assert st == 0
    assert_bits_equal(kc, _t(g("kcout"), torch.bfloat16), f"{name} k cache")
    assert_bits_equal(vc, _t(g("vcout"), torch.bfloat16), f"{name} v cache")


def test_rope_append_q_scale_matches_reference_sequence():
    """Rope -> append -> llama-4 query scale as Devstral2Attention.forward runs them (flashinfer +
    eager torch on a B200) against the oracle's fused form: k/v caches and k within 1 ulp (exact
    where the rotated k agrees), v untouched, q scaled within 1 ulp."""
    Hq, H, D = (int(x) for x in Z["rapp_dims"])
    qkv = _t(Z["rapp_qkv"], torch.bfloat16).clone()
    kc, vc = _t(Z["rapp_kc"], torch.bfloat16).clone(), _t(Z["rapp_vc"], torch.bfloat16).clone()
    st = oracle.rope_append_paged_kv_cache(
        _i(Z["rapp_pos"]), qkv[:, : Hq * D], qkv[:, Hq * D: (Hq + H) * D], qkv[:, (Hq + H) * D:], D,
        _i(Z["rapp_cache"]), _i(Z["rapp_bi"]), (kc, vc), _i(Z["rapp_table"]).flatten(), _i(Z["rapp_indptr"]),
        beta=float(Z["rapp_beta"]), original_max_position_embeddings=int(Z["rapp_orig"]))
    assert st == 0
    ref = _t(Z["rapp_qkvout"], torch.bfloat16)
    assert_ulp(qkv[:, Hq * D:], ref[:, Hq * D:], what="k rotated, v untouched")
    assert_ulp(qkv[:, : Hq * D], _t(Z["rapp_qscaled"], torch.bfloat16), what="q rotated and scaled")
    assert_ulp(kc, _t(Z["rapp_kcout"], torch.bfloat16), what="k cache")
    assert_bits_equal(vc, _t(Z["rapp_vcout"], torch.bfloat16), "v cache")
