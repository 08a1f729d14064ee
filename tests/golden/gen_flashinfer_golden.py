"""Generates golden fixtures from flashinfer 0.6.11.post2 -- the kernels the reference calls -- on a GPU.

    python tests/golden/gen_flashinfer_golden.py [out_dir]      (needs a CUDA GPU and flashinfer)

mini-agent-serve computes RMSNorm, SiLU-and-mul and rope through flashinfer (imports at
miniagentserve/models/devstral2/devstral2.py:18-23). This script calls those same functions with the
arguments the reference's call sites pass -- fused_add_rmsnorm (devstral2.py:305-307),
fused_add_rmsnorm_quant (:241-252), silu_and_mul (:224) and the compiled quantize_fp8 after it
(:93-95), apply_rope_with_cos_sin_cache_inplace on strided q/k views of one qkv row (:158-166),
append_paged_kv_cache with the runner's page-table metadata (:170-173, :289-290) and the llama-4
query scale (:175-179) -- on small seeded inputs, and saves inputs and outputs
(bf16/fp16 as int16 bit patterns, e4m3 as uint8) to flashinfer_golden.npz. The CPU tests pin the
oracle against these outputs; nothing in the product imports flashinfer.
"""
from __future__ import annotations

import sys
import traceback
from pathlib import Path

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def main(out_dir: Path) -> None:
    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(20261201)
    arrays: dict[str, np.ndarray] = {}
    failures: list[str] = []

    def rnd(*shape, scale=1.0, dtype=torch.bfloat16):
        return (torch.randn(*shape, generator=g) * scale).to(dtype)

    # ---- fused_add_rmsnorm (bf16 in place) ---------------------------------------------------
    try:
        from flashinfer.norm import fused_add_rmsnorm
        for name, T, H, stride, dtype in (("n5120", 6, 5120, 5120, torch.bfloat16),
                                           ("n12288", 3, 12288, 12288, torch.bfloat16),
                                           ("n1000", 5, 1000, 1000, torch.bfloat16),
                                           ("nstrided", 4, 2048, 3072, torch.bfloat16),
                                           ("nfp16", 4, 4096, 4096, torch.float16)):
            xb = rnd(T, stride, dtype=dtype)
            rb = rnd(T, stride, scale=2.0, dtype=dtype)
            w = (1 + 0.1 * torch.randn(H, generator=g)).to(dtype)
            x_d, r_d = xb.to(dev), rb.to(dev)
            fused_add_rmsnorm(x_d[:, :H], r_d[:, :H], w.to(dev), 1e-5, enable_pdl=True)
            torch.cuda.synchronize()
            arrays.update({f"norm_{name}_x": bits(xb), f"norm_{name}_r": bits(rb), f"norm_{name}_w": bits(w),
                           f"norm_{name}_H": np.array(H), f"norm_{name}_xout": bits(x_d),
                           f"norm_{name}_rout": bits(r_d), f"norm_{name}_dtype": np.array(str(dtype))})
    except Exception:
        failures.append("fused_add_rmsnorm: " + traceback.format_exc(limit=2))

    # ---- fused_add_rmsnorm_quant (fp8 e4m3 out) -------------------------------------------------
    try:
        from flashinfer.norm import fused_add_rmsnorm_quant
        for name, T, H, scale in (("q5120", 6, 5120, 0.05), ("q12288", 3, 12288, 0.005), ("q1000", 4, 1000, 0.5)):
            xb = rnd(T, H)
            rb = rnd(T, H)
            w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
            out = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
            x_d, r_d = xb.to(dev), rb.to(dev)
            s = torch.tensor(scale, dtype=torch.float32, device=dev)
            fused_add_rmsnorm_quant(out, x_d, r_d, w.to(dev), s, 1e-5, enable_pdl=True)
            torch.cuda.synchronize()
            arrays.update({f"quant_{name}_x": bits(xb), f"quant_{name}_r": bits(rb), f"quant_{name}_w": bits(w),
                           f"quant_{name}_scale": np.array(scale, dtype=np.float32),
                           f"quant_{name}_out": bits(out), f"quant_{name}_rout": bits(r_d),
                           f"quant_{name}_xafter": bits(x_d)})
    except Exception:
        failures.append("fused_add_rmsnorm_quant: " + traceback.format_exc(limit=2))

    # ---- silu_and_mul ------------------------------------------------------------------------------
    try:
        from flashinfer.activation import silu_and_mul
        for name, T, d, scale, dtype in (("s4096", 4, 4096, 1.0, torch.bfloat16), ("s8", 3, 8, 1.0, torch.bfloat16),
                                         ("swide", 2, 1024, 12.0, torch.bfloat16),
                                         ("sfp16", 3, 1024, 3.0, torch.float16)):
            xin = rnd(T, 2 * d, scale=scale, dtype=dtype)
            out = silu_and_mul(xin.to(dev), enable_pdl=True)
            torch.cuda.synchronize()
            arrays.update({f"silu_{name}_in": bits(xin), f"silu_{name}_out": bits(out)})
        # Gate values down to -100 (where 1 + exp(-v) passes 2^126 and then overflows): pins how the
        # fp32 quotient of the activation behaves at the edge of its range.
        gate = -torch.linspace(60.0, 100.0, 2048)
        up = 1 + torch.rand(2048, generator=g)
        xin = torch.cat([gate, up]).view(1, -1).to(torch.bfloat16)
        out = silu_and_mul(xin.to(dev), enable_pdl=True)
        torch.cuda.synchronize()
        arrays.update({"silu_sneg_in": bits(xin), "silu_sneg_out": bits(out)})
        # The silu output quantised for down_proj: FP8Linear.forward's quantize_fp8, the expression
        # `(x / scale).clamp(-FP8_MAX, FP8_MAX).to(FP8)` under torch.compile(dynamic=True)
        # (devstral2.py:93-95, :110-111), on flashinfer's silu output.
        fp8 = torch.float8_e4m3fn
        fp8_max = torch.finfo(fp8).max

        @torch.compile(dynamic=True)
        def quantize_fp8(x, scale):
            return (x / scale).clamp(-fp8_max, fp8_max).to(fp8)

        for name, T, d, sc in (("qs1", 8, 4096, 0.05), ("qs2", 3, 28672, 0.0137), ("qs3", 2, 1024, 1.7)):
            xin = rnd(T, 2 * d, scale=3.0)
            act = silu_and_mul(xin.to(dev), enable_pdl=True)
            scale = torch.tensor(sc, dtype=torch.float32, device=dev)
            q = quantize_fp8(act, scale)
            torch.cuda.synchronize()
            arrays.update({f"siluq_{name}_in": bits(xin), f"siluq_{name}_act": bits(act), f"siluq_{name}_out": bits(q),
                           f"siluq_{name}_scale": np.array(sc, dtype=np.float32)})
    except Exception:
        failures.append("silu_and_mul: " + traceback.format_exc(limit=2))

    # ---- apply_rope_with_cos_sin_cache_inplace -----------------------------------------------------
    try:
        from flashinfer.rope import apply_rope_with_cos_sin_cache_inplace
        for name, T, Hq, Hkv, D, rd, P, neox, pdt in (("r128", 16, 4, 2, 128, 128, 64, True, torch.int32),
                                                       ("r128i64", 9, 3, 1, 128, 128, 64, True, torch.int64),
                                                       ("r64", 7, 2, 2, 64, 64, 32, True, torch.int32),
                                                       ("rinter", 8, 2, 1, 128, 128, 64, False, torch.int32)):
            width = (Hq + 2 * Hkv) * D
            qkv = rnd(T, width)
            ang = torch.rand(P, rd // 2, generator=g) * 6.283185307179586
            cache = torch.cat([ang.cos(), ang.sin()], dim=-1).to(torch.float32)
            pos = torch.randint(0, P, (T,), generator=g)
            pos[0] = P - 1
            pos = pos.to(pdt)
            qkv_d = qkv.to(dev)
            q, k = qkv_d[:, : Hq * D], qkv_d[:, Hq * D: (Hq + Hkv) * D]
            apply_rope_with_cos_sin_cache_inplace(pos.to(dev), q, k, D, cache.to(dev), is_neox=neox)
            torch.cuda.synchronize()
            arrays.update({f"rope_{name}_qkv": bits(qkv), f"rope_{name}_cache": cache.numpy(),
                           f"rope_{name}_pos": pos.numpy(), f"rope_{name}_out": bits(qkv_d),
                           f"rope_{name}_dims": np.array([Hq, Hkv, D, int(neox)], dtype=np.int64)})
        # Near-cancellation pairs: partners chosen so that a*cos - b*sin (or b*cos + a*sin) nearly
        # vanishes, which exposes how the kernel's fp32 expression is evaluated (fused multiply-add
        # or two rounded products).
        for name, neox in (("rcancel", True), ("rcancel_inter", False)):
            T, Hq, Hkv, D, P = 24, 4, 2, 128, 64
            half = D // 2
            ang = torch.rand(P, half, generator=g) * 6.283185307179586
            cache = torch.cat([ang.cos(), ang.sin()], dim=-1).to(torch.float32)
            pos = torch.randint(0, P, (T,), generator=g)
            heads = torch.randn(T, Hq + Hkv, D, generator=g, dtype=torch.float64)
            c = cache[pos][:, None, :half].double()
            s = cache[pos][:, None, half:].double()
            a = heads[..., :half] if neox else heads[..., 0::2]
            sel = torch.rand(a.shape, generator=g) < 0.5
            b = torch.where(sel, a * c / s, -a * s / c)  # first or second output nearly cancels
            b = b.clamp(-64, 64)
            if neox:
                heads[..., half:] = b
            else:
                heads[..., 1::2] = b
            qkv = torch.cat([heads.reshape(T, -1), torch.randn(T, Hkv * D, generator=g, dtype=torch.float64)], dim=1)
            qkv = qkv.to(torch.bfloat16)
            pos = pos.to(torch.int32)
            qkv_d = qkv.to(dev)
            q, k = qkv_d[:, : Hq * D], qkv_d[:, Hq * D: (Hq + Hkv) * D]
            apply_rope_with_cos_sin_cache_inplace(pos.to(dev), q, k, D, cache.to(dev), is_neox=neox)
            torch.cuda.synchronize()
            arrays.update({f"rope_{name}_qkv": bits(qkv), f"rope_{name}_cache": cache.numpy(),
                           f"rope_{name}_pos": pos.numpy(), f"rope_{name}_out": bits(qkv_d),
                           f"rope_{name}_dims": np.array([Hq, Hkv, D, int(neox)], dtype=np.int64)})
    except Exception:
        failures.append("apply_rope_with_cos_sin_cache_inplace: " + traceback.format_exc(limit=2))

    # ---- append_paged_kv_cache, alone and after rope (+ llama-4 query scale) ------------------------
    # Metadata as ModelRunner / Devstral2Model.forward build it (devstral2.py:283-290): decode rows
    # first, then prompt rows; kv_indices = block_tables.flatten(), kv_indptr = arange(batch+1) *
    # max_blocks, kv_last_page_len = (seq_lens - 1) % page_size + 1; pages drawn from a shared pool.
    try:
        from flashinfer.page import append_paged_kv_cache
        from flashinfer.rope import apply_rope_with_cos_sin_cache_inplace

        def paged_meta(new, page_size):
            cached = torch.randint(0, 200, (len(new),), generator=g).tolist()
            seq_lens = [c + n for c, n in zip(cached, new)]
            blocks = [-(-L // page_size) for L in seq_lens]
            mb, used = max(blocks), sum(blocks)
            num_pages = used + 4
            perm = torch.randperm(num_pages - 1, generator=g)[:used].to(torch.int32)
            table = torch.full((len(new), mb), num_pages - 1, dtype=torch.int32)
            o = 0
            for b_, nb in enumerate(blocks):
                table[b_, :nb] = perm[o:o + nb]
                o += nb
            pos = torch.cat([torch.arange(c, c + n) for c, n in zip(cached, new)]).to(torch.int32)
            bi = torch.cat([torch.full((n,), b_) for b_, n in enumerate(new)]).to(torch.int32)
            sl = torch.tensor(seq_lens, dtype=torch.int32)
            indptr = torch.arange(len(new) + 1, dtype=torch.int32) * mb
            return pos, bi, table, indptr, (sl - 1) % page_size + 1, num_pages

        for name, new, page_size, layout, H, D in (("anhd", [1, 1, 1, 1, 9, 17], 16, "NHD", 8, 128),
                                                   ("ahnd", [1, 1, 5, 30], 16, "HND", 2, 64),
                                                   ("ap1", [1, 1, 3], 1, "NHD", 2, 64)):
            pos, bi, table, indptr, last, num_pages = paged_meta(new, page_size)
            T = pos.shape[0]
            k = rnd(T, H, D)
            v = rnd(T, H, D)
            shape = (num_pages, H, page_size, D) if layout == "HND" else (num_pages, page_size, H, D)
            kc, vc = rnd(*shape), rnd(*shape)
            kc_d, vc_d = kc.to(dev), vc.to(dev)
            append_paged_kv_cache(k.to(dev), v.to(dev), bi.to(dev), pos.to(dev), (kc_d, vc_d),
                                  table.flatten().to(dev), indptr.to(dev), last.to(dev), kv_layout=layout)
            torch.cuda.synchronize()
            arrays.update({f"append_{name}_k": bits(k), f"append_{name}_v": bits(v), f"append_{name}_pos": pos.numpy(),
                           f"append_{name}_bi": bi.numpy(), f"append_{name}_table": table.numpy(),
                           f"append_{name}_indptr": indptr.numpy(), f"append_{name}_kc": bits(kc),
                           f"append_{name}_vc": bits(vc), f"append_{name}_kcout": bits(kc_d),
                           f"append_{name}_vcout": bits(vc_d), f"append_{name}_hnd": np.array(int(layout == "HND"))})

        # Devstral2Attention.forward's sequence on one qkv row (devstral2.py:158-179)
        Hq, H, D, P, beta, orig = 8, 2, 128, 4096, 0.1, 256
        pos, bi, table, indptr, last, num_pages = paged_meta([1, 1, 1, 40], 16)
        T = pos.shape[0]
        qkv = rnd(T, (Hq + 2 * H) * D)
        ang = torch.rand(P, D // 2, generator=g) * 6.283185307179586
        cache = torch.cat([ang.cos(), ang.sin()], dim=-1).to(torch.float32)
        kc, vc = rnd(num_pages, 16, H, D), rnd(num_pages, 16, H, D)
        qkv_d, kc_d, vc_d, pos_d = qkv.to(dev), kc.to(dev), vc.to(dev), pos.to(dev)
        q, k, v = qkv_d.split([Hq * D, H * D, H * D], dim=-1)
        apply_rope_with_cos_sin_cache_inplace(pos_d, q, k, D, cache.to(dev), is_neox=True)
        append_paged_kv_cache(k.unflatten(-1, (-1, D)), v.unflatten(-1, (-1, D)), bi.to(dev), pos_d, (kc_d, vc_d),
                              table.flatten().to(dev), indptr.to(dev), last.to(dev), kv_layout="NHD")
        scale = 1 + beta * torch.log1p(torch.floor(pos_d.float() / orig))
        q_scaled = q.unflatten(-1, (-1, D)) * scale[:, None, None].to(q.dtype)
        torch.cuda.synchronize()
        arrays.update({"rapp_qkv": bits(qkv), "rapp_cache": cache.numpy(), "rapp_pos": pos.numpy(),
                       "rapp_bi": bi.numpy(), "rapp_table": table.numpy(), "rapp_indptr": indptr.numpy(),
                       "rapp_kc": bits(kc), "rapp_vc": bits(vc), "rapp_qkvout": bits(qkv_d),
                       "rapp_qscaled": bits(q_scaled.flatten(1)), "rapp_kcout": bits(kc_d), "rapp_vcout": bits(vc_d),
                       "rapp_dims": np.array([Hq, H, D], dtype=np.int64),
                       "rapp_beta": np.array(beta, dtype=np.float32), "rapp_orig": np.array(orig)})
    except Exception:
        failures.append("append_paged_kv_cache: " + traceback.format_exc(limit=2))

    import flashinfer
    arrays["flashinfer_version"] = np.array(getattr(flashinfer, "__version__", "unknown"))
    arrays["gpu"] = np.array(torch.cuda.get_device_name())
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "flashinfer_golden.npz", **arrays)
    (out_dir / "flashinfer_golden_failures.txt").write_text("\n".join(failures) or "none\n")
    print("wrote", out_dir / "flashinfer_golden.npz", "failures:", len(failures))
    for f in failures:
        print(f)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
