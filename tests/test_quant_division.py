"""The fp8 SiLU-mul kernel divides by the activation scale without a divide instruction: it takes
q0 = x * RN(1/s) and applies one Markstein remainder step, q1 = fma(RN(1/s), fma(-s, q0, x), q0),
where |q0| is in [2^-12, 512) (outside that range e4m3 gives a signed zero or saturates).

This test re-checks, on the CPU and exhaustively over every bf16 and every fp16 input, that the
method gives the IEEE quotient wherever it is applied and the right sign everywhere, for random and
power-of-two scales. The C below restates the kernel's expression (silu.cuh, QuantDiv); gcc compiles
it with contraction off so each operation rounds as on the GPU.
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

C_SRC = r"""
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
static float from16(uint16_t h, int fp16) {
  if (fp16) { _Float16 v; memcpy(&v, &h, 2); return (float)v; }
  uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f;
}
static uint32_t bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
int main(int argc, char** argv) {
  const int nscales = atoi(argv[1]);
  srand(11);
  long bad = 0, n = 0;
  for (int k = 0; k < nscales; ++k) {
    float s;
    if (k < 120) s = ldexpf(k % 2 ? 1.0f : 1.5f, (k % 60) - 30);
    else s = (float)pow(10.0, -4.0 + 5.0 * ((double)rand() / RAND_MAX)) * ((rand() & 1) ? 1.0f : -1.0f);
    const float r = 1.0f / s;
    if (!isnormal(r)) continue;
    for (int fp16 = 0; fp16 < 2; ++fp16) {
      for (uint32_t h = 0; h < 65536; ++h) {
        const float x = from16((uint16_t)h, fp16);
        if (isnan(x)) continue;
        const float qi = x / s;
        const float q0 = x * r;
        const float q1 = fmaf(r, fmaf(-s, q0, x), q0);
        const float a = fabsf(q0);
        const float q = (a >= 0x1p-12f && a < 512.0f) ? q1 : q0;
        ++n;
        if (signbit(q) != signbit(qi) || (a >= 0x1p-12f && a < 512.0f && bits(q) != bits(qi))) ++bad;
      }
    }
  }
  printf("%ld %ld\n", n, bad);
  return 0;
}
"""


def test_markstein_quotient_equals_ieee_division(tmp_path: Path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src, exe = tmp_path / "qdiv.c", tmp_path / "qdiv"
    src.write_text(C_SRC)
    subprocess.run([cc, "-O2", "-ffp-contract=off", "-o", str(exe), str(src), "-lm"], check=True)
    out = subprocess.run([str(exe), "1500"], check=True, capture_output=True, text=True).stdout.split()
    n, bad = int(out[0]), int(out[1])
    assert n > 150_000_000
    assert bad == 0
