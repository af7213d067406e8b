"""Exhaustive device checks of the INT8 quantizer's two arithmetic shortcuts.

quantize_one (cache/int8.rs:65-81) divides each value by its row scale and
rounds half away from zero.  The commit kernels and the K/V producer's
epilogue instead take the quotient from a reciprocal with one FMA
correction (Markstein) and round with a round-toward-zero add of 1.5 * 2^23
(nkv_quant.cuh).  tests/cuda/quant_identity_check.cu checks, with the
product's own device functions, that

* the resulting code byte, scalar and packed, equals the IEEE-division
  path's (quant_exact) for every bf16 value x and every finite bf16 row peak
  p >= |x| whose scale takes the fast path (31,618 peaks, 1,064,356,734
  signed pairs);
* the rounding equals roundf for every f32 in [0, 128];
* the corrected quotient is within one ulp of the IEEE quotient for every one
  of those pairs.  It is not always equal to it: the program also reports
  where they differ, by the magnitude of the quotient.

The kernels' inputs are always bf16 (history.rs:249-250 casts K/V to bf16
before quantizing), so these domains are complete.
"""
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _expected_counts():
    pb = np.arange(1, 0x7F80, dtype=np.uint32)
    p = (pb << np.uint32(16)).view(np.float32)
    s = p * np.float32(1.0 / 127.0) + np.float32(0.0)
    fast = (s >= np.finfo(np.float32).tiny) & (s <= np.float32(1e37))
    pairs = int((2 * (pb[fast].astype(np.uint64) + 1)).sum())
    return int(fast.sum()), pairs


def test_quantizer_shortcuts_exhaustively(tmp_path):
    exe = str(tmp_path / "quant_identity_check")
    subprocess.run(["nvcc", "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-fmad=false",
                    "-I", os.path.join(ROOT, "hy-nomas-rs_b200", "csrc"),
                    os.path.join(ROOT, "tests", "cuda", "quant_identity_check.cu"), "-o", exe],
                   check=True, capture_output=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=300).stdout.split()
    got = {out[i]: int(out[i + 1]) for i in range(0, len(out), 2)}
    peaks, pairs = _expected_counts()
    assert (peaks, pairs) == (31618, 1064356734)
    assert got["fast_peaks"] == peaks and got["pairs"] == pairs, got
    assert got["quotient_off_by_more_than_1ulp"] == 0, got
    assert got["code_mismatches"] == 0, got
    assert got["packed_code_mismatches"] == 0, got
    assert got["rounding_values"] == 0x43000000 + 1, got  # every f32 bit pattern in [0, 128]
    assert got["rounding_mismatches"] == 0, got
