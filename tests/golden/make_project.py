"""Golden vectors for the commit producer (the captured K / V of one layer,
modules/attention.rs:107-124, 143-144, and quantize_kv_pair of them), generated
by the oracle.

Two cases at head_dim 128 with x and the weights on power-of-two grids (every
partial sum of the product exact in any order, so the vectors are also what
the device kernel must produce): 160 tokens x 2 heads with bias, RMS norm with
gain and RoPE; 96 tokens x 4 heads, plain Lin.  Inputs come from numpy's
seeded generator (PCG64) as written below (rotary tables from IEEE
arithmetic only, no libm), so only outputs are stored: the
SHA-256 of the bf16 K and V bits, of the INT8 codes and of the scales, plus a
few values in the clear.

    python tests/golden/make_project.py      # rewrites project_int8.json

Test infrastructure: only tests import this module.
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

D = 128
CASES = {"m160_h2_full": dict(M=160, H=2, seed=20, bias=True, norm=True, rope=True),
         "m96_h4_plain": dict(M=96, H=4, seed=21, bias=False, norm=False, rope=False)}


def inputs(orc, M, H, seed):
    rng = np.random.default_rng(seed)
    dim = H * D
    b = lambda a: orc.bf16_bits(np.asarray(a, np.float32))  # noqa: E731
    x = b(rng.integers(-4, 5, (M, dim)) * 0.25)
    wk = b(rng.integers(-4, 5, (dim, dim)) * 0.0625)
    wv = b(rng.integers(-4, 5, (dim, dim)) * 0.0625)
    bk, bv = b(rng.standard_normal(dim) * 0.1), b(rng.standard_normal(dim) * 0.1)
    gain = b(1.0 + 0.1 * rng.standard_normal(D))
    # unit-circle points from IEEE arithmetic only (no libm), so the tables
    # are the same on every machine: (1 - t^2, 2t) / (1 + t^2)
    t = rng.uniform(-1.0, 1.0, (M, D // 2))
    den = 1.0 + t * t
    return dict(x=x, wk=wk, wv=wv, bk=bk, bv=bv, gain=gain, cos=((1.0 - t * t) / den).astype(np.float32),
                sin=((2.0 * t) / den).astype(np.float32))


def outputs(orc, case):
    c = CASES[case]
    a = inputs(orc, c["M"], c["H"], c["seed"])
    k, v = orc.kv_project(a["x"], a["wk"], a["wv"], bk=a["bk"] if c["bias"] else None,
                          bv=a["bv"] if c["bias"] else None, k_gain=a["gain"], qk_norm=c["norm"], eps=1e-6,
                          cos=a["cos"] if c["rope"] else None, sin=a["sin"] if c["rope"] else None)
    M, H = c["M"], c["H"]
    kq, vq, ks, vs = orc.quantize_kv_pair(k.reshape(1, M, H, D), v.reshape(1, M, H, D), orc.BF16)
    return a, dict(k=k, v=v, kq=kq, vq=vq, ks=ks, vs=vs)


def digest(arr) -> str:
    return hashlib.sha256(np.ascontiguousarray(arr).tobytes()).hexdigest()


def main():
    import oracle as orc
    orc.build()
    out = {"note": "sha256 of the oracle's outputs for seeded exact-grid inputs; see make_project.py", "cases": {}}
    for case in CASES:
        _, o = outputs(orc, case)
        out["cases"][case] = {**CASES[case], **{n: digest(t) for n, t in o.items()},
                              "k_first": [int(t) for t in o["k"][0, :4]], "ks_first": [float(t) for t in
                                                                                      o["ks"].reshape(-1)[:4]]}
    with open(os.path.join(HERE, "project_int8.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
