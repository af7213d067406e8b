"""Pin the oracle's restatement of the captured K / V chain (the producer
side of a commit: modules/attention.rs:107-124, 143-144; modules/mod.rs:122-142;
modules/norm.rs:55-65; rope.rs:257-306).

* an independent numpy restatement (per-operation f32 rounding, explicit
  bf16 rounding) agrees with it bit for bit;
* the reference's own RoPE and RmsNorm tests, replayed on it:
  rope.rs apply_rotary_identity_at_zero_position and
  apply_rotary_is_orthogonal_rotation, norm.rs rms_norm_unit_variance and
  zero_vector_stays_finite.
"""
import numpy as np
import pytest

D = 128


def _bf(orc, x):
    return orc.bf16_to_f32(orc.bf16_bits(np.asarray(x, np.float32)))


def numpy_chain(orc, x, wk, wv, bk, bv, gain, qk_norm, eps, cos, sin):
    """The same chain in numpy float32 (one rounding per operation)."""
    xf = orc.bf16_to_f32(x).astype(np.float64)
    outs = []
    for side, (w, b) in enumerate(((wk, bk), (wv, bv))):
        acc = (xf @ orc.bf16_to_f32(w).astype(np.float64).T).astype(np.float32)
        y = _bf(orc, acc)
        if b is not None:
            y = _bf(orc, y + orc.bf16_to_f32(b)[None, :])
        M, dim = y.shape
        y = y.reshape(M, dim // D, D)
        if side == 0 and qk_norm:
            s = np.zeros((M, dim // D, 4), np.float32)
            for d in range(D):
                s[..., d & 3] = s[..., d & 3] + y[..., d] * y[..., d]
            ss = (s[..., 0] + s[..., 1]) + (s[..., 2] + s[..., 3])
            var = ss * np.float32(1.0 / D)
            inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))
            o = y * inv[..., None]
            if gain is not None:
                o = o * orc.bf16_to_f32(gain)[None, None, :]
            y = _bf(orc, o)
        if side == 0 and cos is not None:
            xr, xi = y[..., 0::2], y[..., 1::2]
            c, sn = cos[:, None, :], sin[:, None, :]
            o_r = _bf(orc, xr * c - xi * sn)
            o_i = _bf(orc, xi * c + xr * sn)
            y = np.stack([o_r, o_i], axis=-1).reshape(M, dim // D, D)
        outs.append(orc.bf16_bits(y.reshape(M, dim)))
    return outs


def _inputs(orc, M, H, seed, integer=False):
    rng = np.random.default_rng(seed)
    dim = H * D
    if integer:
        x = rng.integers(-4, 5, (M, dim)) * 0.25
        wk = rng.integers(-4, 5, (dim, dim)) * 0.0625
        wv = rng.integers(-4, 5, (dim, dim)) * 0.0625
    else:
        x = rng.standard_normal((M, dim))
        wk = rng.standard_normal((dim, dim)) / np.sqrt(dim)
        wv = rng.standard_normal((dim, dim)) / np.sqrt(dim)
    bk = rng.standard_normal(dim) * 0.1
    bv = rng.standard_normal(dim) * 0.1
    gain = 1.0 + 0.1 * rng.standard_normal(D)
    ang = rng.uniform(0, 6.3, (M, D // 2)).astype(np.float32)
    b = lambda a: orc.bf16_bits(np.asarray(a, np.float32))  # noqa: E731
    return dict(x=b(x), wk=b(wk), wv=b(wv), bk=b(bk), bv=b(bv), gain=b(gain), cos=np.cos(ang), sin=np.sin(ang))


@pytest.mark.parametrize("integer", [True, False])
@pytest.mark.parametrize("opts", [(True, True, True), (False, False, False), (True, False, True)])
def test_oracle_matches_numpy_restatement(orc, integer, opts):
    bias, norm, rope = opts
    a = _inputs(orc, 37, 2, seed=11, integer=integer)
    args = dict(bk=a["bk"] if bias else None, bv=a["bv"] if bias else None, k_gain=a["gain"], qk_norm=norm,
                eps=1e-6, cos=a["cos"] if rope else None, sin=a["sin"] if rope else None)
    k, v = orc.kv_project(a["x"], a["wk"], a["wv"], **args)
    nk_, nv_ = numpy_chain(orc, a["x"], a["wk"], a["wv"], args["bk"], args["bv"], a["gain"], norm, 1e-6,
                           args["cos"], args["sin"])
    if integer:  # every partial sum exact: the f64 product is the f32 one
        assert np.array_equal(k, nk_) and np.array_equal(v, nv_)
    else:  # numpy's f64 GEMM sums in its own order: equal up to rare last-bit flips
        assert np.mean(k == nk_) > 0.999 and np.mean(v == nv_) > 0.999


def test_rope_identity_at_zero_angle(orc):  # rope.rs apply_rotary_identity_at_zero_position
    a = _inputs(orc, 8, 2, seed=3)
    ones, zeros = np.ones((8, D // 2), np.float32), np.zeros((8, D // 2), np.float32)
    k_rot, _ = orc.kv_project(a["x"], a["wk"], a["wv"], cos=ones, sin=zeros)
    k_plain, _ = orc.kv_project(a["x"], a["wk"], a["wv"])
    assert np.array_equal(k_rot, k_plain)


def test_rope_preserves_norms(orc):  # rope.rs apply_rotary_is_orthogonal_rotation
    a = _inputs(orc, 16, 2, seed=5)
    k_rot, _ = orc.kv_project(a["x"], a["wk"], a["wv"], cos=a["cos"], sin=a["sin"])
    k_plain, _ = orc.kv_project(a["x"], a["wk"], a["wv"])
    n = lambda b: np.linalg.norm(orc.bf16_to_f32(b).reshape(16, 2, D).astype(np.float64), axis=-1)  # noqa: E731
    assert np.allclose(n(k_rot), n(k_plain), rtol=1e-2)


def test_rms_norm_unit_variance(orc):  # norm.rs rms_norm_unit_variance
    a = _inputs(orc, 10, 2, seed=7)
    k, _ = orc.kv_project(a["x"], a["wk"], a["wv"], qk_norm=True, eps=1e-6)
    kf = orc.bf16_to_f32(k).reshape(10, 2, D).astype(np.float64)
    assert np.allclose((kf ** 2).mean(-1), 1.0, atol=1e-2)  # bf16 outputs: 1e-3 of the reference is f32


def test_rms_norm_zero_vector_stays_finite(orc):  # norm.rs zero_vector_stays_finite
    dim = 2 * D
    x = np.zeros((3, dim), np.uint16)
    w = orc.bf16_bits(np.ones((dim, dim), np.float32))
    k, _ = orc.kv_project(x, w, w, qk_norm=True, eps=1e-6)
    assert np.all(np.isfinite(orc.bf16_to_f32(k)))
