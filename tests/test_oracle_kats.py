"""Pin the CPU oracle (and the product's host-side policy) to the reference's
own tests.  Each test names the reference test it replays.

Exact known answers exist for the frame samplers and SWA trim plans
(cache/uniform_history.rs:131-196, cache/swa.rs:146-230); INT8 and QVG are
pinned by the reference's invariants (cache/int8.rs:162-244,
cache/qvg.rs:450-527).
"""
import numpy as np
import pytest


# ---------------------------------------------------- uniform_history.rs
@pytest.fixture(params=["oracle", "product"])
def sampler(request, orc):
    """Both the oracle and the product's host policy (C ABI, no GPU needed)."""
    if request.param == "oracle":
        return lambda kind, t, p, s=1, g=2.0: orc.frame_indices(kind, t, p, s, g)
    import nomas_kv as nk

    def f(kind, t, p, s=1, g=2.0):
        k = {"uniform": 0, "recent_mix": 1, "temporal": 2, "history": 3}[kind]
        return nk._indices(k, t, p, s, g)

    return f


def test_uniform_endpoints_inclusive(sampler):  # uniform_history.rs:131-137
    assert sampler("uniform", 10, 4) == [0, 3, 6, 9]
    assert sampler("uniform", 0, 4) == []
    assert sampler("uniform", 1, 4) == [0]
    assert sampler("uniform", 5, 10) == [0, 1, 2, 3, 4]


def test_recent_mix_keeps_contiguous_tail(sampler):  # uniform_history.rs:139-148
    ids = sampler("recent_mix", 20, 6)
    assert len(ids) == 6
    assert ids[3:] == [17, 18, 19]
    assert ids[:3] == [0, 8, 16]
    assert all(a < b for a, b in zip(ids, ids[1:]))


def test_short_history_kept_completely(sampler):  # uniform_history.rs:150-153
    assert sampler("recent_mix", 4, 10) == [0, 1, 2, 3]


def test_temporal_context_gamma_one_is_uniform(sampler):  # uniform_history.rs:155-161
    a = sampler("temporal", 17, 5, 3, 1.0)
    assert a == sampler("uniform", 17, 5)
    assert a == [0, 4, 8, 12, 16]


def test_temporal_context_biases_recent_for_large_gamma(sampler):  # uniform_history.rs:163-171
    ids = sampler("temporal", 100, 5, 3, 4.0)
    assert len(ids) == 5 and ids[-1] == 99 and ids[0] < 40
    assert all(a < b for a, b in zip(ids, ids[1:]))


def test_validator_rejects_bad_gamma(orc):  # uniform_history.rs:173-177
    with pytest.raises(orc.OracleError) as e:
        orc.frame_indices("history", 10, 4, orc.TEMPORAL, 0.0)
    assert e.value.code == orc.ERR_INVALID_CONFIG
    import nomas_kv as nk
    with pytest.raises(nk.InvalidConfigError):
        nk.history_frame_indices(10, 4, nk.HistorySampling.temporal_context(0.0))


def test_all_samplers_pass_validation_on_random_budgets(sampler):  # uniform_history.rs:179-196
    for total in range(40):
        for past in range(1, 12):
            for s, g in ((1, 2.0), (2, 2.0), (3, 2.0)):
                ids = sampler("history", total, past, s, g)
                assert len(ids) == min(total, past)
                assert all(a < b for a, b in zip(ids, ids[1:]))


def test_product_samplers_equal_oracle_exhaustive(orc):
    """The product's host planner and the oracle agree on every sampler over
    the long-session grid (config 4: up to 1024 frames, 32 past frames)."""
    import nomas_kv as nk
    for total in list(range(0, 130)) + [255, 256, 511, 512, 1023, 1024, 4096]:
        for past in (1, 2, 3, 5, 6, 16, 31, 32, 64):
            for kind, s, g in (("uniform", 1, 2.0), ("recent_mix", 2, 2.0), ("temporal", 3, 0.9),
                               ("temporal", 3, 2.0), ("temporal", 3, 1.0), ("temporal", 3, 0.37)):
                a = orc.frame_indices(kind, total, past, s, g)
                k = {"uniform": 0, "recent_mix": 1, "temporal": 2}[kind]
                assert nk._indices(k, total, past, s, g) == a, (kind, total, past, g)
                assert nk._indices(3, total, past, s, g) == a


def test_uniform_8b_geometry_kat(sampler):
    # 32 segments x 4 frames, 16 sampled frames (the 8B rebuild)
    assert sampler("uniform", 128, 16) == [0, 8, 16, 25, 33, 42, 50, 59, 67, 76, 84, 93, 101, 110, 118, 127]
    # tiny config: 4 segments x 3 frames, 6 sampled frames
    assert sampler("uniform", 12, 6) == [0, 2, 4, 6, 8, 11]


# ---------------------------------------------------------------- swa.rs
def _rec(seg, frames, tpf, text):
    return (seg, seg * frames, frames, frames * tpf, text)


@pytest.fixture(params=["oracle", "product"])
def trim(request, orc):
    if request.param == "oracle":
        def f(recs, cap, tpf):
            r = orc.plan_recent_trim(recs, cap, tpf)
            return r.drop_frames, r.drop_records, r.evicted_tokens, r.kept
        return f
    import nomas_kv as nk
    return nk.plan_recent_trim


def test_no_trim_when_under_capacity(trim):  # swa.rs:154-161
    df, dr, ev, kept = trim([_rec(0, 2, 4, 3), _rec(1, 2, 4, 3)], 100, 4)
    assert df == [] and dr == [] and ev == 0 and len(kept) == 2


def test_frame_aligned_partial_trim(trim):  # swa.rs:163-180
    df, dr, ev, kept = trim([_rec(0, 2, 8, 2), _rec(1, 2, 8, 2)], 30, 8)
    assert df == [(0, 1)] and dr == []
    assert kept[0][2] == 1 and kept[0][3] == 8 and kept[0][4] == 2
    assert kept[1][2] == 2
    assert sum(k[3] + k[4] for k in kept) <= 30


def test_whole_segment_eviction_drops_text(trim):  # swa.rs:182-192
    df, dr, ev, kept = trim([_rec(0, 2, 4, 3), _rec(1, 2, 4, 3)], 11, 4)
    assert dr == [0] and len(kept) == 1 and kept[0][0] == 1 and ev == 11


def test_video_gone_but_text_within_budget_is_kept(trim):  # swa.rs:194-216
    df, dr, ev, kept = trim([_rec(0, 2, 4, 3), _rec(1, 2, 4, 3)], 14, 4)
    assert df == [(0, 2)] and dr == []
    assert len(kept) == 2 and kept[0][2] == 0 and kept[0][4] == 3 and kept[1][2] == 2
    assert sum(k[3] + k[4] for k in kept) == 14


def test_text_dropped_when_video_and_text_both_needed(trim):  # swa.rs:218-228
    df, dr, ev, kept = trim([_rec(0, 2, 4, 3), _rec(1, 2, 4, 3)], 13, 4)
    assert dr == [0] and len(kept) == 1 and kept[0][0] == 1


def test_capacity_smaller_than_one_segment(trim):  # swa.rs:230-238
    df, dr, ev, kept = trim([_rec(0, 4, 4, 3)], 8, 4)
    assert sum(k[3] + k[4] for k in kept) <= 8
    assert all(k[2] >= 1 for k in kept)


def test_trim_product_equals_oracle_sweep(orc):
    import nomas_kv as nk
    rng = np.random.default_rng(0)
    for _ in range(400):
        n = int(rng.integers(0, 6))
        tpf = int(rng.integers(1, 9))
        recs, start = [], 0
        for i in range(n):
            fr = int(rng.integers(1, 5))
            recs.append((i, start, fr, fr * tpf, int(rng.integers(0, 5))))
            start += fr
        cap = int(rng.integers(1, 80))
        r = orc.plan_recent_trim(recs, cap, tpf)
        assert nk.plan_recent_trim(recs, cap, tpf) == (r.drop_frames, r.drop_records, r.evicted_tokens, r.kept)


# --------------------------------------------------------------- int8.rs
def test_int8_roundtrip_error_bound(orc):  # int8.rs:170-192
    k = orc.randn((1, 16, 3, 32), 11)
    kq, vq, ks, vs = orc.quantize_kv_pair(k, k, orc.F32)
    assert kq.dtype == np.uint8
    back = orc.dequantize(kq, ks, 16, orc.F32)
    peak = np.abs(k).max(axis=-1, keepdims=True)
    bound = peak / 127.0 / 2.0 + 1e-6
    assert np.all(np.abs(k - back) <= bound)


def test_int8_zero_rows_get_unit_scale(orc):  # int8.rs:194-213
    k = np.zeros((1, 4, 2, 8), np.float32)
    kq, vq, ks, vs = orc.quantize_kv_pair(k, k, orc.F32)
    assert np.all(ks == 1.0)
    back = orc.dequantize(kq, ks, 4, orc.F32)
    assert np.all(np.abs(back) < 1e-6)


def test_int8_clamps_to_int8_range(orc):  # int8.rs:215-234
    k = np.array([-1000, 0, 1000, 0.5, -0.5, 1.0, -1.0, 0.0], np.float32).reshape(1, 1, 1, 8)
    kq, *_ = orc.quantize_kv_pair(k, k, orc.F32)
    assert np.all((kq >= 1) & (kq <= 255))


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf, np.finfo(np.float32).max])
def test_int8_rejects_non_finite(orc, bad):  # int8.rs:236-244 (NaN, Inf; |x| >= f32::MAX)
    d = np.zeros(8, np.float32)
    d[3] = bad
    k = d.reshape(1, 1, 1, 8)
    with pytest.raises(orc.OracleError) as e:
        orc.quantize_kv_pair(k, k, orc.F32)
    assert e.value.code == orc.ERR_MSG and "non-finite k" in e.value.msg
    ok = np.zeros_like(k)
    with pytest.raises(orc.OracleError) as e:
        orc.quantize_kv_pair(ok, k, orc.F32)
    assert "non-finite v" in e.value.msg


def _int8_numpy(x: np.ndarray):
    """Independent numpy restatement of quantize_one (int8.rs:65-81) used to
    cross-check the C++ oracle's arithmetic on f32 input."""
    x = x.astype(np.float32)
    peak = np.abs(x).max(axis=-1, keepdims=True)
    inv = np.float32(1.0 / 127.0)
    s = np.where(peak > 0, (peak * inv) + np.float32(0.0), np.float32(1.0)).astype(np.float32)
    q = (x / s).astype(np.float32)
    t = np.trunc(q)
    q = np.where(np.abs(q - t) >= np.float32(0.5), t + np.sign(q), t)  # half away from zero
    q = np.clip(q, -127, 127) + 128
    return q.astype(np.uint8), s[..., 0]


def test_int8_oracle_equals_numpy_restatement(orc):
    rng = np.random.default_rng(1)
    for shape in ((1, 37, 3, 32), (2, 5, 4, 128), (1, 9, 2, 7)):
        x = (rng.standard_normal(shape) * rng.choice([1e-3, 1.0, 300.0])).astype(np.float32)
        x[0, 0, 0, :] = 0.0
        kq, _, ks, _ = orc.quantize_kv_pair(x, x, orc.F32)
        q2, s2 = _int8_numpy(x)
        assert np.array_equal(kq, q2)
        assert np.array_equal(ks.view(np.uint32), s2.view(np.uint32))


def test_int8_half_integer_ties_round_away(orc):
    # peak 127 -> scale 127 * f32(1/127); x = k + 0.5 lands on exact ties
    row = np.array([127.0] + [k + 0.5 for k in range(-63, 63, 2)], np.float32)
    x = row.reshape(1, 1, 1, -1)
    kq, _, ks, _ = orc.quantize_kv_pair(x, x, orc.F32)
    q2, s2 = _int8_numpy(x)
    assert np.array_equal(kq, q2)


# ---------------------------------------------------------------- qvg.rs
def test_qvg_bit_packing_roundtrip(orc):  # qvg.rs:450-463
    buf = np.zeros(1, np.uint8)
    for s in range(4):
        orc.pack_bits(buf, s * 2, 2, (s + 1) % 4)
    for s in range(4):
        assert orc.unpack_bits(buf, s * 2, 2) == (s + 1) % 4


def test_qvg_quality_improves_with_stages(orc):  # qvg.rs:465-496
    k = orc.randn((1, 128, 2, 16), 42)
    errors = []
    for stages in (1, 2, 4):
        cb = orc.qvg_fit(k, k, stages=stages)
        codes, scales = orc.qvg_encode(cb, 0, k, 128)
        back = orc.qvg_decode(cb, 0, codes, scales, 128)
        errors.append(float(((k.astype(np.float64) - back.astype(np.float64)) ** 2).sum()))
    assert errors[2] < errors[1] < errors[0]


def test_qvg_storage_is_int8_comparable(orc):  # qvg.rs:498-511
    assert orc.qvg_payload_bytes(1024, 24) / 1024 / 24 < 1.3
    import nomas_kv as nk
    assert nk.QvgConfig().bytes_per_token() == 1
    assert nk.QvgConfig().payload_bytes(1024, 24) == orc.qvg_payload_bytes(1024, 24)


def test_qvg_frozen_codebooks(orc):  # qvg.rs:513-527
    k = orc.randn((1, 64, 2, 8), 5)
    cfg = orc.Config(storage=orc.QVG, sampling=orc.UNIFORM, past_frames=4)
    bank = orc.Bank(cfg, 1, 1, 2, 8, orc.F32)
    seg = dict(segment_index=0, frame_start=0, frame_count=1, image_tokens=64, text_tokens=0)
    bank.commit(seg, orc.F32, [k], [k])
    cb1 = bank.codebooks(0).copy()
    k2 = orc.randn((1, 64, 2, 8), 9)
    bank.commit(dict(seg, segment_index=1, frame_start=1), orc.F32, [k2], [k2])
    assert np.array_equal(bank.codebooks(0), cb1)


def test_qvg_nearest_ties_go_to_lower_index(orc):
    """Duplicate codewords: every residual ties and must pick the first."""
    H, D = 1, 8
    cb = np.zeros((2, H, 1, 4, D), np.float32)
    cb[:, :, 0, 0] = cb[:, :, 0, 2] = 1.0
    cb[:, :, 0, 1] = cb[:, :, 0, 3] = -1.0
    x = np.ones((1, 5, H, D), np.float32)
    codes, scales = orc.qvg_encode(cb, 0, x, 5)
    assert all(c & 3 == 0 for c in codes)
    codes, _ = orc.qvg_encode(cb, 0, -x, 5)
    assert all(c & 3 == 1 for c in codes)
