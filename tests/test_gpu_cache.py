"""GPU parity of the whole cache API against the CPU oracle (bit-exact).

Sessions replay the reference's cache-observable scenarios
(nomas-core/tests/session.rs, tests/interactive.rs) plus the tiny
benchmark config (2 layers, 4 heads, head_dim 32, F32 K/V, 4 segments of
3 x 64 + 16 tokens) under every storage x sampling combination; after
every operation the harness compares status, layouts, metrics, working sets
(bitwise) and archived payload bytes.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

STORAGES = {"float": 0, "int8": 1, "qvg": 2}
SAMPLINGS = {"recent": (0, 2.0), "uniform": (1, 2.0), "recent_mix": (2, 2.0), "temporal": (3, 2.0),
             "temporal09": (3, 0.9)}


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    return cache_harness


def _pair(H, storage="int8", sampling="uniform", past=6, capacity=None, phase_swap=False, **geo):
    s, g = SAMPLINGS[sampling]
    spec = H.Spec(storage=STORAGES[storage], sampling=s, gamma=g, past_frames=past, capacity=capacity,
                  phase_swap=phase_swap)
    return H.Pair(H.Geometry(**geo), spec)


def test_inputs_bit_identical_on_both_sides(H):
    p = _pair(H, input_dtype="bf16")
    kd, vd, kh, vh = p.inputs(3, 208)
    for t, h in zip(kd + vd, kh + vh):
        assert np.array_equal(H.torch_to_raw(t), h)
    p.close()


@pytest.mark.parametrize("model_dtype", ["f32", "bf16"])
def test_config1_tiny_int8_uniform6(H, model_dtype):
    """The tiny configuration (config 1): INT8, uniform history of 6 past frames."""
    p = _pair(H, "int8", "uniform", past=6, model_dtype=model_dtype)
    for _ in range(4):
        assert p.commit() is None
        p.check()
    p.close()


@pytest.mark.parametrize("capacity", [192, 208])
def test_config1_tiny_recent_swa(H, capacity):
    """The tiny configuration's SWA window of 3 frames as Recent capacity."""
    p = _pair(H, "int8", "recent", capacity=capacity)
    for _ in range(4):
        assert p.commit() is None
        p.check()
    assert p.p.metrics().evicted_tokens > 0
    p.close()


@pytest.mark.parametrize("storage", list(STORAGES))
@pytest.mark.parametrize("sampling", list(SAMPLINGS))
def test_every_storage_and_sampling(H, storage, sampling):
    p = _pair(H, storage, sampling, past=4, capacity=300 if sampling == "recent" else None, frames=2,
              model_dtype="bf16", input_dtype="f32")
    for i in range(5):
        assert p.commit(text=16 if i % 2 else 9, action_start=-1 if i % 2 else 3) is None
        p.check()
    if sampling != "recent":
        assert p.rollback() is None
        p.check()
        assert p.commit() is None
        p.check()
    p.close()


@pytest.mark.parametrize("dtypes", [("f32", "f32"), ("bf16", "bf16"), ("f16", "f16"), ("bf16", "f32"),
                                    ("f32", "f16"), ("f16", "bf16")])
@pytest.mark.parametrize("storage", ["float", "int8"])
def test_dtype_combinations(H, dtypes, storage):
    model, inp = dtypes
    p = _pair(H, storage, "uniform", past=5, model_dtype=model, input_dtype=inp)
    for _ in range(3):
        assert p.commit() is None
        p.check()
    p.close()


@pytest.mark.parametrize("head_dim,heads", [(8, 2), (24, 3), (16, 4), (64, 2), (128, 2), (256, 1)])
def test_head_dims_vector_and_generic_paths(H, head_dim, heads):
    for storage in ("int8", "float"):
        p = _pair(H, storage, "uniform", past=4, heads=heads, head_dim=head_dim, tpf=32, frames=2, text=5,
                  model_dtype="bf16", input_dtype="bf16")
        for _ in range(3):
            assert p.commit() is None
        p.check()
        p.close()


def test_batch_two(H):
    for storage in ("int8", "float"):
        p = _pair(H, storage, "recent_mix", past=4, batch=2, frames=2, model_dtype="bf16")
        for _ in range(4):
            assert p.commit() is None
            p.check()
        assert p.rollback() is None
        p.check()
        p.close()


# ------------------------------------------------------------------ QVG
def test_qvg_fit_on_first_commit_matches_oracle(H):
    p = _pair(H, "qvg", "uniform", past=6, model_dtype="bf16", input_dtype="bf16", tpf=40, text=16)
    assert p.commit() is None
    for layer in range(p.geo.n_layers):
        cbo = p.o.codebooks(layer)
        cbp = p.p.layer(layer).qvg_codebooks()
        assert cbo is not None and cbp is not None
        assert np.array_equal(cbo.view(np.uint32), cbp.view(np.uint32)), "host fit differs from oracle fit"
    p.check()
    for _ in range(3):
        assert p.commit() is None
        p.check()
    p.close()


@pytest.mark.parametrize("input_dtype", ["bf16", "f32"])
def test_qvg_head_dim_128_fast_encoder_in_the_bank(H, input_dtype):
    """head_dim 128 with the default codec takes the screened d128 encoder."""
    p = _pair(H, "qvg", "uniform", past=4, model_dtype="bf16", input_dtype=input_dtype, heads=2, head_dim=128,
              tpf=40, frames=2, text=5)
    for _ in range(3):
        assert p.commit() is None
        p.check()
    p.close()


def test_qvg_d128_block_sums_near_zero(H):
    """Blocks whose numerator is exactly 0 or tiny and of either sign: the d128
    encoder's fast block sum cannot certify alpha there and takes the
    sequential sums (qvg.rs:220-230), which must still equal the oracle."""
    p = _pair(H, "qvg", "uniform", past=4, model_dtype="bf16", input_dtype="bf16", heads=2, head_dim=128,
              tpf=64, frames=3, text=4)

    import oracle as orc

    def flatten(layer, side, h):  # h: bf16 bit patterns (uint16)
        if layer == 0:
            h[0, 0:64] = 0                                  # a whole block of zero residuals: num = 0
            h[0, 64:96] = 0                                 # half a block zero ...
            tiny = orc.bf16_to_f32(h[0, 96:128]) * np.float32(1e-20)
            h[0, 96:128] = orc.bf16_bits(tiny)              # ... the rest tiny
            h[0, 128:192, :, 1::2] ^= np.uint16(0x8000)     # sign-mixed products

    for _ in range(2):
        assert p.commit(poison=flatten) is None
        p.check()
    p.close()


def test_qvg_frozen_codebooks_and_partial_blocks(H):
    """Frozen synthetic codebooks (as in the QVG benchmark), a last block of
    fewer than 64 tokens, and the sigma_s = 1, .5, .25, .125 stage scales."""
    p = _pair(H, "qvg", "uniform", past=6, model_dtype="bf16", input_dtype="bf16", tpf=50, text=7)
    rng = np.random.default_rng(7)
    cbs = []
    for layer in range(p.geo.n_layers):
        cb = np.zeros((2, p.geo.heads, 4, 4, p.geo.head_dim), np.float32)
        for s, sig in enumerate((1.0, 0.5, 0.25, 0.125)):
            cb[:, :, s] = rng.standard_normal(cb[:, :, s].shape).astype(np.float32) * np.float32(sig)
        cbs.append(cb)
    p.set_codebooks(cbs)
    for _ in range(4):
        assert p.commit() is None
        p.check()
    p.close()


def test_qvg_duplicate_codewords_tie_to_lower_index(H):
    p = _pair(H, "qvg", "uniform", past=6, model_dtype="f32", input_dtype="f32", frames=1, tpf=64, text=0)
    cb = np.zeros((2, p.geo.heads, 4, 4, p.geo.head_dim), np.float32)
    cb[:, :, :, 1] = cb[:, :, :, 3] = 0.5  # entries 1 and 3 identical, 0 and 2 identical (zeros)
    p.set_codebooks([cb] * p.geo.n_layers)
    assert p.commit() is None
    p.check()
    p.close()


def test_qvg_text_nonfinite_rejected_video_nan_accepted(H):
    p = _pair(H, "qvg", "uniform", past=6, model_dtype="bf16", input_dtype="f32", tpf=32, text=8, frames=2)
    assert p.commit() is None  # fits codebooks

    def nan_text(layer, side, h):
        if layer == 0 and side == 1:
            h[0, 64 + 3, 0, 0] = np.nan  # a text token of V

    err = p.commit(poison=nan_text)
    assert err is not None and "non-finite v" in err.msg
    p.check()

    def nan_video(layer, side, h):
        if layer == 0 and side == 0:
            h[0, 5, 1, 2] = np.nan  # video tokens are not checked (history.rs:263-267)

    assert p.commit(poison=nan_video) is None
    p.check()
    p.close()


def test_qvg_failed_first_commit_keeps_fitted_codebooks(H):
    """history.rs:256-276: the fit runs before the text is quantized, so a
    first commit rejected for its text still freezes the codebooks."""
    p = _pair(H, "qvg", "uniform", past=6, model_dtype="bf16", input_dtype="f32", tpf=32, text=8, frames=2,
              n_layers=1)

    def inf_text(layer, side, h):
        if layer == 0 and side == 0:
            h[0, 70, 0, 0] = np.inf

    err = p.commit(poison=inf_text)
    assert err is not None and "non-finite k" in err.msg
    assert p.o.codebooks(0) is not None
    p.check()
    assert p.commit() is None
    p.check()
    p.close()


def test_qvg_bank_fit_state_after_failed_first_commit(H):
    """In KvBank's loop a commit failing at layer 0 never reaches layer 1's
    fit; the bank drops the fits of the layers after the first failing one."""
    p = _pair(H, "qvg", "uniform", past=6, model_dtype="bf16", input_dtype="f32", tpf=32, text=8, frames=2)

    def inf_text(layer, side, h):
        if layer == 0 and side == 0:
            h[0, 70, 0, 0] = np.inf

    assert p.commit(poison=inf_text) is not None
    assert p.o.codebooks(0) is not None and p.o.codebooks(1) is None
    assert p.p.layer(0).qvg_codebooks() is not None and p.p.layer(1).qvg_codebooks() is None
    # bitwise; the inf in the fitted rows makes NaN entries, compared by position
    assert H.same_values(p.o.codebooks(0), p.p.layer(0).qvg_codebooks(), "f32").all()
    p.close()


# ---------------------------------------------------------------- errors
@pytest.mark.parametrize("storage", ["int8", "float"])
def test_nonfinite_rejection_leaves_cache_unchanged(H, storage):
    p = _pair(H, storage, "uniform", past=6, model_dtype="bf16", input_dtype="f32")
    assert p.commit() is None

    def poison(layer, side, h):
        if layer == 0 and side == 0:
            h[0, 17, 2, 5] = np.float32(np.finfo(np.float32).max)  # |x| >= f32::MAX (int8.rs:110-116)

    err = p.commit(poison=poison)
    if storage == "int8":
        assert err is not None and err.msg == "cannot quantize non-finite k values"
    else:
        assert err is None  # FLOAT storage does not scan (history.rs:243-247)
    p.check()
    assert p.commit() is None
    p.check()
    p.close()


def test_bank_commit_is_all_or_nothing(H):
    """Deliberate deviation: the reference's KvBank::commit (cache/mod.rs:
    257-268) stops at the first failing layer and leaves the layers before it
    committed; the bank rejects the segment on every layer.  The error itself
    (kind and message) is the reference's."""
    p = _pair(H, "int8", "uniform", past=6, model_dtype="bf16", input_dtype="f32")
    assert p.commit() is None

    def poison(layer, side, h):
        if layer == 1 and side == 1:
            h[0, 3, 0, 0] = np.nan

    err = p.commit(poison=poison)
    assert err is not None and err.msg == "cannot quantize non-finite v values"
    assert p.o.info(0)["n_segments"] == 2 and p.o.info(1)["n_segments"] == 1  # reference: partial
    for layer in range(2):
        assert p.p.layer(layer).n_segments() == 1  # bank: unchanged
    assert p.p.metrics().archived_segments == 1 and p.p.metrics().rebuilds == 1
    p.close()


def test_geometry_and_chronology_errors(H):
    p = _pair(H, "int8", "uniform", past=6)
    assert p.commit(frame_start=1) is not None  # first segment must start at frame 0
    assert p.commit() is None
    assert p.commit(segment_index=0) is not None  # chronological writes
    assert p.commit(frame_start=7) is not None  # frame_start continues the timeline
    assert p.commit(action_start=17) is not None  # outside the text block
    assert p.commit(action_start=-2) is not None
    assert p.commit(frames=0, image_tokens=0) is not None
    assert p.commit(frames=3, image_tokens=100) is not None  # not divisible
    assert p.commit(frames=2, image_tokens=200) is not None  # tokens_per_frame changed
    assert p.commit(action_start=16) is None
    p.check()
    p.close()


def test_tokens_per_frame_recorded_by_failed_first_commit(H):
    # one layer: in a multi-layer KvBank only the first layer would record it
    p = _pair(H, "int8", "uniform", past=6, n_layers=1)
    assert p.commit(frame_start=2) is not None  # fails after learning tpf = 64
    assert p.commit(frames=2, image_tokens=100, frame_start=0) is not None  # tpf 50 != 64
    p.check()
    p.close()


def test_rollback_errors(H):
    p = _pair(H, "int8", "uniform")
    assert p.rollback() is not None  # nothing to roll back (interactive.rs:86-95 style)
    p.close()
    p = _pair(H, "int8", "recent")
    assert p.commit() is None
    err = p.rollback()
    assert err is not None and "recent-mode SWA" in err.msg
    p.check()
    p.close()


def test_capacity_overflow_archives_then_errors(H):
    """history.rs:416-421: the rebuild fails after the segment was archived."""
    p = _pair(H, "int8", "uniform", past=6, capacity=300, n_layers=1)
    assert p.commit() is None
    err = p.commit()
    assert err is not None and "capacity is 300" in err.msg
    p.check()  # archive grew, working set and rebuild counter did not
    assert p.rollback() is None
    p.check()
    p.close()


def test_capacity_overflow_in_a_bank_archives_every_layer(H):
    """KvBank stops after the first layer's rebuild error; the bank keeps its
    layers in lockstep, so every layer holds the archived segment (each
    layer exactly as the reference's HistoryCache leaves it)."""
    p = _pair(H, "int8", "uniform", past=6, capacity=300)
    assert p.commit() is None
    err = p.commit()
    assert err is not None and "capacity is 300" in err.msg
    for layer in range(2):
        assert p.p.layer(layer).n_segments() == 2 and p.p.layer(layer).total_frames() == 6
    assert p.o.info(0)["n_segments"] == 2 and p.o.layer_metrics(0) == p.p.layer(0).metrics().as_dict()
    p.close()


# --------------------------------------------------------- session.rs
def test_session_f32_lifelong_cache_grows_unbounded(H):  # session.rs:89-102
    p = _pair(H, "float", "recent", past=64, heads=4, head_dim=16, tpf=64, frames=3, text=32)
    toks = []
    for _ in range(4):
        assert p.commit() is None
        toks.append(p.p.layer(0).valid_len())
    assert all(a < b for a, b in zip(toks, toks[1:]))
    m = p.p.metrics()
    assert m.archived_segments == 4 and m.rebuilds == 4 and p.p.layer(0).total_frames() == 12
    p.check()
    p.close()


def test_session_int8_uniform_history_respects_frame_budget(H):  # session.rs:104-134
    p = _pair(H, "int8", "uniform", past=5, heads=4, head_dim=16, tpf=64, frames=3, text=32)
    for _ in range(4):
        assert p.commit() is None
    tokens = p.p.layer(0).valid_len()
    assert (tokens - 5 * 64) % 32 == 0 and tokens < 12 * 64 + 4 * 32
    assert p.p.metrics().encode_calls >= 4
    p.check()
    p.close()


def test_session_qvg_storage_smaller_than_float(H):  # session.rs:136-155
    p = _pair(H, "qvg", "uniform", past=6, heads=4, head_dim=16, tpf=64, frames=3, text=32)
    for _ in range(3):
        assert p.commit() is None
    m = p.p.metrics()
    assert p.p.layer(0).total_frames() == 9 and m.encode_calls >= 3
    assert m.archived_bytes < 3 * 9 * 8 * 8 * 4 * 64 * 8 * 2
    p.check()
    p.close()


def test_session_swa_capacity_bounds_working_set(H):  # session.rs:172-187
    tpf = 64
    p = _pair(H, "float", "recent", capacity=2 * tpf + 40, heads=4, head_dim=16, tpf=tpf, frames=3, text=32)
    for _ in range(4):
        assert p.commit() is None
        assert p.p.layer(0).valid_len() <= 2 * tpf + 40 + 2 * tpf
    assert p.p.metrics().evicted_tokens > 0
    p.check()
    p.close()


# ----------------------------------------------------- interactive.rs
def test_rollback_restores_cache_state(H):  # interactive.rs:60-83
    p = _pair(H, "float", "uniform", past=32, heads=4, head_dim=16, tpf=64, frames=2, text=20)
    for i in range(3):
        assert p.commit() is None
        assert p.p.layer(0).n_segments() == i + 1
    before = p.p.layer(0).valid_len()
    assert p.rollback() is None
    assert p.p.layer(0).n_segments() == 2 and p.p.layer(0).total_frames() == 4
    assert p.p.layer(0).valid_len() <= before
    assert p.commit() is None
    assert p.p.layer(0).n_segments() == 3 and p.p.layer(0).total_frames() == 6
    p.check()
    p.close()


@pytest.mark.parametrize("storage", ["float", "int8", "qvg"])
def test_phase_swap_moves_working_set(H, storage):  # interactive.rs:106-125
    p = _pair(H, storage, "uniform", past=32, phase_swap=True, frames=2, model_dtype="bf16")
    assert p.commit() is None
    assert p.park() is None
    p.check()
    with pytest.raises(Exception):
        p.p.layer(0).working_set()  # parked (phase_swap.rs:107-114)
    assert p.park() is None  # idempotent
    assert p.unpark() is None
    p.check()
    m = p.p.metrics()
    assert m.d2h_bytes > 0 and m.h2d_bytes > 0
    p.close()


def test_commit_and_rollback_while_parked_keep_reference_quirk(H):
    """phase_swap.rs:69-81: unpark restores the stale parked set even if a
    commit or rollback rebuilt the inner cache while parked."""
    p = _pair(H, "int8", "uniform", past=32, phase_swap=True, frames=2)
    assert p.commit() is None
    assert p.commit() is None
    assert p.park() is None
    assert p.commit() is None
    p.check(working_sets=False)
    assert p.rollback() is None
    assert p.unpark() is None
    p.check()
    p.close()


def test_multi_turn_session_with_rollback_flow(H):  # interactive.rs:127-151
    p = _pair(H, "float", "uniform", past=32, phase_swap=True, frames=2)
    for _ in range(2):
        assert p.commit() is None
        assert p.park() is None and p.unpark() is None
    assert p.rollback() is None
    assert p.commit() is None
    assert p.park() is None and p.unpark() is None
    assert p.p.layer(0).total_frames() == 4 and p.p.metrics().rollbacks == 1
    p.check()
    p.close()


def test_long_random_sessions(H):
    """Random op sequences (commits of varying size, rollbacks, park/unpark)."""
    rng = np.random.default_rng(11)
    for trial in range(6):
        storage = ["int8", "float", "qvg"][trial % 3]
        sampling = ["uniform", "recent_mix", "temporal09", "temporal"][trial % 4]
        p = _pair(H, storage, sampling, past=int(rng.integers(2, 9)), phase_swap=bool(trial % 2), frames=2,
                  tpf=16, text=5, model_dtype="bf16", input_dtype="bf16")
        for _ in range(14):
            op = rng.random()
            if op < 0.6:
                p.commit(frames=int(rng.integers(1, 4)), text=int(rng.integers(0, 7)))
            elif op < 0.8:
                p.rollback()
            elif op < 0.9:
                p.park()
            else:
                p.unpark()
            p.check(archive=False)
        p.unpark()
        p.check()
        p.close()


def test_decode_segment_matches_oracle(H):
    import torch
    for storage in ("int8", "qvg", "float"):
        p = _pair(H, storage, "uniform", past=4, model_dtype="bf16", input_dtype="bf16", tpf=32, frames=2, text=9)
        for _ in range(3):
            assert p.commit() is None
        L = 2 * 32 + 9
        ko = [torch.empty((1, L, 4, 32), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
        vo = [torch.empty_like(k) for k in ko]
        for pos in range(3):
            p.p.decode_segment(pos, ko, vo)
            for layer in range(2):
                kr, vr = p.o.decode_segment(layer, pos, L)
                assert np.array_equal(H.torch_to_raw(ko[layer]), kr)
                assert np.array_equal(H.torch_to_raw(vo[layer]), vr)
        p.close()


def _sigma_codebooks(p, seed):
    rng = np.random.default_rng(seed)
    cbs = []
    for _ in range(p.geo.n_layers):
        cb = np.zeros((2, p.geo.heads, 4, 4, p.geo.head_dim), np.float32)
        for s, sig in enumerate((1.0, 0.5, 0.25, 0.125)):
            cb[:, :, s] = rng.standard_normal(cb[:, :, s].shape).astype(np.float32) * np.float32(sig)
        cbs.append(cb)
    return cbs


@pytest.mark.parametrize("model_dtype", ["bf16", "f16", "f32"])
def test_qvg_table_gather_d128_ragged_heads_and_blocks(H, model_dtype):
    """head_dim 128 with the default codec takes the table-driven decoder:
    6 heads (a group of 4 and a group of 2), 100-token frames so frame runs
    start and end inside 64-token payload blocks, frozen codebooks."""
    p = _pair(H, "qvg", "uniform", past=4, model_dtype=model_dtype, input_dtype="bf16", heads=6, head_dim=128,
              tpf=100, frames=3, text=9)
    p.set_codebooks(_sigma_codebooks(p, 11))
    for _ in range(4):
        assert p.commit() is None
        p.check()
    p.close()


@pytest.mark.parametrize("sampling", ["recent_mix", "temporal09"])
def test_qvg_table_gather_d128_fitted_codebooks(H, sampling):
    p = _pair(H, "qvg", sampling, past=4, model_dtype="bf16", input_dtype="f32", heads=5, head_dim=128,
              tpf=70, frames=2, text=6)
    for _ in range(5):
        assert p.commit() is None
        p.check()
    assert p.rollback() is None
    p.check()
    p.close()


def test_qvg_table_gather_d128_video_nan(H):
    p = _pair(H, "qvg", "uniform", past=4, model_dtype="bf16", input_dtype="f32", heads=4, head_dim=128,
              tpf=64, frames=2, text=4)
    p.set_codebooks(_sigma_codebooks(p, 3))

    def nan_video(layer, side, h):
        if side == 0:
            h[0, 70, 3, 100] = np.nan
            h[0, 5, 0, :] = np.inf

    assert p.commit(poison=nan_video) is None
    p.check()
    assert p.commit() is None
    p.check()
    p.close()


def test_qvg_decode_segment_d128_aligned_and_unaligned_outputs(H):
    """Aligned caller buffers take the table-driven decoder, unaligned ones
    the element-wise kernel; both must equal the oracle."""
    import torch
    p = _pair(H, "qvg", "uniform", past=4, model_dtype="bf16", input_dtype="bf16", heads=4, head_dim=128,
              tpf=90, frames=2, text=5)
    for _ in range(3):
        assert p.commit() is None
    L = 2 * 90 + 5
    n = L * 4 * 128
    for offset in (0, 1):
        ko = [torch.empty(n + offset, dtype=torch.bfloat16, device="cuda")[offset:].view(1, L, 4, 128)
              for _ in range(2)]
        vo = [torch.empty(n + offset, dtype=torch.bfloat16, device="cuda")[offset:].view(1, L, 4, 128)
              for _ in range(2)]
        for pos in range(3):
            p.p.decode_segment(pos, ko, vo)
            for layer in range(2):
                kr, vr = p.o.decode_segment(layer, pos, L)
                assert np.array_equal(H.torch_to_raw(ko[layer]), kr), (offset, pos, layer)
                assert np.array_equal(H.torch_to_raw(vo[layer]), vr), (offset, pos, layer)
    p.close()


def _qvg_pair(H, stages, bits, block=64, **geo):
    import nomas_kv as nk
    spec = H.Spec(storage=STORAGES["qvg"], sampling=SAMPLINGS["uniform"][0], past_frames=4,
                  qvg=nk.QvgConfig(stages=stages, bits_per_stage=bits, block_size=block))
    return H.Pair(H.Geometry(**geo), spec)


@pytest.mark.parametrize("stages,bits,head_dim,input_dtype", [(4, 2, 128, "bf16"), (2, 3, 32, "f32"),
                                                              (3, 4, 24, "f16"), (8, 2, 16, "bf16"),
                                                              (1, 8, 8, "f32")])
def test_qvg_device_fit_matches_oracle(H, stages, bits, head_dim, input_dtype):
    """The first commit fits every layer's codebooks on the device
    (farthest-point init + two Lloyd iterations per stage, qvg.rs:351-442);
    they must equal the oracle's bit for bit, as must everything after."""
    p = _qvg_pair(H, stages, bits, model_dtype="bf16", input_dtype=input_dtype, heads=3, head_dim=head_dim, tpf=40,
                  frames=2, text=7)
    for _ in range(3):
        assert p.commit() is None
        p.check()
    p.close()


def test_qvg_device_fit_identical_rows_take_the_jitter_path(H):
    """Rows that all coincide make the farthest-point total 0 (<= 1e-12):
    the reference copies entry 0 and nudges its first value by k * 1e-3."""
    p = _qvg_pair(H, 4, 2, model_dtype="f32", input_dtype="f32", heads=2, head_dim=16, tpf=32, frames=2, text=4)

    def constant(layer, side, h):
        h[...] = 0.75 if side == 0 else -1.25

    assert p.commit(poison=constant) is None
    p.check()
    assert p.commit() is None
    p.check()
    p.close()


def test_qvg_device_fit_with_nan_and_inf_rows(H):
    """Non-finite values in the fitted video rows (not checked by the
    reference before the fit) must steer the fit exactly as on the CPU."""
    p = _qvg_pair(H, 4, 2, model_dtype="bf16", input_dtype="f32", heads=2, head_dim=32, tpf=32, frames=2, text=0)

    def poison(layer, side, h):
        h[0, 3, 1, 5] = np.nan
        h[0, 40, 0, :] = np.inf

    assert p.commit(poison=poison) is None
    p.check()
    p.close()
