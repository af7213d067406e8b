"""Bit-exact parity with the oracle at the geometry the benchmark measures.

The benchmark times the Nomas-8B geometry (24 heads, head_dim 128, segments
of 4 frames x 1,560 tokens + 256 text tokens, BF16 K/V with keys scaled per
channel by exp(N(0, 1)), uniform history of 16 past frames).  These sessions
run that geometry on two layers (INT8) and one layer (QVG with the bench's
frozen codebooks) through 17 commits: at 68 frames uniform_frame_indices
(cache/uniform_history.rs:10-19) picks 16 frames in 16 distinct segments,
so the rebuilt working set is the bench's 16 x 1,560 + 16 x 256 = 29,056
tokens (history.rs:341-446).  After the last commit the harness compares
with the oracle bit for bit: counters, layouts, every working set, every
archived payload (int8.rs:65-134; qvg.rs:173-256 with 98 blocks per side
and head, the last one 32 tokens), and the newest segment decoded in full
(history.rs:308-338, the bench's "+1 recent segment").
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GEO8 = dict(heads=24, head_dim=128, tpf=1560, frames=4, text=256, model_dtype="bf16", input_dtype="bf16", seed=0,
            key_sigma=1.0)
SEGMENTS = 17
WORKING_SET = 16 * 1560 + 16 * 256


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    # the oracle's independent loops (QVG heads, the segments a rebuild
    # decodes) on every host core; results do not depend on the count
    orc.set_threads(os.cpu_count() or 1)
    yield cache_harness
    orc.set_threads(1)


def _newest_segment_equal(H, p, n_layers):
    import torch
    L = 4 * 1560 + 256
    pos = p.o.info(0)["n_segments"] - 1
    ko = [torch.empty((1, L, 24, 128), dtype=torch.bfloat16, device="cuda") for _ in range(n_layers)]
    vo = [torch.empty_like(k) for k in ko]
    p.p.decode_segment(pos, ko, vo)
    for layer in range(n_layers):
        kr, vr = p.o.decode_segment(layer, pos, L)
        assert H.same_values(H.torch_to_raw(ko[layer]), kr).all(), f"layer {layer} newest segment K"
        assert H.same_values(H.torch_to_raw(vo[layer]), vr).all(), f"layer {layer} newest segment V"


def test_device_generator_equals_host_generator_at_8b_geometry(H):
    """The parity sessions below hand the oracle the device generator's
    tensors; here one 8B segment of both sides matches synth.host_values."""
    from nomas_kv import synth
    p = H.Pair(H.Geometry(n_layers=1, **GEO8), H.Spec(past_frames=16))
    kd, vd, kh, vh = p.inputs(5, 4 * 1560 + 256)
    for side, t in ((0, kd[0]), (1, vd[0])):
        host = synth.host_values(0, 1.0, 1, 4 * 1560 + 256, 24, 128, 0, 5, side, H.DT["bf16"][0])
        assert np.array_equal(H.torch_to_raw(t), host)
    p.close()


def test_config2_int8_uniform16_at_8b_geometry(H):
    """Config 2: INT8 storage, uniform history of 16 past frames, 2 layers."""
    import nomas_kv as nk
    spec = H.Spec(storage=nk.NKV_STORAGE_INT8, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=16)
    p = H.Pair(H.Geometry(n_layers=2, **GEO8), spec, host_from_device=True)
    try:
        for _ in range(SEGMENTS):
            assert p.commit() is None
        assert p.p.layer(0).valid_len() == WORKING_SET
        assert len({lay[0] for lay in p.o.layout(0)}) == 16  # 16 distinct segments represented
        p.check(working_sets=True, archive=True)
        _newest_segment_equal(H, p, 2)
    finally:
        p.close()


def test_config3_qvg_frozen_codebooks_at_8b_geometry(H):
    """Config 3: QVG storage with the bench's frozen codebooks (stages of
    sigma 1, 0.5, 0.25, 0.125), INT8 text, uniform decode-gather of 16 frames."""
    import nomas_kv as nk
    from nomas_kv import synth
    spec = H.Spec(storage=nk.NKV_STORAGE_QVG, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=16)
    p = H.Pair(H.Geometry(n_layers=1, **GEO8), spec, host_from_device=True)
    try:
        p.set_codebooks([synth.qvg_codebooks(0)])
        for _ in range(SEGMENTS):
            assert p.commit() is None
        assert p.p.layer(0).valid_len() == WORKING_SET
        # 6,240 video tokens: 98 blocks per side and head, the last of 32 tokens
        kc, vc, ksc, vsc = p.o.archive_qvg(0, 0, 4 * 1560)
        assert ksc.size == 24 * 98 * 4
        p.check(working_sets=True, archive=True)
        _newest_segment_equal(H, p, 1)
    finally:
        p.close()
