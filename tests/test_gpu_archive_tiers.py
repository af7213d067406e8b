"""The tiered archive: slabs beyond a device byte limit live in pinned host
memory mapped into the device's address space, and the cache's kernels read
(rebuild, decode) and write (quantize, QVG encode, float archive) them over
the host link.  Results must not depend on where a slab lives: every
session here runs with most of its archive in the host tier and is compared
with the oracle bit for bit after every operation (working sets, layouts,
counters, exported payloads), including rollback into the host tier, the
one-launch commit + decode, and save / load.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    return cache_harness


def _pair_with_limit(H, storage, segments_on_device=2, **geo):
    import nomas_kv as nk
    spec = H.Spec(storage=storage, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=4)
    p = H.Pair(H.Geometry(**geo), spec)
    desc = nk._abi.nkv_segment_desc(0, 0, p.geo.frames, p.geo.frames * p.geo.tpf, p.geo.text, -1)
    seg = p.p.segment_bytes(desc) * p.geo.n_layers
    p.p.set_archive_device_limit(segments_on_device * seg)
    return p, seg


@pytest.mark.parametrize("storage", ["int8", "qvg", "float"])
def test_host_tier_session_matches_oracle(H, storage):
    import nomas_kv as nk
    st = {"int8": nk.NKV_STORAGE_INT8, "qvg": nk.NKV_STORAGE_QVG, "float": nk.NKV_STORAGE_FLOAT}[storage]
    p, seg = _pair_with_limit(H, st, model_dtype="bf16", input_dtype="bf16")
    try:
        for _ in range(7):
            assert p.commit() is None
            p.check(working_sets=True, archive=True)
        dev, host = p.p.archive_usage()
        assert host >= 4 * seg and dev <= 2 * seg + 4096, (dev, host)
        for _ in range(3):  # rollbacks pop host slabs
            assert p.rollback() is None
            p.check(working_sets=True, archive=True)
        for _ in range(2):
            assert p.commit() is None
            p.check(working_sets=True, archive=True)
    finally:
        p.close()


def test_host_tier_commit_decode_and_save_load(H, tmp_path):
    import torch
    import nomas_kv as nk
    p, seg = _pair_with_limit(H, nk.NKV_STORAGE_INT8, model_dtype="bf16", input_dtype="bf16", head_dim=128)
    try:
        for _ in range(4):
            assert p.commit() is None
        g = p.geo
        L = g.frames * g.tpf + g.text
        kd, vd, kh, vh = p.inputs(4, L)
        dk = [torch.empty((1, L, g.heads, g.head_dim), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
        dv = [torch.empty_like(t) for t in dk]
        desc = nk._abi.nkv_segment_desc(4, 4 * g.frames, g.frames, g.frames * g.tpf, g.text, -1)
        p.o.commit(dict(segment_index=4, frame_start=4 * g.frames, frame_count=g.frames, image_tokens=g.frames * g.tpf,
                        text_tokens=g.text, action_start=-1), p.idt_o, kh, vh)
        p.p.commit_tensors(desc, kd, vd, decode_k=dk, decode_v=dv)
        p.next_index, p.next_frame = 5, 5 * g.frames
        p.sizes.append((g.frames * g.tpf, g.text))
        p.check(working_sets=True, archive=True)
        for layer in range(2):
            kr, vr = p.o.decode_segment(layer, 4, L)
            assert np.array_equal(H.torch_to_raw(dk[layer]), kr) and np.array_equal(H.torch_to_raw(dv[layer]), vr)
        # save from the tiered bank, load into a bank without a limit
        path = tmp_path / "tiered.nkv"
        p.p.save(path)
        fresh = nk.KvBank(p.spec.product(), g.n_layers, g.batch, g.heads, g.head_dim, torch.bfloat16, device="cuda")
        fresh.load(path)
        for layer in range(2):
            a, b = p.p.layer(layer).working_set(), fresh.layer(layer).working_set()
            assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
            for pos in range(5):
                assert np.array_equal(p.p.layer(layer).export_segment(pos), fresh.layer(layer).export_segment(pos))
        fresh.close()
    finally:
        p.close()


def test_staged_commit_refused_with_a_device_limit(H):
    import nomas_kv as nk
    p, _ = _pair_with_limit(H, nk.NKV_STORAGE_INT8, model_dtype="bf16", input_dtype="bf16", head_dim=128)
    try:
        desc = nk._abi.nkv_segment_desc(0, 0, p.geo.frames, p.geo.frames * p.geo.tpf, p.geo.text, -1)
        with pytest.raises(nk.InvalidConfigError, match="archive device limit"):
            p.p.stage_segment(desc)
        p.p.set_archive_device_limit(0)  # no limit: staging works again
        p.p.stage_segment(desc)
        p.p.discard_staged()
    finally:
        p.close()
