"""The fused dequant-in-attention consumer (nkv_bank_attend_history).

The history part of the reference's attention (modules/attention.rs:
143-189; masks.rs: every current token sees every history token) computed
straight from the INT8 archive by the tcgen05 kernel of kernels_attn.cu,
against the oracle's dequantized working set (int8.rs:139-155, history.rs:
341-446) followed by a float64 PyTorch softmax attention.  Tolerances: the
row log-sum-exp within 2e-3 (scores are f32 sums of exact bf16 products), the
outputs within 2e-2 absolute (the kernel rounds its unnormalised
probabilities to bf16 for the P V product, as the reference rounds its
normalised ones; 2^-9 relative on values of magnitude ~4).
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    return cache_harness


def _reference(k_raw, v_raw, q, scale):
    """float64 softmax(q k^T * scale) v per head; k_raw / v_raw (1, L, H, D)
    bf16 bit patterns, q (n, H, D) bf16 tensor."""
    import torch
    k = torch.from_numpy(k_raw.view(np.int16)).view(torch.bfloat16)[0].to("cuda").double()
    v = torch.from_numpy(v_raw.view(np.int16)).view(torch.bfloat16)[0].to("cuda").double()
    qd = q.double()
    s = torch.einsum("qhd,khd->hqk", qd, k) * scale
    lse = torch.logsumexp(s, dim=-1)
    o = torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v)
    return o.cpu(), lse.cpu()


def _check(H, pair, layer, q, scale=None):
    import torch
    out, lse = pair.p.layer(layer).attend_history(q, scale)
    torch.cuda.synchronize()
    ko, vo = pair.o.working_set(layer)
    s = scale if scale is not None else 1.0 / math.sqrt(pair.geo.head_dim)
    o_ref, lse_ref = _reference(ko, vo, q, s)
    dl = (lse.double().cpu() - lse_ref).abs().max().item()
    do = (out.double().cpu() - o_ref).abs().max().item()
    assert dl < 2e-3, f"lse differs by {dl}"
    assert do < 2e-2, f"out differs by {do}"
    return do, dl


def _pair(H, **geo):
    import nomas_kv as nk
    spec = H.Spec(storage=nk.NKV_STORAGE_INT8, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=5)
    g = dict(n_layers=2, heads=4, head_dim=128, tpf=70, frames=3, text=9, model_dtype="bf16", input_dtype="bf16")
    g.update(geo)
    return H.Pair(H.Geometry(**g), spec)


def test_attend_history_matches_oracle_attention(H):
    import torch
    p = _pair(H)
    try:
        gen = torch.Generator(device="cuda").manual_seed(3)
        for n in range(6):
            assert p.commit() is None
            if n in (0, 2, 5):
                # a partial query tile; ragged key tiles (runs of 70 / 140 video and 9 text tokens)
                q = torch.randn((200, 4, 128), generator=gen, device="cuda").to(torch.bfloat16)
                for layer in range(2):
                    _check(H, p, layer, q)
        q = (3.0 * torch.randn((129, 4, 128), generator=gen, device="cuda")).to(torch.bfloat16)
        _check(H, p, 1, q, scale=0.2)  # sharper rows: the running maximum moves
    finally:
        p.close()


def test_attend_history_follows_rollback_and_phase_swap(H):
    import torch
    import nomas_kv as nk
    spec = H.Spec(storage=nk.NKV_STORAGE_INT8, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=5, phase_swap=True)
    p = H.Pair(H.Geometry(n_layers=1, heads=2, head_dim=128, tpf=40, frames=2, text=5, model_dtype="bf16",
                          input_dtype="bf16"), spec)
    try:
        q = torch.randn((64, 2, 128), device="cuda").to(torch.bfloat16)
        for _ in range(4):
            assert p.commit() is None
        assert p.rollback() is None
        _check(H, p, 0, q)
        assert p.park() is None
        with pytest.raises(nk.CacheStateError, match="parked"):
            p.p.layer(0).attend_history(q)
        assert p.unpark() is None
        _check(H, p, 0, q)
    finally:
        p.close()


def test_attend_history_rejects_other_storage_and_empty_history(H):
    import torch
    import nomas_kv as nk
    q = torch.zeros((8, 4, 128), dtype=torch.bfloat16, device="cuda")
    p = _pair(H)
    try:
        with pytest.raises(nk.CacheStateError, match="no history"):
            p.p.layer(0).attend_history(q)
        assert p.commit() is None
        for bad in (0.0, -0.1, float("inf"), float("nan")):
            with pytest.raises(nk.ArgumentError, match="scale"):
                p.p.layer(0).attend_history(q, bad)
        with pytest.raises(nk.GeometryError, match="out / lse"):
            p.p.layer(0).attend_history(q, out=torch.empty((7, 4, 128), device="cuda"))
    finally:
        p.close()
    spec = H.Spec(storage=nk.NKV_STORAGE_QVG, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=5)
    p = H.Pair(H.Geometry(n_layers=1, heads=4, head_dim=128, tpf=64, frames=2, text=4, model_dtype="bf16",
                          input_dtype="bf16"), spec)
    try:
        assert p.commit() is None
        with pytest.raises(nk.InvalidConfigError, match="INT8"):
            p.p.layer(0).attend_history(q)
    finally:
        p.close()


def test_attend_history_at_8b_geometry(H, orc):
    """24 heads, 17 segments of 4 x 1,560 + 256 tokens, uniform history of
    16 frames: 29,056 history keys; 640 queries checked (a full segment's
    queries take the same path)."""
    import os
    import torch
    import nomas_kv as nk
    orc.set_threads(os.cpu_count() or 1)
    spec = H.Spec(storage=nk.NKV_STORAGE_INT8, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=16)
    p = H.Pair(H.Geometry(n_layers=1, heads=24, head_dim=128, tpf=1560, frames=4, text=256, model_dtype="bf16",
                          input_dtype="bf16", key_sigma=1.0), spec, host_from_device=True)
    try:
        for _ in range(17):
            assert p.commit() is None
        assert p.p.layer(0).valid_len() == 29056
        q = torch.randn((640, 24, 128), device="cuda").to(torch.bfloat16)
        _check(H, p, 0, q)
    finally:
        p.close()
        orc.set_threads(1)


def test_attend_history_with_host_tier_archive(H):
    """Records in the pinned-host tier are read with plain loads, records in
    device memory by TMA: the same result either way."""
    import torch
    import nomas_kv as nk
    p = _pair(H)
    try:
        desc = nk._abi.nkv_segment_desc(0, 0, p.geo.frames, p.geo.frames * p.geo.tpf, p.geo.text, -1)
        p.p.set_archive_device_limit(2 * p.p.segment_bytes(desc) * p.geo.n_layers)
        for _ in range(6):
            assert p.commit() is None
        dev, host = p.p.archive_usage()
        assert dev > 0 and host > 0, (dev, host)
        q = torch.randn((200, 4, 128), device="cuda").to(torch.bfloat16)
        for layer in range(2):
            _check(H, p, layer, q)
    finally:
        p.close()


def test_attend_history_whole_and_split_units(H):
    """10,000 queries x 4 heads = 160 units of 256 queries: the first 148 run
    whole, the last 12 are split into key ranges and merged."""
    import torch
    p = _pair(H)
    try:
        for _ in range(6):
            assert p.commit() is None
        gen = torch.Generator(device="cuda").manual_seed(5)
        q = (2.0 * torch.randn((10000, 4, 128), generator=gen, device="cuda")).to(torch.bfloat16)
        _check(H, p, 1, q)
    finally:
        p.close()
