"""Config 1 golden vectors (tests/golden/config1_int8.json).

The CPU test pins the oracle to the committed vectors.  The GPU test runs
the product through the C ABI on the same seeded inputs and checks every
committed figure: per commit and layer the working set's bytes (SHA-256),
layout, info counters and metrics; after the session every archived
segment's INT8 payload (SHA-256 of codes K, codes V, scales K, scales V,
the export layout of nkv_cache_export_segment)."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_config1 as g1  # noqa: E402

GOLDEN = json.load(open(g1.PATH))


def test_golden_geometry_is_config1():
    geo = GOLDEN["geometry"]
    assert (geo["n_layers"], geo["heads"], geo["head_dim"], geo["tokens_per_frame"], geo["frames"], geo["text"],
            geo["segments"]) == (2, 4, 32, 64, 3, 16, 4)
    assert set(GOLDEN["scenarios"]) == {"uniform6", "recent192", "recent208"}


def test_oracle_reproduces_config1_golden(orc):
    fresh = json.loads(json.dumps(g1.generate()))  # same float formatting as the file
    assert fresh == GOLDEN


def test_config1_golden_session_counters():
    """The tiny session's accounting: one rebuild and two encode calls per
    commit per layer, 4 archived segments of 208 tokens (59,904 B each)."""
    for name, s in GOLDEN["scenarios"].items():
        m = s["commits"][-1]["metrics"]
        assert m["rebuilds"] == 4 and m["encode_calls"] == 8 and m["archived_segments"] == 4, name
        assert m["archived_bytes"] == 2 * 4 * 208 * (2 * 4 * 32 + 2 * 4 * 4), name
        assert all(a["bytes"] == 208 * (2 * 4 * 32 + 2 * 4 * 4) for per in s["archive"] for a in per)


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["uniform6", "recent192", "recent208"])
def test_product_matches_config1_golden(nkv, name):
    import torch
    nk = nkv
    gold = GOLDEN["scenarios"][name]
    samp = {"uniform": nk.NKV_SAMPLING_UNIFORM, "recent": nk.NKV_SAMPLING_RECENT}[gold["sampling"]]
    cfg = nk.CacheConfig(storage=nk.CacheStorage.int8(), sampling=nk.HistorySampling(samp, 2.0),
                         capacity=gold["capacity"], past_frames=gold["past_frames"])
    bank = nk.KvBank(cfg, g1.N_LAYERS, 1, g1.H, g1.D, torch.float32, device=torch.device("cuda:0"))
    for i, step in enumerate(gold["commits"]):
        seg = g1.segment_desc(i)
        ks, vs = g1.inputs(i, g1.FRAMES * g1.TPF + g1.TEXT)
        desc = nk._abi.nkv_segment_desc(seg["segment_index"], seg["frame_start"], seg["frame_count"],
                                        seg["image_tokens"], seg["text_tokens"], seg["action_start"])
        bank.commit_tensors(desc, [torch.from_numpy(k).cuda() for k in ks], [torch.from_numpy(v).cuda() for v in vs])
        assert bank.metrics().as_dict() == step["metrics"]
        for l, want in enumerate(step["layers"]):
            lc = bank.layer(l)
            info = {"valid_len": lc.valid_len(), "capacity": lc.capacity(), "n_segments": lc.n_segments(),
                    "total_frames": lc.total_frames(), "tokens_per_frame": lc.tokens_per_frame(),
                    "parked": int(lc.is_parked())}
            assert info == want["info"]
            assert [list(x.as_tuple()) for x in lc.working_layout()] == want["layout"]
            assert lc.metrics().as_dict() == want["metrics"]
            k, v = lc.working_set()
            k, v = k.cpu().numpy(), v.cpu().numpy()
            assert _sha(k) == want["k_sha256"], f"commit {i} layer {l} K working set"
            assert _sha(v) == want["v_sha256"], f"commit {i} layer {l} V working set"
            assert [float(x) for x in k.ravel()[:4]] == want["k_first"]
    for l, per in enumerate(gold["archive"]):
        assert bank.layer(l).n_segments() == len(per)
        for pos, want in enumerate(per):
            blob = np.asarray(bank.layer(l).export_segment(pos))
            assert blob.size == want["bytes"]
            assert _sha(blob) == want["sha256"], f"layer {l} segment {pos} payload"
    bank.close()


# ----------------------------------------------------- the commit producer
def test_oracle_reproduces_project_golden(orc):
    """The oracle's restatement of the captured K / V chain (+ quantize) still
    gives the committed digests (tests/golden/make_project.py)."""
    import make_project as mp

    golden = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "project_int8.json")))["cases"]
    for case, want in golden.items():
        _, got = mp.outputs(orc, case)
        for name in ("k", "v", "kq", "vq", "ks", "vs"):
            assert mp.digest(got[name]) == want[name], (case, name)
