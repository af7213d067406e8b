"""Config 4 (long session): 256 segments x 4 frames = 1,024 frames, bit-exact.

The samplers' index arithmetic, the Recent (SWA) trim and the rebuild
layouts depend on the session length, not on the per-token geometry, so
the full 1,024-frame session runs here at a small geometry (2 layers,
2 heads, head_dim 16, 8 tokens per frame, 4 text tokens) where the oracle
keeps up.  Cache configs: TemporalContext(0.9) and RecentMixUniform with
past = 32, and Recent with a capacity of 10 frames (the SWA mode; its
eviction only exists there, history.rs:345-360).  Eight rollbacks of 1-4
segments (20 in all) are spread over the session; Recent rejects them, as
the reference does.  After every operation: status, layout, counters and
the working set (bitwise) against the oracle; every 32 commits and at the
end also every archived payload."""
import pytest

pytestmark = pytest.mark.gpu

SEGMENTS = 256
ROLLBACK_AT = {20: 1, 45: 2, 77: 3, 101: 4, 140: 1, 171: 2, 205: 3, 240: 4}  # commit call -> segments


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    return cache_harness


def _session(H, sampling, gamma, capacity=None, storage=1, model_dtype="bf16"):
    geo = H.Geometry(n_layers=2, heads=2, head_dim=16, tpf=8, frames=4, text=4, model_dtype=model_dtype,
                     input_dtype="bf16")
    spec = H.Spec(storage=storage, sampling=sampling, gamma=gamma, past_frames=32, capacity=capacity)
    p = H.Pair(geo, spec)
    commits = 0  # commit calls so far (rollbacks are keyed on this, so each fires once)
    rollbacks = 0
    while p.o.info(0)["total_frames"] < 4 * SEGMENTS:
        assert p.commit() is None
        commits += 1
        p.check(archive=(commits % 32 == 0))
        for _ in range(ROLLBACK_AT.get(commits, 0)):
            if p.rollback() is None:
                rollbacks += 1
            p.check(archive=False)
        assert commits <= SEGMENTS + sum(ROLLBACK_AT.values())
    assert p.o.info(0)["total_frames"] == 4 * SEGMENTS
    p.check(archive=True)
    metrics = p.o.metrics()
    p.close()
    return rollbacks, metrics


def test_long_session_temporal_context_09(H):
    rollbacks, m = _session(H, 3, 0.9)
    assert rollbacks == 20 and m["rollbacks"] > 0


def test_long_session_recent_mix_uniform_32(H):
    rollbacks, m = _session(H, 2, 2.0)
    assert rollbacks == 20


def test_long_session_recent_swa_capacity(H):
    """Recent + capacity 10 frames: the trim evicts head frames / whole
    records every commit; rollbacks are rejected."""
    rollbacks, m = _session(H, 0, 2.0, capacity=10 * 8)
    assert rollbacks == 0 and m["evicted_tokens"] > 0


def test_long_session_qvg_temporal(H):
    """The same session with QVG storage (codebooks fitted on the first
    commit) under TemporalContext(0.9)."""
    rollbacks, m = _session(H, 3, 0.9, storage=2)
    assert rollbacks == 20
