"""Archive persistence: nkv_bank_save / nkv_bank_load (no counterpart in the
reference, whose archive lives in memory only).

A session runs on a bank and on the oracle; the bank is saved, a fresh bank
with the same configuration loads the file and must match the original in
every observable (status, layouts, counters, working sets bit for bit,
archived payload bytes, QVG codebooks); then it replaces the original and the
session continues, still bit-exact against the oracle.  The refusals (fresh
bank required, same configuration, not parked, current working set, an
intact file) are checked too."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    return cache_harness


def _pair(H, storage, sampling, capacity=None, phase_swap=False, **geo):
    spec = H.Spec(storage=storage, sampling=sampling, gamma=2.0, past_frames=4, capacity=capacity,
                  phase_swap=phase_swap)
    return H.Pair(H.Geometry(**geo), spec)


def _fresh_bank(p):
    import nomas_kv as nk
    g = p.geo
    return nk.KvBank(p.spec.product(), g.n_layers, g.batch, g.heads, g.head_dim, p.mdt_p, device=p.device)


def _same_bank(H, p, q):
    """Every observable of bank q equals bank p's."""
    g = p.geo
    assert p.p.metrics().as_dict() == q.metrics().as_dict()
    for layer in range(g.n_layers):
        a, b = p.p.layer(layer), q.layer(layer)
        assert (a.valid_len(), a.capacity(), a.n_segments(), a.total_frames(), a.tokens_per_frame()) == \
            (b.valid_len(), b.capacity(), b.n_segments(), b.total_frames(), b.tokens_per_frame())
        assert [x.as_tuple() for x in a.working_layout()] == [x.as_tuple() for x in b.working_layout()]
        assert a.metrics().as_dict() == b.metrics().as_dict()
        ka, va = a.working_set()
        kb, vb = b.working_set()
        for x, y in ((ka, kb), (va, vb)):
            assert np.array_equal(H.torch_to_raw(x), H.torch_to_raw(y))
        for pos in range(a.n_segments()):
            assert np.array_equal(np.asarray(a.export_segment(pos)), np.asarray(b.export_segment(pos)))
        if p.spec.storage == 2:
            ca, cb = a.qvg_codebooks(), b.qvg_codebooks()
            assert (ca is None) == (cb is None)
            if ca is not None:
                assert H.same_values(ca, cb, "f32").all()


def _round_trip(H, p, tmp_path, more=3):
    path = tmp_path / "bank.nkv"
    p.p.save(path)
    q = _fresh_bank(p)
    q.load(path)
    _same_bank(H, p, q)
    p.p.close()
    p.p = q  # the session continues on the loaded bank
    for _ in range(more):
        assert p.commit() is None
        p.check()


@pytest.mark.parametrize("storage,sampling,model_dtype", [(1, 1, "bf16"), (1, 3, "f32"), (0, 2, "f16")])
def test_save_load_round_trip_and_continue(H, tmp_path, storage, sampling, model_dtype):
    p = _pair(H, storage, sampling, model_dtype=model_dtype, input_dtype="bf16")
    for _ in range(5):
        assert p.commit() is None
    p.check()
    _round_trip(H, p, tmp_path)
    assert p.rollback() is None  # the loaded archive rolls back like the original
    p.check()
    p.close()


def test_save_load_qvg_with_fitted_codebooks(H, tmp_path):
    p = _pair(H, 2, 1, model_dtype="bf16", input_dtype="bf16", heads=3, head_dim=128, tpf=40, frames=2, text=5)
    for _ in range(3):
        assert p.commit() is None
    p.check()
    _round_trip(H, p, tmp_path)
    p.close()


def test_save_load_recent_swa_with_evictions(H, tmp_path):
    p = _pair(H, 1, 0, capacity=2 * 64 + 16)
    for _ in range(4):
        assert p.commit() is None
    p.check()
    _round_trip(H, p, tmp_path)
    p.close()


def test_save_load_empty_bank(H, tmp_path):
    p = _pair(H, 1, 1)
    _round_trip(H, p, tmp_path, more=2)
    p.close()


def test_load_refusals(H, tmp_path, nkv):
    nk = nkv
    p = _pair(H, 1, 1)
    for _ in range(3):
        assert p.commit() is None
    path = tmp_path / "bank.nkv"
    p.p.save(path)
    with pytest.raises(nk.CacheStateError):
        p.p.load(path)  # not fresh
    other = _pair(H, 1, 3)  # different sampling
    with pytest.raises(nk.InvalidConfigError):
        other.p.load(path)
    other.close()
    truncated = tmp_path / "short.nkv"
    truncated.write_bytes(path.read_bytes()[:-1000])
    q = _fresh_bank(p)
    with pytest.raises(nk.MsgError):
        q.load(truncated)
    assert q.layer(0).n_segments() == 0 and q.layer(0).valid_len() == 0
    q.load(path)  # a failed load leaves the bank fresh
    _same_bank(H, p, q)
    q.close()
    (tmp_path / "junk.nkv").write_bytes(b"not an archive" * 10)
    q = _fresh_bank(p)
    with pytest.raises(nk.MsgError):
        q.load(tmp_path / "junk.nkv")
    q.close()
    p.close()


def test_save_refused_while_parked_or_stale(H, tmp_path, nkv):
    nk = nkv
    p = _pair(H, 1, 1, phase_swap=True)
    for _ in range(2):
        assert p.commit() is None
    assert p.park() is None
    with pytest.raises(nk.CacheStateError):
        p.p.save(tmp_path / "a.nkv")
    assert p.commit() is None  # a commit while parked: unpark restores the older set
    assert p.unpark() is None
    with pytest.raises(nk.CacheStateError):
        p.p.save(tmp_path / "a.nkv")
    assert p.commit() is None  # a fresh rebuild makes the working set current again
    p.p.save(tmp_path / "a.nkv")
    p.close()
    # a rebuild over capacity archives the segment but keeps the old working set
    p = _pair(H, 1, 1, capacity=250)  # one segment (208 tokens) fits, two sampled segments do not
    assert p.commit() is None
    err = p.commit()
    assert err is not None and "capacity" in err.msg
    with pytest.raises(nk.CacheStateError):
        p.p.save(tmp_path / "b.nkv")
    p.close()
