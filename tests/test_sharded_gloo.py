"""World-size-2 gloo test of the layer-sharded bank's host logic on CPU.

Each rank owns half the layers.  The per-rank bank is the CPU oracle (the
test injects it through ShardedKvBank's bank_factory), so the test checks
the sharding logic itself: layer partition, descriptor agreement, error
propagation across ranks, and that the all-reduced metrics equal a single
unsharded KvBank's (cache/mod.rs:305-319)."""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class OracleShard:
    """Oracle bank with the KvBank methods ShardedKvBank calls."""

    def __init__(self, orc, cfg, begin, count, H, D):
        self.orc, self.begin = orc, begin
        self.bank = orc.Bank(cfg, count, 1, H, D, orc.F32)

    def commit_tensors(self, desc, ks, vs):
        import nomas_kv as nk
        seg = dict(segment_index=desc.segment_index, frame_start=desc.frame_start, frame_count=desc.frame_count,
                   image_tokens=desc.image_tokens, text_tokens=desc.text_tokens, action_start=desc.action_start)
        try:
            self.bank.commit(seg, self.orc.F32, ks, vs)
        except self.orc.OracleError as e:
            raise nk._ERRORS[e.code](e.msg)

    def rollback(self):
        self.bank.rollback()

    def park_all(self):
        self.bank.park()

    def unpark_all(self):
        self.bank.unpark()

    def metrics(self):
        return self.bank.metrics()

    def close(self):
        self.bank.close()


def _inputs(seed, layer, seg, L, H, D):
    from nomas_kv import synth
    k = synth.host_values(seed, 0.5, 1, L, H, D, layer, seg, 0, 0)
    v = synth.host_values(seed, 0.5, 1, L, H, D, layer, seg, 1, 0)
    return k, v


def _worker(rank, world, port, q):
    try:
        for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "hy-nomas-rs_b200")):
            sys.path.insert(0, p)
        import torch.distributed as dist
        from datetime import timedelta
        import nomas_kv as nk
        import oracle as orc
        from nomas_kv.sharded import ShardedKvBank

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        n_layers, H, D, tpf, frames, text = 4, 2, 16, 8, 2, 3
        L = frames * tpf + text
        ocfg = orc.Config(storage=orc.INT8, sampling=orc.UNIFORM, past_frames=3)
        sb = ShardedKvBank(nk.CacheConfig(), n_layers, 1, H, D, 0,
                           bank_factory=lambda b, c: OracleShard(orc, ocfg, b, c, H, D), verify="strict")
        assert (sb.begin, sb.count) == nk.partition_layers(n_layers, world, rank)
        for s in range(3):
            desc = nk._abi.nkv_segment_desc(s, s * frames, frames, frames * tpf, text, -1)
            kv = [_inputs(0, sb.begin + i, s, L, H, D) for i in range(sb.count)]
            sb.commit(desc, [k for k, _ in kv], [v for _, v in kv])
        m = sb.metrics().as_dict()
        # the same session on one unsharded bank of all layers
        full = orc.Bank(ocfg, n_layers, 1, H, D, orc.F32)
        for s in range(3):
            kv = [_inputs(0, l, s, L, H, D) for l in range(n_layers)]
            full.commit(dict(segment_index=s, frame_start=s * frames, frame_count=frames, image_tokens=frames * tpf,
                             text_tokens=text, action_start=-1), orc.F32, [k for k, _ in kv], [v for _, v in kv])
        assert m == full.metrics(), (m, full.metrics())
        sb.rollback()
        full.rollback()
        assert sb.metrics().as_dict() == full.metrics()
        full.close()
        # descriptor disagreement is caught on every rank
        bad = nk._abi.nkv_segment_desc(2, 4 + rank, frames, frames * tpf, text, -1)
        try:
            sb.commit(bad, [], [])
            raise AssertionError("disagreement not detected")
        except nk.CacheStateError:
            pass
        # a non-finite input on rank 1 only: every rank reports the failure
        desc = nk._abi.nkv_segment_desc(2, 4, frames, frames * tpf, text, -1)
        kv = [_inputs(0, sb.begin + i, 2, L, H, D) for i in range(sb.count)]
        if rank == 1:
            kv[0][0][0, 1, 0, 0] = np.nan
        try:
            sb.commit(desc, [k for k, _ in kv], [v for _, v in kv])
            raise AssertionError("failure not propagated")
        except nk.NomasError as e:
            assert e.code == nk.MsgError.code
        sb.close()
        # Recent mode with SWA eviction: the turn records carry the trim plan,
        # which every rank derives alike (swa.rs:52-95)
        rcfg = orc.Config(storage=orc.INT8, sampling=orc.RECENT, capacity=2 * L + tpf)
        rb = ShardedKvBank(nk.CacheConfig(sampling=nk.HistorySampling.recent(), capacity=2 * L + tpf), n_layers, 1,
                           H, D, 0, bank_factory=lambda b, c: OracleShard(orc, rcfg, b, c, H, D))
        for s in range(4):
            desc = nk._abi.nkv_segment_desc(s, s * frames, frames, frames * tpf, text, -1)
            kv = [_inputs(1, rb.begin + i, s, L, H, D) for i in range(rb.count)]
            rb.commit(desc, [k for k, _ in kv], [v for _, v in kv])
        rec = rb._record(1, nk._abi.nkv_segment_desc(4, 8, frames, frames * tpf, text, -1))
        assert rec[8] > 0  # the trim plan of the next turn is not empty
        assert rb.metrics().evicted_tokens > 0
        rb.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        import traceback
        q.put((rank, f"fail: {e!r}\n{traceback.format_exc()}"))


def _worker_broadcast(rank, world, port, q):
    """The default verification: one broadcast of rank 0's turn record per
    commit / rollback, compared after the local turn; a disagreeing rank
    raises by itself."""
    try:
        for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "hy-nomas-rs_b200")):
            sys.path.insert(0, p)
        import torch.distributed as dist
        from datetime import timedelta
        import nomas_kv as nk
        import oracle as orc
        from nomas_kv.sharded import ShardedKvBank

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        n_layers, H, D, tpf, frames, text = 4, 2, 16, 8, 2, 3
        L = frames * tpf + text
        ocfg = orc.Config(storage=orc.INT8, sampling=orc.UNIFORM, past_frames=3)
        sb = ShardedKvBank(nk.CacheConfig(), n_layers, 1, H, D, 0,
                           bank_factory=lambda b, c: OracleShard(orc, ocfg, b, c, H, D))
        assert sb.verify == "broadcast"

        def kv_of(s):
            kv = [_inputs(0, sb.begin + i, s, L, H, D) for i in range(sb.count)]
            return [k for k, _ in kv], [v for _, v in kv]

        for s in range(3):
            sb.commit(nk._abi.nkv_segment_desc(s, s * frames, frames, frames * tpf, text, -1), *kv_of(s))
        full = orc.Bank(ocfg, n_layers, 1, H, D, orc.F32)
        for s in range(3):
            kv = [_inputs(0, l, s, L, H, D) for l in range(n_layers)]
            full.commit(dict(segment_index=s, frame_start=s * frames, frame_count=frames, image_tokens=frames * tpf,
                             text_tokens=text, action_start=-1), orc.F32, [k for k, _ in kv], [v for _, v in kv])
        assert sb.metrics().as_dict() == full.metrics()
        full.close()
        # a descriptor that differs on rank 1: the turn is applied everywhere,
        # and rank 1 (only) raises CacheState in its next call
        bad = nk._abi.nkv_segment_desc(3, 6, frames, frames * tpf, text, -1 if rank == 0 else 0)
        sb.commit(bad, *kv_of(3))
        try:
            sb.check()
            assert rank == 0, "disagreement not detected"
        except nk.CacheStateError:
            assert rank == 1
        sb.rollback()
        sb.check()  # the rollback's records agree again
        # a non-finite input on rank 1 only: rank 1 raises its own error at
        # once, and the divergence (rank 1 archived nothing) stops rank 1 at
        # the next turn (its own timeline check or the record comparison)
        ks, vs = kv_of(3)
        if rank == 1:
            ks[0][0, 1, 0, 0] = np.nan
        try:
            sb.commit(nk._abi.nkv_segment_desc(3, 6, frames, frames * tpf, text, -1), ks, vs)
            assert rank == 0, "failure not raised"
        except nk.NomasError as e:
            assert rank == 1 and e.code == nk.MsgError.code
        try:
            sb.commit(nk._abi.nkv_segment_desc(4, 8, frames, frames * tpf, text, -1), *kv_of(4))
            sb.check()
            assert rank == 0, "divergence not detected"
        except nk.NomasError:
            assert rank == 1
        sb.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        import traceback
        q.put((rank, f"fail: {e!r}\n{traceback.format_exc()}"))


def _run_two(target):
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg = q.get(timeout=240)
        results[r] = msg
    for p in procs:
        p.join(timeout=60)
    return results


def test_sharded_bank_broadcast_verification_two_gloo_ranks():
    results = _run_two(_worker_broadcast)
    assert results == {0: "ok", 1: "ok"}, results


def test_sharded_bank_two_gloo_ranks():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        r, msg = q.get(timeout=240)
        results[r] = msg
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def test_sharded_bank_without_a_process_group_is_one_rank():
    """Without torch.distributed initialised the sharded bank is the whole
    model on one rank, with no collectives."""
    import nomas_kv as nk
    import oracle as orc
    from nomas_kv.sharded import ShardedKvBank

    n_layers, H, D, tpf, frames, text = 3, 2, 16, 8, 2, 3
    L = frames * tpf + text
    ocfg = orc.Config(storage=orc.INT8, sampling=orc.UNIFORM, past_frames=3)
    sb = ShardedKvBank(nk.CacheConfig(), n_layers, 1, H, D, 0,
                       bank_factory=lambda b, c: OracleShard(orc, ocfg, b, c, H, D))
    assert (sb.rank, sb.world, sb.begin, sb.count) == (0, 1, 0, n_layers)
    full = orc.Bank(ocfg, n_layers, 1, H, D, orc.F32)
    for s in range(3):
        desc = nk._abi.nkv_segment_desc(s, s * frames, frames, frames * tpf, text, -1)
        kv = [_inputs(0, layer, s, L, H, D) for layer in range(n_layers)]
        sb.commit(desc, [k for k, _ in kv], [v for _, v in kv])
        full.commit(dict(segment_index=s, frame_start=s * frames, frame_count=frames, image_tokens=frames * tpf,
                         text_tokens=text, action_start=-1), orc.F32, [k for k, _ in kv], [v for _, v in kv])
    assert sb.metrics().as_dict() == full.metrics()
    assert sb._record(2)[7] == 4  # a rollback would leave 4 frames
    sb.close()
    full.close()


def test_sharded_bank_verify_modes():
    """verify accepts "broadcast" (the default), "strict" and "off", with True
    / False as "strict" / "off"; anything else is refused."""
    import pytest
    import nomas_kv as nk
    import oracle as orc
    from nomas_kv.sharded import ShardedKvBank

    ocfg = orc.Config(storage=orc.INT8, sampling=orc.UNIFORM, past_frames=3)

    def make(**kw):
        return ShardedKvBank(nk.CacheConfig(), 2, 1, 2, 16, 0,
                             bank_factory=lambda b, c: OracleShard(orc, ocfg, b, c, 2, 16), **kw)

    for kw, want in (({}, "broadcast"), ({"verify": True}, "strict"), ({"verify": False}, "off"),
                     ({"verify": "strict"}, "strict"), ({"verify": "off"}, "off")):
        sb = make(**kw)
        assert sb.verify == want
        sb.check()  # nothing pending: a no-op
        sb.close()
    with pytest.raises(ValueError, match="verify"):
        make(verify="sometimes")
