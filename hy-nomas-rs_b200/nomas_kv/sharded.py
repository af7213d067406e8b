"""Layer-sharded KvBank across the GPUs of one node (one process per GPU).

The reference's KvBank fans every commit / rollback / park out to one
independent cache per DiT layer (cache/mod.rs:257-297).  Sharding therefore
needs no data exchange: rank r owns the contiguous layer block
``partition_layers(n_layers, world, r)`` and every archive, working set and
codebook of those layers stays in that GPU's HBM.  The only cross-rank
traffic is host metadata, at most 1 KB per turn.  The turn record of a
commit or rollback is rank 0's operation, segment descriptor, timeline
length after the turn, and the frames the history sampler picks then, or the
Recent-mode trim plan (cache/uniform_history.rs:76-125, cache/swa.rs:52-95);
every rank evaluates the same samplers on its own state and compares.

* ``verify="broadcast"`` (default): rank 0's record is broadcast on the
  communication stream while the local commit runs, and compared in the
  rank's next call (the next turn, park, unpark, metrics, ``check()`` or
  close): one collective per turn, off the cache's stream, never waited for
  inside the turn that posted it, so the ranks keep a turn of slack instead
  of meeting at every turn's end.  A rank whose record of a turn differs
  raises CacheState in its next call (its bank applied the turn); a rank
  whose own operation fails raises its own error at once, and the
  divergence stops it at the next turn (its own timeline check, or the
  record comparison);
* ``verify="strict"``: the records are compared before anything is touched,
  one all-reduce of the comparisons lets every rank take the same decision
  (when any rank disagrees no bank is touched and every rank raises
  CacheState), and every rank's outcome is all-reduced (MAX of the status
  code), so when one rank fails every rank raises.  Three collectives per
  turn, each waited for on the host;
* ``verify="off"``: no collectives.
* ``metrics()`` reproduces KvBank::metrics (cache/mod.rs:305-319) over all
  layers of the model: MAX of archived_segments / rebuilds / evicted_tokens /
  rollbacks, SUM of the byte and encode counters.

On NCCL the per-turn collectives run on a dedicated high-priority stream
that does not wait for the cache's stream, so they overlap the rebuild
gather the commit left running instead of waiting for it to drain.  Works with any torch.distributed
backend (NCCL on the GPUs, gloo in the CPU tests), and without an
initialised process group as a single-rank bank (no collectives).
``bank_factory(begin, count)`` builds the local bank; by default a KvBank
on the current CUDA device.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import (NKV_SAMPLING_RECENT, CacheConfig, CacheMetrics, CacheStateError, KvBank, NomasError, _ERRORS,
               history_frame_indices, partition_layers, plan_recent_trim)
from . import _abi

_MAX_FIELDS = ("archived_segments", "rebuilds", "evicted_tokens", "rollbacks")
_SUM_FIELDS = ("archived_bytes", "encode_calls", "d2h_bytes", "h2d_bytes")

RECORD_WORDS = 128  # int64 words: 1 KB per turn
_HEADER = 16  # op, 6 descriptor fields, frames after the turn, n items, FNV-1a of the items, ...
OP_COMMIT, OP_ROLLBACK = 1, 2
_FNV_OFFSET, _FNV_PRIME, _M64 = 0xCBF29CE484222325, 0x100000001B3, (1 << 64) - 1


def _fnv1a(values) -> int:
    h = _FNV_OFFSET
    for v in values:
        h = ((h ^ (int(v) & _M64)) * _FNV_PRIME) & _M64
    return h - (1 << 64) if h >= (1 << 63) else h  # as a signed int64


class ShardedKvBank:
    def __init__(self, cfg: CacheConfig, n_layers: int, batch: int, heads: int, head_dim: int, dtype,
                 group=None, bank_factory: Optional[Callable[[int, int], object]] = None, verify="broadcast",
                 device: Optional[torch.device] = None):
        self.cfg = cfg
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.n_layers = n_layers
        self.begin, self.count = partition_layers(n_layers, self.world, self.rank)
        if verify is True:
            verify = "strict"
        elif verify is False or verify is None:
            verify = "off"
        if verify not in ("broadcast", "strict", "off"):
            raise ValueError(f"verify must be 'broadcast', 'strict' or 'off', not {verify!r}")
        self.verify = verify
        nccl = self.distributed and dist.get_backend(group) == "nccl"
        self.comm_device = torch.device("cuda", torch.cuda.current_device()) if nccl else torch.device("cpu")
        # strict mode waits for its collectives inside the turn: high priority
        # schedules their kernels ahead of the rebuild gather's pending CTAs.
        # Broadcast mode checks a turn later, so its kernel runs at normal
        # priority in the gaps of the cache's stream and never holds back the
        # gather's CTAs while it waits for the other ranks
        self.comm_stream = torch.cuda.Stream(self.comm_device, priority=-1 if verify == "strict" else 0) \
            if nccl else None
        pin = nccl
        self._rec_host = torch.zeros(RECORD_WORDS, dtype=torch.int64, pin_memory=pin)
        # broadcast mode: two slots, so turn t + 1 posts while turn t's
        # broadcast is still unchecked
        self._bc_in = [torch.zeros(RECORD_WORDS, dtype=torch.int64, pin_memory=pin) for _ in range(2)]
        self._bc_out = [torch.zeros(RECORD_WORDS, dtype=torch.int64, pin_memory=pin) for _ in range(2)]
        self._bc_dev = [torch.zeros(RECORD_WORDS, dtype=torch.int64, device=self.comm_device) for _ in range(2)]
        self._bc_ev = [torch.cuda.Event(blocking=True) for _ in range(2)] if nccl else [None, None]
        self._bc_slot = 0
        self._bc_pending: Optional[tuple[int, list[int]]] = None  # (slot, this rank's record)
        self._rec_dev = torch.zeros(RECORD_WORDS, dtype=torch.int64, device=self.comm_device)
        self._st_host = torch.zeros(1, dtype=torch.int64, pin_memory=pin)
        self._st_dev = torch.zeros(1, dtype=torch.int64, device=self.comm_device)
        # the descriptors this bank holds, oldest first: the Recent-mode trim
        # plan of the next turn needs them (swa.rs:52-95)
        self._records: list[tuple[int, int, int, int, int]] = []
        self._total_frames = 0
        self._tpf = 0
        if bank_factory is None:
            bank_factory = lambda begin, count: KvBank(cfg, count, batch, heads, head_dim, dtype,  # noqa: E731
                                                       device=device, layer_begin=begin)
        self.local = bank_factory(self.begin, self.count)

    # ------------------------------------------------------------ helpers
    def owns(self, layer: int) -> bool:
        return self.begin <= layer < self.begin + self.count

    def local_index(self, layer: int) -> int:
        if not self.owns(layer):
            raise CacheStateError(f"layer {layer} lives on another rank")
        return layer - self.begin

    def _sampled(self, records, total_frames: int, tpf: int) -> list[int]:
        """What the history sampler selects after a turn: the frame ids, or
        for Recent mode the trim plan (evicted tokens, dropped records, then
        (record, frames) pairs of dropped head frames)."""
        if not records:
            return []
        s = self.cfg.sampling
        if s.kind == NKV_SAMPLING_RECENT:
            cap = self.cfg.capacity if self.cfg.capacity is not None else (1 << 63) - 1
            drop_frames, drop_records, evicted, _ = plan_recent_trim(list(records), cap, max(tpf, 1))
            out = [evicted, len(drop_records), *drop_records]
            for r, f in drop_frames:
                out += [r, f]
            return out
        return history_frame_indices(total_frames, self.cfg.past_frames, s)

    def _record(self, op: int, desc=None) -> list[int]:
        """This rank's record of the next turn, from its own state."""
        records, total, tpf = list(self._records), self._total_frames, self._tpf
        d = [0] * 6
        if op == OP_COMMIT:
            d = [desc.segment_index, desc.frame_start, desc.frame_count, desc.image_tokens, desc.text_tokens,
                 desc.action_start]
            if desc.frame_count > 0 and tpf == 0:
                tpf = desc.image_tokens // desc.frame_count
            records.append((desc.segment_index, desc.frame_start, desc.frame_count, desc.image_tokens,
                            desc.text_tokens))
            total += desc.frame_count
        elif records:
            total -= records.pop()[2]
        items = self._sampled(records, total, tpf)
        head = [op, *d, total, len(items), _fnv1a(items)]
        body = items[: RECORD_WORDS - _HEADER]
        rec = head + [0] * (_HEADER - len(head)) + body
        return rec + [0] * (RECORD_WORDS - len(rec))

    def _collective(self, fn):
        if self.comm_stream is None:
            return fn()
        with torch.cuda.stream(self.comm_stream):
            return fn()

    def _check_record(self, mine: list[int]) -> bool:
        """Broadcast rank 0's turn record; True when this rank's equals it."""
        def run():
            self._rec_host.copy_(torch.tensor(mine, dtype=torch.int64))
            self._rec_dev.copy_(self._rec_host, non_blocking=True)
            dist.broadcast(self._rec_dev, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                           group=self.group)
            self._rec_host.copy_(self._rec_dev, non_blocking=True)
            if self.comm_stream is not None:
                self.comm_stream.synchronize()
            return self._rec_host.tolist() == mine
        return self._collective(run)

    def _post_record(self, mine: list[int]) -> None:
        """Enqueue the broadcast of rank 0's turn record into the next slot (no
        host wait on NCCL); the comparison is left pending."""
        k = self._bc_slot
        self._bc_slot ^= 1

        def run():
            self._bc_in[k].copy_(torch.tensor(mine, dtype=torch.int64))
            buf = self._bc_in[k]
            if self.comm_stream is not None:
                self._bc_dev[k].copy_(self._bc_in[k], non_blocking=True)
                buf = self._bc_dev[k]
            dist.broadcast(buf, src=dist.get_global_rank(self.group, 0) if self.group else 0, group=self.group)
            if self.comm_stream is not None:
                self._bc_out[k].copy_(self._bc_dev[k], non_blocking=True)
                self._bc_ev[k].record(self.comm_stream)
            else:
                self._bc_out[k].copy_(self._bc_in[k])
        self._collective(run)
        self._bc_pending = (k, mine)

    def check(self) -> None:
        """Compare the pending turn record with rank 0's (broadcast mode);
        raises CacheState when they differ.  Every call of the bank does this
        first; call it after the last turn to check that one."""
        pending, self._bc_pending = self._bc_pending, None
        self._check_one(pending)

    def _check_one(self, pending) -> None:
        if pending is None:
            return
        k, mine = pending
        if self._bc_ev[k] is not None:
            self._bc_ev[k].synchronize()
        if self._bc_out[k].tolist() != mine:
            raise CacheStateError("this rank's record of the last turn (segment descriptor or sampled history) "
                                  "differs from rank 0's")

    def _any(self, flag: int) -> int:
        return self._status(flag)

    def _status(self, code: int) -> int:
        def run():
            self._st_host[0] = code
            self._st_dev.copy_(self._st_host, non_blocking=True)
            dist.all_reduce(self._st_dev, op=dist.ReduceOp.MAX, group=self.group)
            self._st_host.copy_(self._st_dev, non_blocking=True)
            if self.comm_stream is not None:
                self.comm_stream.synchronize()
            return int(self._st_host[0])
        return self._collective(run)

    def _turn(self, op: int, fn, desc=None) -> None:
        """Check the turn record, run fn locally, make every rank raise if any
        rank failed."""
        err: Optional[NomasError] = None
        if self.world > 1 and self.verify == "broadcast":
            if op in (OP_COMMIT, OP_ROLLBACK):
                # post this turn's broadcast first, so every rank's sequence of
                # collectives stays the same even when the check below raises
                prev, self._bc_pending = self._bc_pending, None
                self._post_record(self._record(op, desc))
                self._check_one(prev)  # the previous turn's record
            else:
                self.check()
            fn()
            return
        if self.world > 1 and self.verify == "strict" and op in (OP_COMMIT, OP_ROLLBACK):
            same = self._check_record(self._record(op, desc))
            if self._any(0 if same else 1) != 0:
                raise CacheStateError("ranks disagree on the turn record (segment descriptor or sampled history)")
        if err is None:
            try:
                fn()
            except NomasError as e:
                err = e
        code = err.code if err is not None else 0
        c = self._status(code) if self.world > 1 and self.verify == "strict" else code
        if err is None and c == 0:
            return
        if err is not None:
            raise err
        raise _ERRORS.get(c, NomasError)(f"operation failed on another rank (status {c})")

    # ------------------------------------------------------------ API
    def commit(self, desc: _abi.nkv_segment_desc, ks, vs, decode_k=None, decode_v=None) -> None:
        """Commit one segment: ks / vs are this rank's layers' K / V; with
        decode_k / decode_v the new segment is also decoded into them."""
        def run():
            try:
                if decode_k is None:
                    self.local.commit_tensors(desc, ks, vs)
                else:
                    self.local.commit_tensors(desc, ks, vs, decode_k, decode_v)
            except NomasError as e:
                # a rebuild over capacity still archived the segment (history.rs:416-421)
                if not (e.code == _abi.NKV_ERR_GEOMETRY and "capacity" in e.msg):
                    raise
                self._archived(desc)
                raise
            self._archived(desc)
        self._turn(OP_COMMIT, run, desc)

    def _archived(self, desc) -> None:
        self._records.append((desc.segment_index, desc.frame_start, desc.frame_count, desc.image_tokens,
                              desc.text_tokens))
        self._total_frames += desc.frame_count
        if self._tpf == 0 and desc.frame_count > 0:
            self._tpf = desc.image_tokens // desc.frame_count

    def rollback(self) -> None:
        def run():
            self.local.rollback()
            if self._records:
                self._total_frames -= self._records.pop()[2]
        self._turn(OP_ROLLBACK, run)

    def park_all(self) -> None:
        self._turn(0, self.local.park_all)

    def unpark_all(self) -> None:
        self._turn(0, self.local.unpark_all)

    def metrics(self) -> CacheMetrics:
        if self.world > 1 and self.verify == "broadcast":
            self.check()
        m = self.local.metrics()
        d = m.as_dict() if isinstance(m, CacheMetrics) else dict(m)
        if self.world == 1:
            return CacheMetrics(**d)
        mx = torch.tensor([d[f] for f in _MAX_FIELDS], dtype=torch.int64, device=self.comm_device)
        sm = torch.tensor([d[f] for f in _SUM_FIELDS], dtype=torch.int64, device=self.comm_device)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=self.group)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM, group=self.group)
        out = {f: int(v) for f, v in zip(_MAX_FIELDS, mx.tolist())}
        out.update({f: int(v) for f, v in zip(_SUM_FIELDS, sm.tolist())})
        return CacheMetrics(**out)

    def close(self) -> None:
        pending = self._bc_pending
        self._bc_pending = None
        if pending is not None and self._bc_ev[pending[0]] is not None:
            self._bc_ev[pending[0]].synchronize()  # the broadcast's buffers outlive it
        if hasattr(self.local, "close"):
            self.local.close()
