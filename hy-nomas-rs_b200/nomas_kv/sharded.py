"""Layer-sharded KvBank across the GPUs of one node (one process per GPU).

The reference's KvBank fans every commit / rollback / park out to one
independent cache per DiT layer (cache/mod.rs:257-297).  Sharding therefore
needs no data exchange: rank r owns the contiguous layer block
``partition_layers(n_layers, world, r)`` and every archive, working set and
codebook of those layers stays in that GPU's HBM.  The only cross-rank
traffic is host metadata:

* ``verify=True`` checks that every rank commits the same segment
  descriptor (one all_gather of six integers per commit; off on the hot path
  of the benchmark, where each rank derives the descriptor itself);
* a failed operation on any rank is reported on every rank (all_reduce MAX
  of the status), so ranks never silently diverge in what they report;
* ``metrics()`` reproduces KvBank::metrics (cache/mod.rs:305-319) over all
  layers of the model: MAX of archived_segments / rebuilds / evicted_tokens /
  rollbacks, SUM of the byte and encode counters.

Works with any torch.distributed backend (NCCL on the GPUs, gloo in the CPU
tests).  ``bank_factory(begin, count)`` builds the local bank; by default a
KvBank on the current CUDA device.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import (CacheConfig, CacheMetrics, CacheStateError, KvBank, NomasError, _ERRORS, partition_layers)
from . import _abi

_MAX_FIELDS = ("archived_segments", "rebuilds", "evicted_tokens", "rollbacks")
_SUM_FIELDS = ("archived_bytes", "encode_calls", "d2h_bytes", "h2d_bytes")


class ShardedKvBank:
    def __init__(self, cfg: CacheConfig, n_layers: int, batch: int, heads: int, head_dim: int, dtype,
                 group=None, bank_factory: Optional[Callable[[int, int], object]] = None, verify: bool = True,
                 device: Optional[torch.device] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.n_layers = n_layers
        self.begin, self.count = partition_layers(n_layers, self.world, self.rank)
        self.verify = verify
        backend = dist.get_backend(group)
        self.comm_device = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" \
            else torch.device("cpu")
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

    def _agree(self, desc) -> None:
        mine = torch.tensor([desc.segment_index, desc.frame_start, desc.frame_count, desc.image_tokens,
                             desc.text_tokens, desc.action_start], dtype=torch.int64, device=self.comm_device)
        allv = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(allv, mine, group=self.group)
        if any(not torch.equal(allv[0], a) for a in allv[1:]):
            raise CacheStateError("ranks disagree on the committed segment descriptor")

    def _collective_status(self, fn) -> None:
        """Run fn locally, then make every rank raise if any rank failed."""
        err: Optional[NomasError] = None
        try:
            fn()
        except NomasError as e:
            err = e
        code = torch.tensor([err.code if err is not None else 0], dtype=torch.int64, device=self.comm_device)
        dist.all_reduce(code, op=dist.ReduceOp.MAX, group=self.group)
        c = int(code.item())
        if err is not None:
            raise err
        if c != 0:
            raise _ERRORS.get(c, NomasError)(f"operation failed on another rank (status {c})")

    # ------------------------------------------------------------ API
    def commit(self, desc: _abi.nkv_segment_desc, ks, vs) -> None:
        """Commit one segment: ks / vs are this rank's layers' K / V."""
        if self.verify:
            self._agree(desc)
        self._collective_status(lambda: self.local.commit_tensors(desc, ks, vs))

    def rollback(self) -> None:
        self._collective_status(self.local.rollback)

    def park_all(self) -> None:
        self._collective_status(self.local.park_all)

    def unpark_all(self) -> None:
        self._collective_status(self.local.unpark_all)

    def metrics(self) -> CacheMetrics:
        m = self.local.metrics()
        d = m.as_dict() if isinstance(m, CacheMetrics) else dict(m)
        mx = torch.tensor([d[f] for f in _MAX_FIELDS], dtype=torch.int64, device=self.comm_device)
        sm = torch.tensor([d[f] for f in _SUM_FIELDS], dtype=torch.int64, device=self.comm_device)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=self.group)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM, group=self.group)
        out = {f: int(v) for f, v in zip(_MAX_FIELDS, mx.tolist())}
        out.update({f: int(v) for f, v in zip(_SUM_FIELDS, sm.tolist())})
        return CacheMetrics(**out)

    def close(self) -> None:
        if hasattr(self.local, "close"):
            self.local.close()
