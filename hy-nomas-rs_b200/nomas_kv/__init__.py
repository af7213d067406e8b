"""nomas_kv — Python mirror of hy-nomas-rs's lifelong KV-cache API over the
B200-native C ABI (include/nomas_kv.h).

Names follow the reference crate ``nomas-core`` (``src/cache/``):
``CacheConfig`` / ``QvgConfig`` / ``HistorySampling`` / ``CacheStorage``
(config.rs:55-174), ``SegmentKv`` / ``SegmentLayout`` / ``CacheMetrics``
(cache/mod.rs:61-151), ``KvBank`` (cache/mod.rs:225-320), ``build_cache``
(cache/mod.rs:208-222) and the per-layer ``LifetimeKvCache`` methods
(cache/mod.rs:154-204).  Errors map to the reference's ``Error`` kinds
(error.rs:7-46).  K/V live in torch CUDA tensors; torch supplies device
memory and the stream, every byte of cache work runs in the library's sm_100a
kernels, and there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

from . import _abi
from ._abi import (NKV_BF16, NKV_F16, NKV_F32, NKV_SAMPLING_RECENT, NKV_SAMPLING_RECENT_MIX,
                   NKV_SAMPLING_TEMPORAL, NKV_SAMPLING_UNIFORM, NKV_STORAGE_FLOAT, NKV_STORAGE_INT8,
                   NKV_STORAGE_QVG)

__all__ = [
    "NomasError", "GeometryError", "CacheStateError", "InvalidConfigError", "MsgError", "CudaError", "ArgumentError",
    "HistorySampling", "CacheStorage", "QvgConfig", "CacheConfig", "SegmentKv", "SegmentLayout", "CacheMetrics",
    "KvBank", "LayerCache", "build_cache", "history_frame_indices", "uniform_frame_indices",
    "recent_mix_uniform_frame_indices", "temporal_context_frame_indices", "plan_recent_trim", "partition_layers",
    "lib",
]


# ------------------------------------------------------------------ errors
class NomasError(RuntimeError):
    """Base of the cache errors; ``code`` is the nkv_status value."""

    code = -1

    def __init__(self, msg: str):
        super().__init__(msg)
        self.msg = msg


class GeometryError(NomasError):  # Error::Geometry
    code = _abi.NKV_ERR_GEOMETRY


class CacheStateError(NomasError):  # Error::CacheState
    code = _abi.NKV_ERR_CACHE_STATE


class InvalidConfigError(NomasError):  # Error::InvalidConfig
    code = _abi.NKV_ERR_INVALID_CONFIG


class MsgError(NomasError):  # Error::Msg
    code = _abi.NKV_ERR_MSG


class CudaError(NomasError):
    code = _abi.NKV_ERR_CUDA


class ArgumentError(NomasError):
    code = _abi.NKV_ERR_ARGUMENT


_ERRORS = {c.code: c for c in (GeometryError, CacheStateError, InvalidConfigError, MsgError, CudaError,
                               ArgumentError)}


def lib():
    return _abi.load()


def _check(rc: int):
    if rc != _abi.NKV_OK:
        msg = lib().nkv_last_error().decode()
        raise _ERRORS.get(rc, NomasError)(msg)


# ------------------------------------------------------------------ config
@dataclass(frozen=True)
class HistorySampling:
    """config.rs:55-67: Recent | Uniform | RecentMixUniform | TemporalContext{gamma}."""

    kind: int
    gamma: float = 2.0

    @staticmethod
    def recent() -> "HistorySampling":
        return HistorySampling(NKV_SAMPLING_RECENT)

    @staticmethod
    def uniform() -> "HistorySampling":
        return HistorySampling(NKV_SAMPLING_UNIFORM)

    @staticmethod
    def recent_mix_uniform() -> "HistorySampling":
        return HistorySampling(NKV_SAMPLING_RECENT_MIX)

    @staticmethod
    def temporal_context(gamma: float) -> "HistorySampling":
        return HistorySampling(NKV_SAMPLING_TEMPORAL, float(gamma))

    def __str__(self) -> str:  # config.rs:69-78
        return {NKV_SAMPLING_RECENT: "recent", NKV_SAMPLING_UNIFORM: "uniform",
                NKV_SAMPLING_RECENT_MIX: "recent_mix_uniform"}.get(self.kind, f"temporal_context(gamma={self.gamma})")


@dataclass(frozen=True)
class QvgConfig:
    """config.rs:89-112 with its defaults (config.rs:101-111)."""

    stages: int = 4
    bits_per_stage: int = 2
    block_size: int = 64
    text_as_int8: bool = True
    codebook_seed: int = 0x5EED0002

    def entries(self) -> int:  # qvg.rs:57-59
        return 1 << self.bits_per_stage

    def bytes_per_token(self) -> int:  # qvg.rs:62-64
        return (self.stages * self.bits_per_stage + 7) // 8

    def payload_bytes(self, tokens: int, heads: int) -> int:  # qvg.rs:67-70
        n_blocks = -(-tokens // self.block_size)
        return tokens * heads * self.bytes_per_token() + n_blocks * heads * self.stages * 4


@dataclass(frozen=True)
class CacheStorage:
    """config.rs:116-124: Floating | Int8 | Qvg(QvgConfig)."""

    kind: int
    qvg: QvgConfig = field(default_factory=QvgConfig)

    @staticmethod
    def floating() -> "CacheStorage":
        return CacheStorage(NKV_STORAGE_FLOAT)

    @staticmethod
    def int8() -> "CacheStorage":
        return CacheStorage(NKV_STORAGE_INT8)

    @staticmethod
    def qvg_(cfg: Optional[QvgConfig] = None) -> "CacheStorage":
        return CacheStorage(NKV_STORAGE_QVG, cfg or QvgConfig())


@dataclass
class CacheConfig:
    """config.rs:142-174 (defaults as CacheConfig::default, config.rs:162-174)."""

    storage: CacheStorage = field(default_factory=CacheStorage.floating)
    sampling: HistorySampling = field(default_factory=HistorySampling.recent)
    capacity: Optional[int] = None
    past_frames: int = 64
    phase_swap: bool = False

    def to_c(self) -> _abi.nkv_cache_config:
        q = self.storage.qvg
        return _abi.nkv_cache_config(
            self.storage.kind,
            _abi.nkv_qvg_config(q.stages, q.bits_per_stage, q.block_size, int(q.text_as_int8), q.codebook_seed),
            self.sampling.kind, self.sampling.gamma, int(self.capacity is not None), self.capacity or 0,
            self.past_frames, int(self.phase_swap))


# -------------------------------------------------------------- records
@dataclass
class SegmentKv:
    """cache/mod.rs:100-118: one completed segment's K/V (torch CUDA tensors,
    shape (B, image_tokens + text_tokens, H, D))."""

    segment_index: int
    frame_start: int
    frame_count: int
    image_tokens: int
    text_tokens: int
    action_start: int
    k: object
    v: object

    def __len__(self) -> int:
        return self.image_tokens + self.text_tokens

    def desc(self) -> _abi.nkv_segment_desc:
        return _abi.nkv_segment_desc(self.segment_index, self.frame_start, self.frame_count, self.image_tokens,
                                     self.text_tokens, self.action_start)


@dataclass(frozen=True)
class SegmentLayout:
    """cache/mod.rs:61-97."""

    segment_index: int
    video_start: int
    video_end: int
    text_start: int
    text_end: int
    action_start: int

    def __len__(self) -> int:
        return (self.video_end - self.video_start) + (self.text_end - self.text_start)

    def as_tuple(self):
        return (self.segment_index, self.video_start, self.video_end, self.text_start, self.text_end,
                self.action_start)


@dataclass(frozen=True)
class CacheMetrics:
    """cache/mod.rs:133-151."""

    archived_segments: int = 0
    archived_bytes: int = 0
    encode_calls: int = 0
    d2h_bytes: int = 0
    h2d_bytes: int = 0
    rebuilds: int = 0
    evicted_tokens: int = 0
    rollbacks: int = 0

    @staticmethod
    def from_c(m: _abi.nkv_metrics) -> "CacheMetrics":
        return CacheMetrics(*(int(getattr(m, n)) for n, _ in _abi.nkv_metrics._fields_))

    def as_dict(self) -> dict:
        return dict(self.__dict__)


# ------------------------------------------------------- torch interop
_TORCH_DTYPES = None


def _torch():
    import torch
    return torch


def dtype_code(dtype) -> int:
    torch = _torch()
    m = {torch.float32: NKV_F32, torch.bfloat16: NKV_BF16, torch.float16: NKV_F16}
    if dtype not in m:
        raise GeometryError(f"segment k must be float, got {dtype}")
    return m[dtype]


def torch_dtype(code: int):
    torch = _torch()
    return {NKV_F32: torch.float32, NKV_BF16: torch.bfloat16, NKV_F16: torch.float16}[code]


class _DeviceView:
    """Zero-copy __cuda_array_interface__ view of bank-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2, "strides": None}


def _wrap_device(ptr: int, shape, code: int, device):
    torch = _torch()
    if ptr == 0 or math.prod(shape) == 0:
        return torch.zeros(shape, dtype=torch_dtype(code), device=device)
    typestr = {NKV_F32: "<f4", NKV_F16: "<f2", NKV_BF16: "<i2"}[code]
    t = torch.as_tensor(_DeviceView(ptr, shape, typestr), device=device)
    return t.view(torch.bfloat16) if code == NKV_BF16 else t


# ------------------------------------------------------------------ bank
class LayerCache:
    """One layer of a bank, with the LifetimeKvCache accessors (mod.rs:154-204)."""

    def __init__(self, bank: "KvBank", layer: int):
        self._bank, self._layer = bank, layer

    def storage_format(self) -> CacheStorage:
        return self._bank.cfg.storage

    def sampling(self) -> HistorySampling:
        return self._bank.cfg.sampling

    def working_set(self):
        """(k, v) zero-copy torch views (B, valid_len, H, D) of the model dtype;
        valid until the bank's next commit / rollback / park."""
        b = self._bank
        k, v, n = C.c_void_p(), C.c_void_p(), C.c_uint64()
        _check(lib().nkv_cache_working_set(b._h, self._layer, C.byref(k), C.byref(v), C.byref(n)))
        shape = (b.batch, n.value, b.heads, b.head_dim)
        return (_wrap_device(k.value or 0, shape, b.dtype_code, b.device),
                _wrap_device(v.value or 0, shape, b.dtype_code, b.device))

    def working_layout(self) -> list[SegmentLayout]:
        b = self._bank
        n = C.c_uint64()
        _check(lib().nkv_cache_layout(b._h, self._layer, None, 0, C.byref(n)))
        arr = (_abi.nkv_segment_layout * max(n.value, 1))()
        _check(lib().nkv_cache_layout(b._h, self._layer, arr, n.value, C.byref(n)))
        return [SegmentLayout(a.segment_index, a.video_start, a.video_end, a.text_start, a.text_end, a.action_start)
                for a in arr[: n.value]]

    def _info(self) -> _abi.nkv_cache_info_t:
        out = _abi.nkv_cache_info_t()
        _check(lib().nkv_cache_info(self._bank._h, self._layer, C.byref(out)))
        return out

    def valid_len(self) -> int:
        return int(self._info().valid_len)

    def capacity(self) -> int:
        return int(self._info().capacity)

    def n_segments(self) -> int:
        return int(self._info().n_segments)

    def total_frames(self) -> int:
        return int(self._info().total_frames)

    def tokens_per_frame(self) -> int:
        return int(self._info().tokens_per_frame)

    def is_parked(self) -> bool:
        return bool(self._info().parked)

    def metrics(self) -> CacheMetrics:
        m = _abi.nkv_metrics()
        _check(lib().nkv_cache_metrics(self._bank._h, self._layer, C.byref(m)))
        return CacheMetrics.from_c(m)

    def attend_history(self, q, scale: Optional[float] = None, out=None, lse=None):
        """softmax(q k^T * scale) v over this layer's history, read from the
        INT8 archive (nkv_bank_attend_history).  q: (q_len, H, 128) bf16 on
        the bank's device; returns (out (q_len, H, 128) f32, lse (H, q_len)
        f32).  scale defaults to 1 / sqrt(head_dim), the reference's."""
        torch = _torch()
        b = self._bank
        if q.dim() != 3 or q.shape[1:] != (b.heads, b.head_dim) or q.dtype != torch.bfloat16 or not q.is_contiguous():
            raise GeometryError(f"q must be a contiguous (q_len, {b.heads}, {b.head_dim}) bf16 tensor")
        n = q.shape[0]
        if out is None:
            out = torch.empty((n, b.heads, b.head_dim), dtype=torch.float32, device=q.device)
        if lse is None:
            lse = torch.empty((b.heads, n), dtype=torch.float32, device=q.device)
        for t, shape in ((out, (n, b.heads, b.head_dim)), (lse, (b.heads, n))):
            if tuple(t.shape) != shape or t.dtype != torch.float32 or not t.is_contiguous() or t.device != q.device:
                raise GeometryError(f"out / lse must be contiguous f32 tensors of shape {shape} on {q.device}")
        s = float(scale) if scale is not None else 1.0 / math.sqrt(b.head_dim)
        _check(lib().nkv_bank_attend_history(b._h, self._layer, C.c_void_p(q.data_ptr()), n, s,
                                             C.c_void_p(out.data_ptr()), C.c_void_p(lse.data_ptr())))
        return out, lse

    # QvgCodec::with_codebooks (qvg.rs:101-104) / codebooks readback
    def set_qvg_codebooks(self, cb) -> None:
        import numpy as np
        a = np.ascontiguousarray(cb, dtype=np.float32)
        _check(lib().nkv_cache_set_qvg_codebooks(self._bank._h, self._layer, a.ctypes.data_as(C.c_void_p)))

    def qvg_codebooks(self):
        import numpy as np
        b = self._bank
        q = b.cfg.storage.qvg
        out = np.zeros((2, b.heads, q.stages, q.entries(), b.head_dim), np.float32)
        fitted = C.c_int32()
        _check(lib().nkv_cache_get_qvg_codebooks(b._h, self._layer, out.ctypes.data_as(C.c_void_p),
                                                 C.byref(fitted)))
        return out if fitted.value else None

    def export_segment(self, archive_pos: int) -> bytes:
        """The archived payload of one segment (layout in nomas_kv.h)."""
        import numpy as np
        n = C.c_uint64()
        _check(lib().nkv_cache_export_segment(self._bank._h, self._layer, archive_pos, None, 0, C.byref(n)))
        buf = np.zeros(n.value, np.uint8)
        _check(lib().nkv_cache_export_segment(self._bank._h, self._layer, archive_pos,
                                              buf.ctypes.data_as(C.c_void_p), n.value, C.byref(n)))
        return buf


class KvBank:
    """KvBank (cache/mod.rs:225-320) for layers [layer_begin, layer_begin+n_layers)
    on one CUDA device, driven on torch's current stream of that device."""

    def __init__(self, cfg: CacheConfig, n_layers: int, batch: int, heads: int, head_dim: int, dtype,
                 device=None, layer_begin: int = 0, stream=None):
        torch = _torch()
        self.cfg = cfg
        self.n_layers, self.layer_begin = n_layers, layer_begin
        self.batch, self.heads, self.head_dim = batch, heads, head_dim
        self.dtype_code = dtype if isinstance(dtype, int) else dtype_code(dtype)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if self.device.type != "cuda":
            raise ArgumentError("the cache runs on a CUDA device only (no CPU fallback)")
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        self.stream = stream
        h = C.c_void_p()
        c = cfg.to_c()
        _check(lib().nkv_bank_create(C.byref(c), n_layers, layer_begin, batch, heads, head_dim, self.dtype_code,
                                     self.device.index or 0, C.c_void_p(stream.cuda_stream), C.byref(h)))
        self._h = h

    # -- lifecycle
    def close(self):
        if getattr(self, "_h", None):
            _check(lib().nkv_bank_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return self.n_layers

    def is_empty(self) -> bool:
        return self.n_layers == 0

    def layer(self, i: int) -> LayerCache:
        if not 0 <= i < self.n_layers:
            raise ArgumentError("layer out of range")
        return LayerCache(self, i)

    def as_refs(self) -> list[LayerCache]:
        return [LayerCache(self, i) for i in range(self.n_layers)]

    # -- cache/mod.rs:257-268
    def commit(self, per_layer: Sequence[SegmentKv]) -> None:
        if len(per_layer) != self.n_layers:
            raise MsgError(f"KvBank::commit got {len(per_layer)} segments for {self.n_layers} layers")
        d0 = per_layer[0]
        key = (d0.segment_index, d0.frame_start, d0.frame_count, d0.image_tokens, d0.text_tokens, d0.action_start)
        for s in per_layer[1:]:
            if (s.segment_index, s.frame_start, s.frame_count, s.image_tokens, s.text_tokens, s.action_start) != key:
                raise GeometryError("every layer of a bank commit must carry the same segment geometry")
        ks = [s.k for s in per_layer]
        vs = [s.v for s in per_layer]
        self.commit_tensors(d0.desc(), ks, vs)

    def commit_tensors(self, desc: _abi.nkv_segment_desc, ks, vs, decode_k=None, decode_v=None) -> None:
        """Commit one segment given per-layer K/V tensors (the C-ABI shape).
        With decode_k / decode_v (per-layer tensors of the same shape, model
        dtype) the new segment is also decoded in full into them, by the
        rebuild's gather launch (nkv_bank_commit_decode)."""
        expected = (self.batch, desc.image_tokens + desc.text_tokens, self.heads, self.head_dim)
        dt = None
        for name, ts in (("k", ks), ("v", vs)):
            for t in ts:
                if tuple(t.shape) != expected:
                    raise GeometryError(f"segment {name} shape {list(t.shape)} != {list(expected)}")
                if not t.is_contiguous():
                    raise GeometryError(f"segment {name} must be contiguous")
                code = dtype_code(t.dtype)
                if dt is None:
                    dt = code
                elif code != dt:
                    raise GeometryError("k and v of every layer must share one dtype")
        kp = (C.c_void_p * self.n_layers)(*[t.data_ptr() for t in ks])
        vp = (C.c_void_p * self.n_layers)(*[t.data_ptr() for t in vs])
        if decode_k is None:
            _check(lib().nkv_bank_commit(self._h, C.byref(desc), dt, kp, vp))
            return
        want = torch_dtype(self.dtype_code)
        for name, ts in (("decode_k", decode_k), ("decode_v", decode_v)):
            if ts is None or len(ts) != self.n_layers:
                raise ArgumentError(f"{name} needs one tensor per layer")
            for t in ts:
                if tuple(t.shape) != expected or t.dtype != want or not t.is_contiguous():
                    raise GeometryError(f"{name} tensors must be contiguous {list(expected)} {want}")
        dkp = (C.c_void_p * self.n_layers)(*[t.data_ptr() for t in decode_k])
        dvp = (C.c_void_p * self.n_layers)(*[t.data_ptr() for t in decode_v])
        _check(lib().nkv_bank_commit_decode(self._h, C.byref(desc), dt, kp, vp, dkp, dvp))

    def commit_ptrs(self, desc: _abi.nkv_segment_desc, kv_dtype: int, k_ptrs, v_ptrs) -> None:
        kp = (C.c_void_p * self.n_layers)(*k_ptrs)
        vp = (C.c_void_p * self.n_layers)(*v_ptrs)
        _check(lib().nkv_bank_commit(self._h, C.byref(desc), kv_dtype, kp, vp))

    def rollback(self) -> None:  # cache/mod.rs:276-281
        _check(lib().nkv_bank_rollback(self._h))

    def park_all(self) -> None:  # cache/mod.rs:284-289
        _check(lib().nkv_bank_park(self._h))

    def unpark_all(self) -> None:  # cache/mod.rs:292-297
        _check(lib().nkv_bank_unpark(self._h))

    def metrics(self) -> CacheMetrics:  # cache/mod.rs:305-319
        m = _abi.nkv_metrics()
        _check(lib().nkv_bank_metrics(self._h, C.byref(m)))
        return CacheMetrics.from_c(m)

    def synchronize(self) -> None:
        _check(lib().nkv_bank_synchronize(self._h))

    def reserve(self, archive_bytes: int, working_tokens: int = 0) -> None:
        _check(lib().nkv_bank_reserve(self._h, archive_bytes, working_tokens))

    def set_archive_device_limit(self, device_bytes: int) -> None:
        """Archive chunks allocated from now on go to pinned, device-mapped
        host memory once the device chunks reach `device_bytes` (0: no limit)."""
        _check(lib().nkv_bank_set_archive_device_limit(self._h, int(device_bytes)))

    def archive_usage(self) -> tuple[int, int]:
        """(device bytes, host bytes) of the archived slabs."""
        d, h = C.c_uint64(), C.c_uint64()
        _check(lib().nkv_bank_archive_usage(self._h, C.byref(d), C.byref(h)))
        return int(d.value), int(h.value)

    def segment_bytes(self, desc: _abi.nkv_segment_desc) -> int:
        n = C.c_uint64()
        _check(lib().nkv_bank_segment_bytes(self._h, C.byref(desc), C.byref(n)))
        return int(n.value)

    def decode_segment(self, archive_pos: int, k_out, v_out) -> None:
        """history.rs:308-338 for every local layer into caller tensors."""
        kp = (C.c_void_p * self.n_layers)(*[t.data_ptr() for t in k_out])
        vp = (C.c_void_p * self.n_layers)(*[t.data_ptr() for t in v_out])
        _check(lib().nkv_bank_decode_segment(self._h, archive_pos, kp, vp))

    def set_timing(self, on: bool) -> None:
        _check(lib().nkv_bank_set_timing(self._h, int(on)))

    # -- archive persistence (no counterpart in the reference)
    def save(self, path) -> None:
        """Write the archive, timeline, counters and QVG codebooks to `path`."""
        _check(lib().nkv_bank_save(self._h, str(path).encode()))

    def load(self, path) -> None:
        """Restore a saved archive into this fresh bank and rebuild the working set."""
        _check(lib().nkv_bank_load(self._h, str(path).encode()))

    # -- two-phase INT8 commit for a producer that writes the archive rows
    def stage_segment(self, desc: _abi.nkv_segment_desc) -> list[dict]:
        """Validate `desc` and reserve its INT8 record; per local layer the
        device addresses of k_codes / v_codes (B, L, H, D) u8, k_scales /
        v_scales (B, L, H) f32 and the layer's status word."""
        arr = (_abi.nkv_staged_layer * self.n_layers)()
        _check(lib().nkv_bank_stage_segment(self._h, C.byref(desc), arr))
        return [{f: int(getattr(a, f) or 0) for f, _ in _abi.nkv_staged_layer._fields_} for a in arr]

    def commit_staged(self) -> None:
        _check(lib().nkv_bank_commit_staged(self._h))

    def discard_staged(self) -> None:
        _check(lib().nkv_bank_discard_staged(self._h))

    def commit_projected(self, desc: _abi.nkv_segment_desc, xs, weights, rope=None, k_outs=None, v_outs=None,
                         qk_norm: bool = True, eps: float = 1e-6) -> None:
        """Commit a segment whose K / V are the projections of xs[i] (layer
        i's (L, H*D) bf16 attention input) by weights[i] = dict(wk, wv, bk,
        bv, k_gain): nkv_kv_project writes the archive rows (and the bf16
        K / V into k_outs / v_outs when given), then the staged commit
        archives and rebuilds.  Batch 1, head_dim 128."""
        staged = self.stage_segment(desc)
        L = desc.image_tokens + desc.text_tokens
        try:
            for i in range(self.n_layers):
                w = weights[i]
                kv_project(xs[i], w["wk"], w["wv"], bk=w.get("bk"), bv=w.get("bv"), k_gain=w.get("k_gain"),
                           qk_norm=qk_norm, eps=eps, rope=rope,
                           k_out=None if k_outs is None else k_outs[i], v_out=None if v_outs is None else v_outs[i],
                           codes=staged[i], ranges=[(0, L, 0)], status_ptr=staged[i]["status"],
                           stream=self.stream)
        except Exception:
            self.discard_staged()
            raise
        self.commit_staged()

    def kernel_stats(self, reset: bool = False) -> dict:
        arr = (_abi.nkv_kernel_stat * _abi.NKV_KERNEL_COUNT)()
        _check(lib().nkv_bank_kernel_stats(self._h, arr, int(reset)))
        return {n: (int(arr[i].launches), float(arr[i].total_ms)) for i, n in enumerate(_abi.KERNEL_NAMES)}


def kv_project(x, wk, wv, bk=None, bv=None, k_gain=None, qk_norm: bool = True, eps: float = 1e-6, rope=None,
               k_out=None, v_out=None, codes=None, ranges=None, status=None, status_ptr: int = 0, stream=None):
    """nkv_kv_project on torch tensors (one layer, batch 1): the captured
    K / V of modules/attention.rs:107-124, 143-144 with the INT8 archive rows
    of the committed ranges.  x (tokens, H*128) bf16; wk / wv (H*128, H*128)
    bf16; bk / bv / k_gain bf16 or None; rope = (cos, sin) f32 (tokens, 64)
    or None; k_out / v_out bf16 (tokens, H*128) or None; codes = dict with
    k_codes / v_codes / k_scales / v_scales (tensors or device addresses) or
    None; ranges = [(lo, hi, dst), ...]; status = a 1-element int32/uint32
    device tensor (or status_ptr an address) that receives the non-finite
    bits."""
    torch = _torch()
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise ArgumentError("x must be a (tokens, H*128) bf16 tensor")
    tokens, dim = x.shape
    addr = lambda t: 0 if t is None else (t if isinstance(t, int) else t.data_ptr())  # noqa: E731
    for name, t in (("x", x), ("wk", wk), ("wv", wv), ("bk", bk), ("bv", bv), ("k_gain", k_gain),
                    ("k_out", k_out), ("v_out", v_out)):
        if t is not None and not isinstance(t, int):
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != x.device:
                raise ArgumentError(f"{name} must be a contiguous bf16 tensor on {x.device}")
    if wk.shape != (dim, dim) or wv.shape != (dim, dim):
        raise GeometryError(f"weights must be ({dim}, {dim})")
    a = _abi.nkv_kv_project_args()
    a.tokens, a.heads, a.head_dim = tokens, dim // 128, 128
    a.x, a.wk, a.wv, a.bk, a.bv = addr(x), addr(wk), addr(wv), addr(bk), addr(bv)
    a.qk_norm, a.eps, a.k_norm_gain = int(bool(qk_norm)), float(eps), addr(k_gain)
    if rope is not None:
        cos, sin = rope
        for t in (cos, sin):
            if t.dtype != torch.float32 or tuple(t.shape) != (tokens, 64) or not t.is_contiguous():
                raise GeometryError("rope tables must be contiguous f32 (tokens, 64)")
        a.rope_cos, a.rope_sin = addr(cos), addr(sin)
    a.k_out, a.v_out = addr(k_out), addr(v_out)
    if codes is not None:
        a.k_codes, a.k_scales = addr(codes["k_codes"]), addr(codes["k_scales"])
        a.v_codes, a.v_scales = addr(codes["v_codes"]), addr(codes["v_scales"])
        rs = list(ranges) if ranges is not None else [(0, tokens, 0)]
        if len(rs) > 2:
            raise ArgumentError("at most two row ranges")
        a.n_ranges = len(rs)
        for i, (lo, hi, dst) in enumerate(rs):
            a.ranges[i].lo, a.ranges[i].hi, a.ranges[i].dst = lo, hi, dst
    a.status = status_ptr if status is None else status.data_ptr()
    if stream is None:
        stream = torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        _check(lib().nkv_kv_project(C.byref(a), C.c_void_p(stream.cuda_stream)))


def build_cache(cfg: CacheConfig, batch: int, heads: int, head_dim: int, dtype, device=None) -> KvBank:
    """cache/mod.rs:208-222: a single-layer cache (phase swap per cfg)."""
    return KvBank(cfg, 1, batch, heads, head_dim, dtype, device)


# ------------------------------------------------------ host policy
def _indices(kind: int, total: int, past: int, sampling: int = NKV_SAMPLING_UNIFORM, gamma: float = 2.0):
    import numpy as np
    n = C.c_uint64()
    _check(lib().nkv_frame_indices(kind, total, past, sampling, gamma, None, 0, C.byref(n)))
    out = np.zeros(max(n.value, 1), np.uint64)
    _check(lib().nkv_frame_indices(kind, total, past, sampling, gamma, out.ctypes.data_as(C.c_void_p), n.value,
                                   C.byref(n)))
    return [int(x) for x in out[: n.value]]


def uniform_frame_indices(total: int, past: int):  # uniform_history.rs:10-19
    return _indices(0, total, past)


def recent_mix_uniform_frame_indices(total: int, past: int):  # uniform_history.rs:23-32
    return _indices(1, total, past)


def temporal_context_frame_indices(total: int, past: int, gamma: float):  # uniform_history.rs:40-70
    return _indices(2, total, past, NKV_SAMPLING_TEMPORAL, gamma)


def history_frame_indices(total: int, past: int, sampling: HistorySampling):  # uniform_history.rs:76-125
    return _indices(3, total, past, sampling.kind, sampling.gamma)


def plan_recent_trim(records, capacity: int, tokens_per_frame: int):
    """swa.rs:52-130: returns (drop_frames, drop_records, evicted_tokens, kept)."""
    import numpy as np
    n = len(records)
    recs = np.ascontiguousarray(np.array(records, np.uint64).reshape(n, 5) if n else np.zeros((0, 5), np.uint64))
    df = np.zeros(2 * n + 2, np.uint64)
    dr = np.zeros(n + 1, np.uint64)
    kept = np.zeros(5 * n + 5, np.uint64)
    ndf, ndr, ev, nk = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    _check(lib().nkv_plan_recent_trim(p(recs), n, capacity, tokens_per_frame, p(df), C.byref(ndf), p(dr),
                                      C.byref(ndr), C.byref(ev), p(kept), C.byref(nk)))
    return ([(int(df[2 * i]), int(df[2 * i + 1])) for i in range(ndf.value)],
            [int(dr[i]) for i in range(ndr.value)], int(ev.value),
            [tuple(int(x) for x in kept[5 * i: 5 * i + 5]) for i in range(nk.value)])


def partition_layers(n_layers: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous layer block (begin, count) of `rank` when `n_layers` caches
    are sharded over `world` GPUs; the first n_layers % world ranks take one
    extra layer."""
    if world < 1 or not 0 <= rank < world:
        raise ArgumentError("bad rank/world")
    base, extra = divmod(n_layers, world)
    count = base + (1 if rank < extra else 0)
    begin = rank * base + min(rank, extra)
    return begin, count
