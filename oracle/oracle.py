"""ctypes wrapper of the CPU oracle (``oracle/_build/libnomas_oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by ``__graft_entry__.smoke()``
as the checker of one GPU call, and by ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` arm.  The product (``hy-nomas-rs_b200/``) never imports it.

The oracle restates the reference's cache path (nomas-core ``cache/*.rs``); see
the header of ``nomas_oracle.cpp`` for the assumed candle/half semantics and the
parity status (samplers and trim plans pinned by the reference's KATs; INT8/QVG
bytes pinned only through the reference's invariant tests).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libnomas_oracle.so")

F32, BF16, F16 = 0, 1, 2
FLOATING, INT8, QVG = 0, 1, 2
RECENT, UNIFORM, RECENT_MIX, TEMPORAL = 0, 1, 2, 3

OK, ERR_GEOMETRY, ERR_CACHE_STATE, ERR_INVALID_CONFIG, ERR_MSG, ERR_ARGUMENT = 0, 1, 2, 3, 4, 6


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class OrcConfig(C.Structure):
    _fields_ = [
        ("storage", C.c_int32),
        ("qvg_stages", C.c_int32),
        ("qvg_bits", C.c_int32),
        ("qvg_block", C.c_int32),
        ("qvg_text_as_int8", C.c_int32),
        ("qvg_seed", C.c_uint64),
        ("sampling", C.c_int32),
        ("gamma", C.c_double),
        ("has_capacity", C.c_int32),
        ("capacity", C.c_uint64),
        ("past_frames", C.c_uint64),
        ("phase_swap", C.c_int32),
    ]


class OrcSegment(C.Structure):
    _fields_ = [
        ("segment_index", C.c_uint64),
        ("frame_start", C.c_uint64),
        ("frame_count", C.c_uint64),
        ("image_tokens", C.c_uint64),
        ("text_tokens", C.c_uint64),
        ("action_start", C.c_int64),
    ]


class OrcLayout(C.Structure):
    _fields_ = [
        ("segment_index", C.c_uint64),
        ("video_start", C.c_uint64),
        ("video_end", C.c_uint64),
        ("text_start", C.c_uint64),
        ("text_end", C.c_uint64),
        ("action_start", C.c_int64),
    ]


class OrcMetrics(C.Structure):
    _fields_ = [
        (n, C.c_uint64)
        for n in (
            "archived_segments",
            "archived_bytes",
            "encode_calls",
            "d2h_bytes",
            "h2d_bytes",
            "rebuilds",
            "evicted_tokens",
            "rollbacks",
        )
    ]

    def as_dict(self) -> dict:
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _lib.orc_last_error.restype = C.c_char_p
        _lib.orc_splitmix_next.restype = C.c_uint64
        _lib.orc_unpack_bits.restype = C.c_uint64
        _lib.orc_qvg_payload_bytes.restype = C.c_uint64
        _lib.orc_bf16_bits.restype = C.c_uint16
        _lib.orc_bf16_bits.argtypes = [C.c_float]
        _lib.orc_f16_bits.restype = C.c_uint16
        _lib.orc_f16_bits.argtypes = [C.c_float]
        _lib.orc_randn.argtypes = [C.c_uint64, C.c_uint64, C.c_double, C.c_double, C.c_void_p]
        _lib.orc_frame_indices.argtypes = [
            C.c_int32, C.c_uint64, C.c_uint64, C.c_int32, C.c_double, C.c_void_p, C.c_uint64, C.c_void_p]
        _lib.orc_bank_create.argtypes = [
            C.POINTER(OrcConfig), C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_int32, C.POINTER(C.c_void_p)]
        _lib.orc_bank_destroy.argtypes = [C.c_void_p]
        _lib.orc_set_threads.argtypes = [C.c_int32]
        _lib.orc_bank_commit.argtypes = [
            C.c_void_p, C.POINTER(OrcSegment), C.c_int32, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int32]
        for name in ("orc_bank_rollback", "orc_bank_park", "orc_bank_unpark"):
            getattr(_lib, name).argtypes = [C.c_void_p]
        _lib.orc_bank_prefill_clone.argtypes = [C.c_void_p, C.c_uint64]
        _lib.orc_bank_metrics.argtypes = [C.c_void_p, C.POINTER(OrcMetrics)]
        _lib.orc_cache_metrics.argtypes = [C.c_void_p, C.c_uint64, C.POINTER(OrcMetrics)]
        _lib.orc_cache_info.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        _lib.orc_cache_layout.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64, C.c_void_p]
        _lib.orc_cache_working_set.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]
        _lib.orc_cache_decode_segment.argtypes = [
            C.c_void_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p]
        _lib.orc_cache_archive_int8.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64] + [C.c_void_p] * 4
        _lib.orc_cache_archive_qvg.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64] + [C.c_void_p] * 4
        _lib.orc_cache_codebooks.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]
        _lib.orc_cache_set_codebooks.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p]
        _lib.orc_quantize_kv_pair.argtypes = [C.c_void_p, C.c_void_p, C.c_int32] + [C.c_uint64] * 4 + [C.c_void_p] * 4
        _lib.orc_dequantize.argtypes = [C.c_void_p, C.c_void_p] + [C.c_uint64] * 5 + [C.c_int32, C.c_void_p]
        _lib.orc_qvg_fit.argtypes = [C.c_void_p, C.c_void_p] + [C.c_uint64] * 6 + [C.c_void_p]
        _lib.orc_qvg_encode.argtypes = [C.c_void_p, C.c_int32, C.c_void_p] + [C.c_uint64] * 7 + [C.c_void_p] * 2
        _lib.orc_qvg_decode.argtypes = [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p] + [C.c_uint64] * 6 + [
            C.c_void_p]
        _lib.orc_pack_bits.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64]
        _lib.orc_unpack_bits.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64]
        _lib.orc_qvg_payload_bytes.argtypes = [C.c_uint64] * 5
        _lib.orc_plan_recent_trim.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64] + [C.c_void_p] * 7
        _lib.orc_splitmix_next.argtypes = [C.POINTER(C.c_uint64)]
        _lib.orc_kv_project.argtypes = [C.c_void_p] * 6 + [C.c_int32, C.c_float, C.c_void_p, C.c_void_p] + [
            C.c_uint64] * 3 + [C.c_void_p] * 2
    return _lib


def set_threads(n: int) -> None:
    """Worker threads for the checker's independent loops (QVG heads, the
    segments a rebuild decodes); 1 keeps everything sequential.  Results do
    not depend on it."""
    lib().orc_set_threads(int(n))


def _check(rc: int):
    if rc != OK:
        raise OracleError(rc, lib().orc_last_error().decode())


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


# ------------------------------------------------------------- free helpers
def randn(shape, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """tensor_utils.rs:114-138 deterministic_randn_affine (f32)."""
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    lib().orc_randn(n, seed, mean, std, _ptr(out))
    return out.reshape(shape)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns (half 2.7.1 round to nearest even)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    rb = 0x8000
    up = ((u & rb) != 0) & ((u & (3 * rb - 1)) != 0)
    out = (u >> 16) + up.astype(np.uint64)
    out = np.where(nan, (u >> 16) | 0x40, out)
    return out.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, np.uint16).astype(np.uint32)
    nan = (b & 0x7FFF) > 0x7F80
    b = np.where(nan, b | 0x40, b)
    return (b << 16).astype(np.uint32).view(np.float32)


def frame_indices(kind: str, total: int, past: int, sampling: int = UNIFORM, gamma: float = 2.0):
    k = {"uniform": 0, "recent_mix": 1, "temporal": 2, "history": 3}[kind]
    cap = max(total, past, 1) + 4
    out = np.zeros(cap, np.uint64)
    n = C.c_uint64()
    _check(lib().orc_frame_indices(k, total, past, sampling, gamma, _ptr(out), cap, C.byref(n)))
    return [int(x) for x in out[: n.value]]


@dataclass
class TrimResult:
    drop_frames: list
    drop_records: list
    evicted_tokens: int
    kept: list


def plan_recent_trim(records, capacity: int, tpf: int) -> TrimResult:
    """records: list of (segment_index, frame_start, frame_count, image_tokens, text_tokens)."""
    n = len(records)
    recs = np.array(records, np.uint64).reshape(n, 5) if n else np.zeros((0, 5), np.uint64)
    recs = np.ascontiguousarray(recs)
    df = np.zeros(2 * n + 2, np.uint64)
    dr = np.zeros(n + 1, np.uint64)
    kept = np.zeros(5 * n + 5, np.uint64)
    n_df, n_dr, ev, n_k = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
    _check(lib().orc_plan_recent_trim(_ptr(recs), n, capacity, tpf, _ptr(df), C.byref(n_df), _ptr(dr), C.byref(n_dr),
                                      C.byref(ev), _ptr(kept), C.byref(n_k)))
    return TrimResult(
        [(int(df[2 * i]), int(df[2 * i + 1])) for i in range(n_df.value)],
        [int(dr[i]) for i in range(n_dr.value)],
        int(ev.value),
        [tuple(int(x) for x in kept[5 * i: 5 * i + 5]) for i in range(n_k.value)],
    )


def quantize_kv_pair(k: np.ndarray, v: np.ndarray, dtype: int):
    """int8.rs:85-134 on raw (B,L,H,D) buffers of `dtype` (f32 array or uint16 bits)."""
    B, L, H, D = k.shape
    kq = np.zeros(k.shape, np.uint8)
    vq = np.zeros(k.shape, np.uint8)
    ks = np.zeros((B, L, H), np.float32)
    vs = np.zeros((B, L, H), np.float32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    _check(lib().orc_quantize_kv_pair(_ptr(k), _ptr(v), dtype, B, L, H, D, _ptr(kq), _ptr(vq), _ptr(ks), _ptr(vs)))
    return kq, vq, ks, vs


def dequantize(q: np.ndarray, s: np.ndarray, valid: int, dtype: int) -> np.ndarray:
    B, L, H, D = q.shape
    out = np.zeros((B, valid, H, D), np.float32 if dtype == F32 else np.uint16)
    q = np.ascontiguousarray(q)
    s = np.ascontiguousarray(s, np.float32)
    _check(lib().orc_dequantize(_ptr(q), _ptr(s), B, L, H, D, valid, dtype, _ptr(out)))
    return out


def kv_project(x, wk, wv, bk=None, bv=None, k_gain=None, qk_norm=False, eps=1e-6, cos=None, sin=None,
               head_dim: int = 128):
    """Captured K / V of one layer (modules/attention.rs:107-124, 143-144):
    bf16 bit arrays in (x: (M, H*D), w*: (H*D, H*D), b*: (H*D,), k_gain:
    (D,)), f32 rope tables (M, D/2); returns the bf16 bits of K and V,
    (M, H*D) each."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    M, dim = x.shape
    H = dim // head_dim
    arrs = [np.ascontiguousarray(a, dtype=np.uint16) if a is not None else None for a in (wk, bk, wv, bv, k_gain)]
    tabs = [np.ascontiguousarray(a, dtype=np.float32) if a is not None else None for a in (cos, sin)]
    k = np.empty((M, dim), np.uint16)
    v = np.empty((M, dim), np.uint16)
    p = lambda a: None if a is None else a.ctypes.data  # noqa: E731
    _check(lib().orc_kv_project(x.ctypes.data, p(arrs[0]), p(arrs[1]), p(arrs[2]), p(arrs[3]), p(arrs[4]),
                                int(bool(qk_norm)), float(np.float32(eps)), p(tabs[0]), p(tabs[1]), M, H, head_dim,
                                k.ctypes.data, v.ctypes.data))
    return k, v


def qvg_fit(k: np.ndarray, v: np.ndarray, stages: int = 4, bits: int = 2, seed: int = 0x5EED0002) -> np.ndarray:
    _, L, H, D = k.shape
    cb = np.zeros((2, H, stages, 1 << bits, D), np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    _check(lib().orc_qvg_fit(_ptr(k), _ptr(v), L, H, D, stages, bits, seed, _ptr(cb)))
    return cb


def qvg_encode(cb: np.ndarray, side: int, t: np.ndarray, tokens: int, block: int = 64):
    _, H, stages, E, D = cb.shape
    bits = E.bit_length() - 1
    L = t.shape[1]
    bpt = (stages * bits + 7) // 8
    nb = (tokens + block - 1) // block
    codes = np.zeros(tokens * H * bpt, np.uint8)
    scales = np.zeros(H * nb * stages, np.float32)
    cb = np.ascontiguousarray(cb, np.float32)
    t = np.ascontiguousarray(t, np.float32)
    _check(lib().orc_qvg_encode(_ptr(cb), side, _ptr(t), L, H, D, tokens, stages, bits, block, _ptr(codes),
                                _ptr(scales)))
    return codes, scales


def qvg_decode(cb: np.ndarray, side: int, codes: np.ndarray, scales: np.ndarray, tokens: int, block: int = 64):
    _, H, stages, E, D = cb.shape
    bits = E.bit_length() - 1
    out = np.zeros((1, tokens, H, D), np.float32)
    cb = np.ascontiguousarray(cb, np.float32)
    _check(lib().orc_qvg_decode(_ptr(cb), side, _ptr(np.ascontiguousarray(codes)),
                                _ptr(np.ascontiguousarray(scales, np.float32)), tokens, H, D, stages, bits, block,
                                _ptr(out)))
    return out


def qvg_payload_bytes(tokens, heads, stages=4, bits=2, block=64) -> int:
    return int(lib().orc_qvg_payload_bytes(tokens, heads, stages, bits, block))


def pack_bits(buf: np.ndarray, bit_off: int, bits: int, value: int):
    lib().orc_pack_bits(_ptr(buf), bit_off, bits, value)


def unpack_bits(buf: np.ndarray, bit_off: int, bits: int) -> int:
    return int(lib().orc_unpack_bits(_ptr(buf), bit_off, bits))


# ------------------------------------------------------------------ bank
@dataclass
class Config:
    storage: int = FLOATING
    sampling: int = RECENT
    gamma: float = 2.0
    capacity: int | None = None
    past_frames: int = 64
    phase_swap: bool = False
    qvg_stages: int = 4
    qvg_bits: int = 2
    qvg_block: int = 64
    qvg_text_as_int8: bool = True
    qvg_seed: int = 0x5EED0002

    def to_c(self) -> OrcConfig:
        return OrcConfig(self.storage, self.qvg_stages, self.qvg_bits, self.qvg_block, int(self.qvg_text_as_int8),
                         self.qvg_seed, self.sampling, self.gamma, int(self.capacity is not None),
                         self.capacity or 0, self.past_frames, int(self.phase_swap))


class Bank:
    """KvBank of oracle HistoryCaches (cache/mod.rs:225-320)."""

    def __init__(self, cfg: Config, n_layers: int, batch: int, heads: int, head_dim: int, dtype: int):
        self.cfg, self.n_layers, self.B, self.H, self.D, self.dtype = cfg, n_layers, batch, heads, head_dim, dtype
        h = C.c_void_p()
        c = cfg.to_c()
        _check(lib().orc_bank_create(C.byref(c), n_layers, batch, heads, head_dim, dtype, C.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().orc_bank_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def commit(self, seg: dict, in_dtype: int, ks, vs, nthreads: int = 1):
        s = OrcSegment(seg["segment_index"], seg["frame_start"], seg["frame_count"], seg["image_tokens"],
                       seg["text_tokens"], seg.get("action_start", -1))
        ks = [np.ascontiguousarray(k) for k in ks]
        vs = [np.ascontiguousarray(v) for v in vs]
        kp = (C.c_void_p * len(ks))(*[k.ctypes.data for k in ks])
        vp = (C.c_void_p * len(vs))(*[v.ctypes.data for v in vs])
        _check(lib().orc_bank_commit(self._h, C.byref(s), in_dtype, kp, vp, nthreads))

    def rollback(self):
        _check(lib().orc_bank_rollback(self._h))

    def park(self):
        _check(lib().orc_bank_park(self._h))

    def unpark(self):
        _check(lib().orc_bank_unpark(self._h))

    def prefill_clone(self, count: int):
        _check(lib().orc_bank_prefill_clone(self._h, count))

    def metrics(self) -> dict:
        m = OrcMetrics()
        _check(lib().orc_bank_metrics(self._h, C.byref(m)))
        return m.as_dict()

    def layer_metrics(self, layer: int) -> dict:
        m = OrcMetrics()
        _check(lib().orc_cache_metrics(self._h, layer, C.byref(m)))
        return m.as_dict()

    def info(self, layer: int = 0) -> dict:
        out = np.zeros(6, np.uint64)
        _check(lib().orc_cache_info(self._h, layer, _ptr(out)))
        keys = ("valid_len", "capacity", "n_segments", "total_frames", "tokens_per_frame", "parked")
        return {k: int(x) for k, x in zip(keys, out)}

    def layout(self, layer: int = 0) -> list:
        n = C.c_uint64()
        cap = 4096
        arr = (OrcLayout * cap)()
        _check(lib().orc_cache_layout(self._h, layer, arr, cap, C.byref(n)))
        return [(a.segment_index, a.video_start, a.video_end, a.text_start, a.text_end, a.action_start)
                for a in arr[: n.value]]

    def _out(self, tokens: int):
        shape = (self.B, tokens, self.H, self.D)
        return np.zeros(shape, np.float32 if self.dtype == F32 else np.uint16)

    def working_set(self, layer: int):
        valid = self.info(layer)["valid_len"]
        k, v = self._out(valid), self._out(valid)
        _check(lib().orc_cache_working_set(self._h, layer, _ptr(k), _ptr(v)))
        return k, v

    def decode_segment(self, layer: int, pos: int, tokens: int):
        k, v = self._out(tokens), self._out(tokens)
        n = C.c_uint64()
        _check(lib().orc_cache_decode_segment(self._h, layer, pos, _ptr(k), _ptr(v), C.byref(n)))
        assert n.value == tokens, (n.value, tokens)
        return k, v

    def archive_int8(self, layer: int, pos: int, tokens: int):
        shape = (self.B, tokens, self.H, self.D)
        kq, vq = np.zeros(shape, np.uint8), np.zeros(shape, np.uint8)
        ks, vs = np.zeros(shape[:3], np.float32), np.zeros(shape[:3], np.float32)
        _check(lib().orc_cache_archive_int8(self._h, layer, pos, _ptr(kq), _ptr(vq), _ptr(ks), _ptr(vs)))
        return kq, vq, ks, vs

    def archive_qvg(self, layer: int, pos: int, video_tokens: int):
        c = self.cfg
        bpt = (c.qvg_stages * c.qvg_bits + 7) // 8
        nb = (video_tokens + c.qvg_block - 1) // c.qvg_block
        kc = np.zeros(video_tokens * self.H * bpt, np.uint8)
        vc = np.zeros_like(kc)
        ksc = np.zeros(self.H * nb * c.qvg_stages, np.float32)
        vsc = np.zeros_like(ksc)
        _check(lib().orc_cache_archive_qvg(self._h, layer, pos, _ptr(kc), _ptr(vc), _ptr(ksc), _ptr(vsc)))
        return kc, vc, ksc, vsc

    def codebooks(self, layer: int):
        c = self.cfg
        cb = np.zeros((2, self.H, c.qvg_stages, 1 << c.qvg_bits, self.D), np.float32)
        fitted = C.c_int32()
        _check(lib().orc_cache_codebooks(self._h, layer, _ptr(cb), C.byref(fitted)))
        return cb if fitted.value else None

    def set_codebooks(self, layer: int, cb: np.ndarray):
        cb = np.ascontiguousarray(cb, np.float32)
        _check(lib().orc_cache_set_codebooks(self._h, layer, _ptr(cb)))
