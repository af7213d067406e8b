"""Deterministic synthetic K/V for tests and benchmarks.

The reference publishes no dataset for its cache path; its tests feed
seeded normal tensors (tensor_utils.rs:114-138).  The benchmark shapes are
8B-geometry segments (48 layers, 24 heads, head_dim 128, BF16), far too many
values to stream from the host, so the generator is counter-based: element
``i`` of a (layer, segment, side) tensor is

    table[mix64(key + (i + 1) * 0x9E3779B97F4A7C15) >> 48] * chan_scale[i % (H*D)]

rounded to the target dtype, where ``table`` holds the 65536 N(0,1) quantiles
at (j + 0.5) / 65536 and ``mix64`` is the SplitMix64 finalizer.  The device
kernel (``nkv_synth_fill``) and :func:`values_numpy` produce identical bits,
so CPU checkers see exactly the tensors the GPU path committed.  Keys get a
per-(layer, head, channel) scale exp(N(0, sigma)) drawn from a SplitMix64 /
Box-Muller stream (sigma 0.5 for the tiny config, 1 for the 8B ones).
"""
from __future__ import annotations

import ctypes as C
import math
from functools import lru_cache
from statistics import NormalDist

import numpy as np

from . import _abi

GOLDEN = 0x9E3779B97F4A7C15
M64 = (1 << 64) - 1


def mix64(z: int) -> int:
    z &= M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def stream_key(seed: int, layer: int, segment: int, side: int) -> int:
    """Key of the (layer, segment, side) tensor; side 0 = K, 1 = V."""
    return mix64(mix64(seed + 0x5EED) ^ ((layer & 0xFFFFF) << 40) ^ ((segment & 0xFFFFFFF) << 8) ^ side)


@lru_cache(maxsize=1)
def quantile_table() -> np.ndarray:
    nd = NormalDist()
    return np.array([nd.inv_cdf((j + 0.5) / 65536.0) for j in range(65536)], dtype=np.float32)


class _SplitMix:
    def __init__(self, seed: int):
        self.state = seed & M64

    def next_u64(self) -> int:
        self.state = (self.state + GOLDEN) & M64
        return mix64(self.state)

    def next_f64(self) -> float:
        return (self.next_u64() >> 11) * (1.0 / (1 << 53))


def _normals(n: int, seed: int) -> list[float]:
    rng = _SplitMix(seed)
    out: list[float] = []
    while len(out) < n:
        u1 = max(rng.next_f64(), 2.2250738585072014e-308)
        u2 = rng.next_f64()
        r = math.sqrt(-2.0 * math.log(u1))
        th = 2.0 * math.pi * u2
        out.append(r * math.cos(th))
        out.append(r * math.sin(th))
    return out[:n]


def chan_scale(seed: int, layer: int, heads: int, head_dim: int, sigma: float) -> np.ndarray:
    """exp(N(0, sigma)) per (head, channel) of one layer's keys, f32 [H*D]."""
    z = _normals(heads * head_dim, mix64(seed * 1000003 + layer + 1))
    return np.array([math.exp(sigma * x) for x in z], dtype=np.float32)


def _round_dtype(x: np.ndarray, dtype: int) -> np.ndarray:
    """f32 -> dtype bits (bf16/f16 round to nearest even) or f32 unchanged."""
    if dtype == _abi.NKV_F32:
        return x.astype(np.float32)
    if dtype == _abi.NKV_F16:
        return x.astype(np.float16).view(np.uint16)
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    out = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    out = np.where(nan, (u >> 16) | 0x40, out)
    return out.astype(np.uint16)


def values_numpy(rows: int, heads: int, head_dim: int, key: int, dtype: int, scale: np.ndarray | None = None,
                 index_offset: int = 0) -> np.ndarray:
    """CPU reproduction of nkv_synth_fill: (rows, H, D) raw dtype array
    (float32, or uint16 bit patterns for bf16 / f16)."""
    n = rows * heads * head_dim
    i = np.arange(n, dtype=np.uint64) + np.uint64(index_offset + 1)
    with np.errstate(over="ignore"):
        z = np.uint64(key) + i * np.uint64(GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    v = quantile_table()[(z >> np.uint64(48)).astype(np.int64)]
    if scale is not None:
        v = (v.reshape(-1, heads * head_dim) * scale[None, :]).reshape(-1).astype(np.float32)
    return _round_dtype(v, dtype).reshape(rows, heads, head_dim)


class DeviceGen:
    """Device-side generator bound to one CUDA device (tables resident)."""

    def __init__(self, device, seed: int = 0, key_sigma: float | None = 1.0):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.seed = seed
        self.key_sigma = key_sigma
        self.table = torch.from_numpy(quantile_table()).to(self.device)
        self._scales: dict[tuple, object] = {}
        self.lib = _abi.load()

    def scale_for(self, layer: int, heads: int, head_dim: int):
        k = (layer, heads, head_dim)
        if k not in self._scales:
            s = chan_scale(self.seed, layer, heads, head_dim, self.key_sigma)
            self._scales[k] = (s, self.torch.from_numpy(s).to(self.device))
        return self._scales[k]

    def fill(self, out, layer: int, segment: int, side: int, dtype: int, stream=None):
        """Fill a contiguous (B, L, H, D) tensor in place."""
        torch = self.torch
        B, L, H, D = out.shape
        sc = None
        if side == 0 and self.key_sigma is not None:
            sc = self.scale_for(layer, H, D)[1]
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        rc = self.lib.nkv_synth_fill(
            C.c_void_p(out.data_ptr()), dtype, B * L, H, D, stream_key(self.seed, layer, segment, side), 0,
            C.c_void_p(self.table.data_ptr()), C.c_void_p(sc.data_ptr() if sc is not None else 0),
            C.c_void_p(st.cuda_stream))
        if rc != 0:
            raise RuntimeError(self.lib.nkv_last_error().decode())
        return out

    def host(self, B: int, L: int, H: int, D: int, layer: int, segment: int, side: int, dtype: int) -> np.ndarray:
        sc = None
        if side == 0 and self.key_sigma is not None:
            sc = chan_scale(self.seed, layer, H, D, self.key_sigma)
        return values_numpy(B * L, H, D, stream_key(self.seed, layer, segment, side), dtype, sc).reshape(B, L, H, D)


def host_values(seed: int, key_sigma: float | None, B: int, L: int, H: int, D: int, layer: int, segment: int,
                side: int, dtype: int) -> np.ndarray:
    """numpy (B, L, H, D) raw-dtype array identical to DeviceGen.fill."""
    sc = chan_scale(seed, layer, H, D, key_sigma) if (side == 0 and key_sigma is not None) else None
    return values_numpy(B * L, H, D, stream_key(seed, layer, segment, side), dtype, sc).reshape(B, L, H, D)


def qvg_codebooks(layer: int, heads: int = 24, head_dim: int = 128, stages: int = 4, entries: int = 4) -> np.ndarray:
    """Frozen synthetic QVG codebooks of the 8B QVG configuration for one
    layer: [side][head][stage][entry][head_dim] f32, codewords ~ N(0, sigma_s)
    with sigma_s = 1, 0.5, 0.25, 0.125 for stages 0..3 (numpy seed
    1000 + layer)."""
    rng = np.random.default_rng(1000 + layer)
    cb = np.zeros((2, heads, stages, entries, head_dim), np.float32)
    for s in range(stages):
        sig = 0.5 ** s
        cb[:, :, s] = rng.standard_normal((2, heads, entries, head_dim)).astype(np.float32) * np.float32(sig)
    return cb
