#!/usr/bin/env python
"""Benchmark of the lifelong KV-cache hot path at 8B geometry.

Workload (the headline configuration, "Nomas-8B geometry INT8 commit +
uniform rebuild"): 48 layers, 24 heads, head_dim 128, BF16 K/V (keys with a
per-channel scale exp(N(0,1))), segments of 4 latent frames x 1560 tokens +
256 text tokens, INT8 storage, uniform history sampling of 16 past frames,
32 archived segments.  One step is one interactive turn through the public
API: commit the new segment (quantize + archive), rebuild the working set
(16 sampled frames + the text blocks of their segments) and gather the
newest segment in full (the "+1 recent segment", HistoryCache::decode_segment
semantics).  Layers are sharded contiguously across ranks (48/N each).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  `value` is device-timed with inputs resident
in HBM; `e2e` repeats the step with the K/V coming from pinned host memory
inside the timed region.  The banks are ShardedKvBanks: every turn carries
the per-turn NCCL broadcast of the 1 KB turn record, on a side stream
while the commit runs.  After the INT8 headline the same run adds, in the same
process, one park + unpark of the working set (phase swap, against the
measured pinned copy bandwidth), a short QVG turn (config 3) and a short
turn with the fused K/V producer against the unfused chain (`--no-extras`
skips them).  `--impl reference` times the CPU restatement of the
reference cache path (oracle/, the reference itself is Rust and cannot be
built here) on the host cores with the same metric.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hy-nomas-rs_b200"))

LAYERS, HEADS, HEAD_DIM = 48, 24, 128
TPF, FRAMES, TEXT = 1560, 4, 256
SEG_TOKENS = FRAMES * TPF + TEXT  # 6496
PAST = 16
ARCHIVED = 32
METRIC = "KV commit+rebuild GB/s (8B geometry, INT8, uniform rebuild)"
METRIC_QVG = "KV commit+rebuild GB/s (8B geometry, QVG, uniform rebuild)"
# The box-run configuration: the same turn with a phase-swapped cache,
# park + unpark of the working set every turn, over a 64-segment archive.
METRIC_SWAP = "KV turn GB/s incl. phase swap (8B geometry, {}, uniform rebuild, park + unpark)"
ARCHIVED_SWAP = 64
WORKLOADS = {"int8": "nomas-8B INT8 commit + uniform rebuild (16 past frames) + newest segment",
             "qvg": "nomas-8B QVG (frozen codebooks) commit + uniform decode-gather rebuild + newest segment"}
# Algorithmic bytes per token per layer: K+V BF16 read (12288) +
# u8 codes and f32 scales written (6336) for a commit; the reverse for a
# gathered output token.
BYTES_PER_TOKEN = 2 * HEADS * HEAD_DIM * 2 + 2 * (HEADS * HEAD_DIM + HEADS * 4)  # 18624


def rebuild_tokens() -> int:
    """Tokens of the rebuilt working set once >= 16 segments are archived:
    16 sampled frames in 16 distinct segments + their text blocks."""
    return PAST * TPF + PAST * TEXT  # 29056


# QVG configuration: per video token and layer 12,288 B read + 48 code
# bytes + 12 scale bytes written = 12,348 B for an encode, the reverse for a
# decode-gathered token (codebooks are cache-resident); text stays INT8.
QVG_BYTES_PER_VIDEO_TOKEN = 2 * HEADS * HEAD_DIM * 2 + 2 * HEADS + 2 * HEADS * 4 * 4 // 64  # 12,348


def working_set_bytes(n_layers: int) -> int:
    """Rebuilt K and V working set in BF16 (what park copies out and unpark back)."""
    return rebuild_tokens() * 2 * HEADS * HEAD_DIM * 2 * n_layers


def step_bytes(n_layers: int, workload: str = "int8", swap: bool = False) -> dict:
    if workload == "qvg":
        video = FRAMES * TPF
        commit = (video * QVG_BYTES_PER_VIDEO_TOKEN + TEXT * BYTES_PER_TOKEN) * n_layers
        rebuild = (PAST * TPF * QVG_BYTES_PER_VIDEO_TOKEN + PAST * TEXT * BYTES_PER_TOKEN) * n_layers
        recent = commit
    else:
        commit = SEG_TOKENS * BYTES_PER_TOKEN * n_layers
        rebuild = rebuild_tokens() * BYTES_PER_TOKEN * n_layers
        recent = SEG_TOKENS * BYTES_PER_TOKEN * n_layers
    sw = 2 * working_set_bytes(n_layers) if swap else 0  # park (D2H) + unpark (H2D)
    return {"commit": commit, "rebuild": rebuild, "recent": recent, "swap": sw,
            "total": commit + rebuild + recent + sw}


def qvg_codebooks(layer: int):
    """Frozen synthetic codebooks of the QVG configuration (nomas_kv.synth)."""
    from nomas_kv import synth
    return synth.qvg_codebooks(layer, HEADS, HEAD_DIM)


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d.get("bf16_tflops", 1400.0))),
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every
    ~5 ms while the timed region runs (nvidia-smi as a fallback)."""

    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
            "hw_power_brake_slowdown": 0x80}

    def __init__(self, local_indices, interval: float = 0.2):
        """Samples the GPUs of `local_indices` (device indices of this
        process) from one thread every `interval` seconds, the first sample
        when start() returns.  Each rank samples only its own GPU: NVML
        queries of GPUs that other processes drive stalled those processes
        (8 ranks: 1.16 ms per turn became 8.7 ms with rank 0 polling all eight
        every 10 ms)."""
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x for x in vis.split(",") if x.strip().isdigit()]
        if isinstance(local_indices, int):
            local_indices = [local_indices]
        self.gpus = [int(ids[i]) if i < len(ids) else i for i in local_indices]
        self.interval = interval
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()
        self._ready = threading.Event()  # first sample taken (or sampling failed)
        self._t = None
        self.err = None

    def _loop(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            hs = [pynvml.nvmlDeviceGetHandleByIndex(g) for g in self.gpus]
            smax = [float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)) for h in hs]
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self._stop.is_set():
                for h, mx in zip(hs, smax):
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    self.samples.append((sm, mx, int(get_reasons(h))))
                self._ready.set()
                self._stop.wait(self.interval)
            pynvml.nvmlShutdown()
        except Exception as e:  # noqa: BLE001
            self.err = repr(e)
            self._smi_loop()
        finally:
            self._ready.set()

    def _smi_loop(self):
        """nvidia-smi polling when NVML is not usable."""
        import subprocess
        q = "clocks.sm,clocks.max.sm,clocks_event_reasons.active"
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                      "-i", ",".join(str(g) for g in self.gpus)], capture_output=True, text=True,
                                     timeout=5).stdout
                for line in out.strip().splitlines():
                    sm, smax, reasons = [x.strip() for x in line.split(",")]
                    self.samples.append((float(sm), float(smax), int(reasons, 16)))
            except Exception as e:  # noqa: BLE001
                self.err = f"{self.err}; nvidia-smi: {e!r}"
                return
            self._ready.set()
            self._stop.wait(self.interval)

    def start(self):
        if not self.gpus:
            return
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._t.start()
        self._ready.wait(timeout=5.0)  # so a short timed region still gets samples

    def stop(self) -> dict:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=5)
        if not self.gpus:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "gpus": 0,
                    "what": "sampled by local rank 0"}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [f"no samples: {self.err}"], "samples": 0}
        reasons = sorted({n for _, _, r in self.samples for n, b in self.BITS.items() if r & b})
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": reasons, "samples": len(self.samples),
                "gpus": len(self.gpus)}


# ------------------------------------------------------------- CPU side
def cpu_sample(threads: int, warmup: int = 1, steps: int = 1, workload: str = "int8", swap: bool = False) -> dict:
    """The oracle (C++ restatement of the reference's CPU cache path, full
    segment decode before index_select) on `threads` layers in parallel, one
    layer per host thread, 8B geometry, archive prefilled like the GPU run
    (32 segments, 64 with the phase swap); `workload` and `swap` select the
    same turn as the GPU arm (QVG with the same frozen codebooks; park and
    unpark every turn)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as orc
    from nomas_kv import synth

    orc.build()
    n = threads
    archived = ARCHIVED_SWAP if swap else ARCHIVED
    cfg = orc.Config(storage=orc.QVG if workload == "qvg" else orc.INT8, sampling=orc.UNIFORM, past_frames=PAST,
                     phase_swap=swap)
    bank = orc.Bank(cfg, n, 1, HEADS, HEAD_DIM, orc.BF16)
    if workload == "qvg":
        for l in range(n):
            bank.set_codebooks(l, qvg_codebooks(l))
    ks = [synth.host_values(0, 1.0, 1, SEG_TOKENS, HEADS, HEAD_DIM, l, 0, 0, 1) for l in range(n)]
    vs = [synth.host_values(0, 1.0, 1, SEG_TOKENS, HEADS, HEAD_DIM, l, 0, 1, 1) for l in range(n)]
    seg = dict(segment_index=0, frame_start=0, frame_count=FRAMES, image_tokens=FRAMES * TPF, text_tokens=TEXT)
    bank.commit(seg, orc.BF16, ks, vs, nthreads=n)
    bank.prefill_clone(archived - 2 - warmup)
    idx = archived - 1 - warmup
    times = []
    for i in range(warmup + steps):
        s = dict(seg, segment_index=idx, frame_start=idx * FRAMES)
        t0 = time.perf_counter()
        bank.commit(s, orc.BF16, ks, vs, nthreads=n)
        # the "+1 recent segment": full decode of the newest segment per layer
        ths = [threading.Thread(target=bank.decode_segment, args=(l, idx, SEG_TOKENS)) for l in range(n)]
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        if swap:  # phase_swap.rs:42-92: the working set to host memory and back
            bank.park()
            bank.unpark()
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
        idx += 1
    bank.close()
    sec = sum(times) / len(times)
    what = "commit + uniform rebuild + newest-segment decode" + (" + park + unpark" if swap else "")
    return {"value": step_bytes(n, workload, swap)["total"] / sec / 1e9, "unit": "GB/s", "cores": n, "kind": "port",
            "sample": f"{n} layer(s) x {len(times)} turn(s) ({workload.upper()}: {what}) at 8B geometry, "
                      f"archive of {archived} segments, one host thread per layer; "
                      f"{sec:.2f} s per turn"}


def cpu_sample_project(threads: int, rows: int = 96) -> dict:
    """The oracle's restatement of the producer chain (Lin + bias, RmsNorm,
    RoPE; modules/attention.rs:107-124, 143-144) plus quantize_kv_pair for
    `rows` tokens of one layer at the 8B geometry, one layer per host
    thread; scaled to segment tokens/s over all 48 layers.  The archive /
    rebuild part of the turn is left out: it is under 0.1 % of the
    projection's CPU time."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as orc

    orc.build()
    rng = np.random.default_rng(0)
    b = lambda a: orc.bf16_bits(np.asarray(a, np.float32))  # noqa: E731
    dim = HEADS * HEAD_DIM
    w = [dict(wk=b(rng.standard_normal((dim, dim)) / np.sqrt(dim)), wv=b(rng.standard_normal((dim, dim)) / np.sqrt(dim)),
              bk=b(0.1 * rng.standard_normal(dim)), bv=b(0.1 * rng.standard_normal(dim)),
              gain=b(1 + 0.1 * rng.standard_normal(HEAD_DIM))) for _ in range(threads)]
    x = b(rng.standard_normal((rows, dim)))
    ang = rng.uniform(0, 6.3, (rows, HEAD_DIM // 2)).astype(np.float32)
    cos, sin = np.cos(ang), np.sin(ang)

    def one(i):
        k, v = orc.kv_project(x, w[i]["wk"], w[i]["wv"], bk=w[i]["bk"], bv=w[i]["bv"], k_gain=w[i]["gain"],
                              qk_norm=True, eps=1e-6, cos=cos, sin=sin)
        orc.quantize_kv_pair(k.reshape(1, rows, HEADS, HEAD_DIM), v.reshape(1, rows, HEADS, HEAD_DIM), orc.BF16)

    t0 = time.perf_counter()
    ths = [threading.Thread(target=one, args=(i,)) for i in range(threads)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    sec = time.perf_counter() - t0
    value = rows * threads / sec / LAYERS  # tokens/s through all 48 layers
    return {"value": value, "unit": "segment tokens/s (all layers)", "cores": threads, "kind": "port",
            "sample": f"{rows} tokens x {threads} layer(s) of the producer chain + quantize at the 8B geometry "
                      f"(f64-accumulated GEMM, one host thread per layer), {sec:.2f} s; scaled to 48 layers"}


def host_policy_latency(reps: int = 2000) -> dict:
    """Host latency of the index evaluation and the SWA trim plan (they move
    ~0 bytes): raw C-ABI calls with preallocated buffers, so the figure is the
    policy code plus one ctypes transition.  Sizes of the long-session
    configuration: 1,024 frames, 32 past frames; a trim over 256 records."""
    import numpy as np
    import nomas_kv as nk

    lib = nk.lib()
    out = np.zeros(1100, np.uint64)
    n = C.c_uint64()
    res = {}
    for name, kind, sampling, gamma in (("uniform_frame_indices_us", 0, nk.NKV_SAMPLING_UNIFORM, 2.0),
                                        ("recent_mix_indices_us", 1, nk.NKV_SAMPLING_RECENT_MIX, 2.0),
                                        ("temporal_context_indices_us", 2, nk.NKV_SAMPLING_TEMPORAL, 0.9)):
        ptr = out.ctypes.data_as(C.c_void_p)
        t0 = time.perf_counter()
        for _ in range(reps):
            lib.nkv_frame_indices(kind, 1024, 32, sampling, gamma, ptr, out.size, C.byref(n))
        res[name] = round((time.perf_counter() - t0) / reps * 1e6, 3)
    recs = np.array([[i, 4 * i, 4, 4 * TPF, TEXT] for i in range(256)], np.uint64)
    df, dr, kept = np.zeros(514, np.uint64), np.zeros(257, np.uint64), np.zeros(1285, np.uint64)
    ndf, ndr, ev, nkp = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
    pr, pdf, pdr, pk = (a.ctypes.data_as(C.c_void_p) for a in (recs, df, dr, kept))
    cap = 200 * SEG_TOKENS + 3 * TPF  # evicts whole records and part of a video block
    t0 = time.perf_counter()
    for _ in range(reps):
        lib.nkv_plan_recent_trim(pr, 256, cap, TPF, pdf, C.byref(ndf), pdr, C.byref(ndr), C.byref(ev), pk,
                                 C.byref(nkp))
    res["recent_trim_plan_us"] = round((time.perf_counter() - t0) / reps * 1e6, 3)
    res["what"] = "host C++ policy per call incl. one ctypes call; 1,024 frames / 32 past; trim over 256 records"
    return res


# ------------------------------------------------------------ GPU side
def _dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        # The group carries only host metadata (the 1 KB turn record, timings,
        # counters): one channel and no NVLS, so its kernels hold one SM while
        # they wait for the other ranks.  High-priority NCCL streams only for
        # the strict protocol, which waits for its collectives inside the
        # turn; the default broadcast is checked a turn later and must not be
        # dispatched ahead of the rebuild gather's CTAs.
        os.environ.setdefault("NCCL_MAX_NCHANNELS", "1")
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = getattr(args, "verify", "broadcast") == "strict"
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev, pg_options=opts)
    return world, rank, local, dev


def _max_over_ranks(world: int, dev, values: list[float]) -> list[float]:
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def _gather_clocks(world: int, mine: dict) -> dict:
    """Every rank's clock summary merged for rank 0's line (after the timed
    region): the median of the ranks' medians, the largest maximum, the union
    of the reasons."""
    if world == 1:
        return mine
    import torch.distributed as dist
    allc = [None] * world
    dist.all_gather_object(allc, mine)
    sm = [c["sm_mhz"] for c in allc if c.get("sm_mhz") is not None]
    mx = [c["sm_max_mhz"] for c in allc if c.get("sm_max_mhz") is not None]
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted({r for c in allc for r in c.get("reasons", [])}),
            "samples": sum(c.get("samples", 0) for c in allc), "gpus": world,
            "per_rank_sm_mhz": [c.get("sm_mhz") for c in allc]}


def _barrier(world: int) -> None:
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def host_link_peaks(world: int, dev, nbytes: int = 1 << 30, reps: int = 3) -> dict:
    """Pinned host <-> device copy bandwidth with every rank copying at the
    same time (the bound of the e2e figure and of park / unpark): per GPU,
    and aggregated over the job (bytes of all ranks / the slowest rank)."""
    import torch
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    devb = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s = torch.cuda.current_stream(dev)
    out = {}
    for name, fn in (("h2d", lambda: devb.copy_(host, non_blocking=True)),
                     ("d2h", lambda: host.copy_(devb, non_blocking=True))):
        best = float("inf")
        for _ in range(reps):
            _barrier(world)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            fn()
            b.record(s)
            b.synchronize()
            best = min(best, a.elapsed_time(b))
        ms = _max_over_ranks(world, dev, [best])[0]
        out[f"{name}_gbs_per_gpu"] = round(nbytes / (best / 1e3) / 1e9, 2)
        out[f"{name}_gbs_aggregate"] = round(world * nbytes / (ms / 1e3) / 1e9, 2)
    del host, devb
    torch.cuda.empty_cache()
    out["what"] = f"pinned {nbytes >> 20} MiB copies, all {world} rank(s) at once, best of {reps}"
    return out


class Turns:
    """One cache workload at the 8B geometry on this rank's layers, driven
    through the layer-sharded bank (its per-turn NCCL record broadcast and
    status exchange included): prefill, warm-up and timed turns (commit +
    rebuild + newest-segment decode), kernel statistics."""

    def __init__(self, args, world, rank, dev, workload: str, phase_swap: bool, archived: int,
                 max_turns: int):
        import torch
        import nomas_kv as nk
        from nomas_kv import synth
        from nomas_kv.sharded import ShardedKvBank

        self.torch, self.nk = torch, nk
        self.world, self.rank, self.dev, self.wl = world, rank, dev, workload
        self.model_layers = args.layers
        storage = nk.CacheStorage.qvg_() if workload == "qvg" else nk.CacheStorage.int8()
        cfg = nk.CacheConfig(storage=storage, sampling=nk.HistorySampling.uniform(), past_frames=PAST,
                             phase_swap=phase_swap)
        self.sb = ShardedKvBank(cfg, args.layers, 1, HEADS, HEAD_DIM, torch.bfloat16, device=dev,
                                verify=getattr(args, "verify", "broadcast"))
        self.bank = self.sb.local
        self.begin, self.n_layers = self.sb.begin, self.sb.count
        self.stream = torch.cuda.current_stream(dev)
        if workload == "qvg":
            for i in range(self.n_layers):
                self.bank.layer(i).set_qvg_codebooks(synth.qvg_codebooks(self.begin + i, HEADS, HEAD_DIM))
        self.prefill = max(1, archived - 1 - args.warmup)
        tier_gb = getattr(args, "archive_device_gb", 0.0) if workload == args.workload else 0.0
        if tier_gb > 0:
            # the tiered archive: slabs beyond this many device bytes live in
            # pinned, device-mapped host memory and are read over the host link
            self.bank.set_archive_device_limit(int(tier_gb * 1e9))
        self.bank.reserve(self.bank.segment_bytes(self.desc(0)) * self.n_layers * (self.prefill + max_turns),
                          rebuild_tokens())
        # two resident input sets (each > L2), alternated turn to turn
        gen = synth.DeviceGen(dev, seed=0, key_sigma=1.0)
        self.shape = (1, SEG_TOKENS, HEADS, HEAD_DIM)
        self.sets = []
        for s in range(2):
            ks = [torch.empty(self.shape, dtype=torch.bfloat16, device=dev) for _ in range(self.n_layers)]
            vs = [torch.empty(self.shape, dtype=torch.bfloat16, device=dev) for _ in range(self.n_layers)]
            for i in range(self.n_layers):
                gen.fill(ks[i], self.begin + i, s, 0, nk.NKV_BF16)
                gen.fill(vs[i], self.begin + i, s, 1, nk.NKV_BF16)
            self.sets.append((ks, vs))
        self.recent_k = [torch.empty(self.shape, dtype=torch.bfloat16, device=dev) for _ in range(self.n_layers)]
        self.recent_v = [torch.empty(self.shape, dtype=torch.bfloat16, device=dev) for _ in range(self.n_layers)]
        self.seg = 0

    def desc(self, i: int):
        return self.nk._abi.nkv_segment_desc(i, i * FRAMES, FRAMES, FRAMES * TPF, TEXT, 0)

    def turn(self, ks=None, vs=None):
        if ks is None:
            ks, vs = self.sets[self.seg % 2]
        # validate + encode + rebuild, and the newest segment decoded in full
        # by the same gather launch (one host wait for the non-finite flags)
        self.sb.commit(self.desc(self.seg), ks, vs, self.recent_k, self.recent_v)
        self.seg += 1

    def fill_archive(self, warmup: int):
        for _ in range(self.prefill + warmup):
            self.turn()
        assert self.bank.layer(0).valid_len() == rebuild_tokens(), self.bank.layer(0).valid_len()

    def timed(self, steps: int):
        """Device time of `steps` turns (max over ranks) and the kernel stats."""
        torch = self.torch
        self.bank.kernel_stats(reset=True)
        self.bank.set_timing(True)
        _barrier(self.world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(self.stream)
        for _ in range(steps):
            self.turn()
        t1.record(self.stream)
        torch.cuda.synchronize()
        _barrier(self.world)
        self.bank.set_timing(False)
        kst = self.bank.kernel_stats(reset=True)
        return _max_over_ranks(self.world, self.dev, [t0.elapsed_time(t1)])[0], kst

    def kernel_figures(self, kst: dict, steps: int, peak: float) -> dict:
        """Achieved GB/s of the turn's kernels on this rank (CUDA events on
        the bank's stream around each launch), algorithmic bytes per launch."""
        sb = step_bytes(self.n_layers, self.wl)
        g_launch, g_ms = kst["gather"]
        d_launch, d_ms = kst["segment_decode"]
        q_launch, q_ms = kst["quantize"]
        e_launch, e_ms = kst["qvg_encode"]
        gbs = lambda b, ms: b / (ms / 1e3) / 1e9 if ms > 0 else None  # noqa: E731
        # one gather launch per turn: the rebuild and the newest segment
        out = {"rebuild_gather_gbs": gbs((sb["rebuild"] + sb["recent"]) * steps, g_ms)}
        if self.wl == "qvg":
            out["qvg_encode_gbs"] = gbs(FRAMES * TPF * QVG_BYTES_PER_VIDEO_TOKEN * self.n_layers * steps, e_ms)
            out["text_quantize_gbs"] = gbs(TEXT * BYTES_PER_TOKEN * self.n_layers * steps, q_ms)
        else:
            out["quantize_gbs"] = gbs(sb["commit"] * steps, q_ms)
        res = {}
        for k, v in out.items():
            res[k] = round(v, 1) if v else None
            res[k.replace("_gbs", "_frac")] = round(v / peak, 4) if v else None
        res["launches"] = g_launch + d_launch + q_launch + e_launch
        res["rebuild_gather_ms_per_launch"] = round(g_ms / max(g_launch, 1), 4)
        return res

    def close(self):
        self.bank.close()
        self.sets = self.recent_k = self.recent_v = None
        self.torch.cuda.synchronize()
        self.torch.cuda.empty_cache()


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    world, rank, local, dev = _dist_setup(args)
    wl = args.workload
    swap = args.swap
    model_layers = args.layers
    peaks = load_peaks()
    extras = wl == "int8" and not swap and not args.no_extras

    # the swap run holds a 64-segment archive (~142 GB at 48 layers on one
    # GPU): fewer e2e turns, and the e2e staging reuses a resident input set
    e2e_steps = min(args.steps, 2 if swap else 4)
    archived = ARCHIVED_SWAP if swap else ARCHIVED
    # the INT8 headline bank is a phase-swapped cache (PhaseSwappedCache,
    # phase_swap.rs:27-161) so that one park + unpark can be timed after the
    # timed turns; while not parked its turns are the plain HistoryCache's
    T = Turns(args, world, rank, dev, wl, phase_swap=swap or extras, archived=archived,
              max_turns=2 * args.warmup + args.steps + e2e_steps + 1)
    n_layers, stream = T.n_layers, T.stream
    swap_ms = [0.0, 0.0]  # park, unpark: device time on the bank's stream
    sev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]

    def park_unpark():
        # phase_swap.rs:42-92: the working set goes to host memory and back;
        # both calls return after their copies completed
        sev[0].record(stream)
        T.sb.park_all()
        sev[1].record(stream)
        T.sb.unpark_all()
        sev[2].record(stream)
        sev[2].synchronize()
        swap_ms[0] += sev[0].elapsed_time(sev[1])
        swap_ms[1] += sev[1].elapsed_time(sev[2])

    def step():
        T.turn()
        if swap:
            park_unpark()

    # the prefill only builds the archive: no swaps while the working set is
    # still growing (a re-grown set would briefly coexist with its successor)
    T.fill_archive(0)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---------------------------------------------------- timed: resident
    # one GPU: 20 ms polling costs nothing measurable; several ranks: the
    # recipe's 200 ms, each rank its own GPU
    clocks = ClockSampler(local, 0.02 if world == 1 else 0.2)
    T.bank.kernel_stats(reset=True)
    T.bank.set_timing(True)
    _barrier(world)
    clocks.start()
    swap_ms[0] = swap_ms[1] = 0.0
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    clk = _gather_clocks(world, clocks.stop())
    T.bank.set_timing(False)
    kst = T.bank.kernel_stats(reset=True)
    ms_max = _max_over_ranks(world, dev, [t0.elapsed_time(t1)])[0]
    bytes_all = step_bytes(model_layers, wl, swap)["total"] * args.steps
    value = bytes_all / (ms_max / 1e3) / 1e9
    link = host_link_peaks(world, dev)
    swap_info = None
    if swap:
        wsb = working_set_bytes(n_layers) * args.steps
        pt = _max_over_ranks(world, dev, swap_ms)
        swap_info = {"bytes_per_direction_per_step": working_set_bytes(model_layers),
                     "park_gbs_per_gpu": round(wsb / (pt[0] / 1e3) / 1e9, 2),
                     "unpark_gbs_per_gpu": round(wsb / (pt[1] / 1e3) / 1e9, 2),
                     "park_ms_per_step": round(pt[0] / args.steps, 3),
                     "unpark_ms_per_step": round(pt[1] / args.steps, 3),
                     "bound": "host link (PCIe), per GPU", "link": link}

    # ---------------------------------------------------- timed: e2e (host buffers)
    host = []
    for s in range(2):
        hk = [torch.empty(T.shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(n_layers)]
        hv = [torch.empty(T.shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(n_layers)]
        for i in range(n_layers):
            hk[i].copy_(T.sets[s][0][i])
            hv[i].copy_(T.sets[s][1][i])
        host.append((hk, hv))
    # Pipelined turns: turn j+1's K/V cross PCIe on a copy stream (into the
    # other resident input set, free again) while turn j commits; commit
    # returns only after its kernels ran, so its buffer is free for turn j+2.
    flag_host = torch.empty(1, dtype=torch.int32, pin_memory=True)
    vlen_dev = torch.empty(1, dtype=torch.int32, device=dev)
    copy_stream = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]

    def enqueue_copy(j: int, b: int):
        hk, hv = host[(T.seg + j) % 2]
        copy_stream.wait_stream(stream)  # after the last reader of buffer b
        with torch.cuda.stream(copy_stream):
            for i in range(n_layers):
                T.sets[b][0][i].copy_(hk[i], non_blocking=True)
                T.sets[b][1][i].copy_(hv[i], non_blocking=True)
        copied[b].record(copy_stream)

    def e2e_turns(n_turns: int):
        enqueue_copy(0, 0)
        for j in range(n_turns):
            b = j % 2
            if j + 1 < n_turns:
                enqueue_copy(j + 1, 1 - b)
            stream.wait_event(copied[b])
            T.turn(*T.sets[b])
            if swap:
                park_unpark()
            # device -> host read of the turn's result: the working-set length
            vlen_dev.fill_(T.bank.layer(0).valid_len())
            flag_host.copy_(vlen_dev, non_blocking=True)

    e2e_turns(args.warmup)
    _barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_turns(e2e_steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = _max_over_ranks(world, dev, [e0.elapsed_time(e1)])[0]
    e2e_value = step_bytes(model_layers, wl, swap)["total"] * e2e_steps / (ems / 1e3) / 1e9
    h2d = 2 * SEG_TOKENS * HEADS * HEAD_DIM * 2 * model_layers
    d2h = (4 + 4) * world  # commit's non-finite flag + the result read, per rank
    # the e2e ceiling when only the K/V upload bounded a turn
    e2e_bound = step_bytes(model_layers, wl, swap)["total"] / (h2d / (link["h2d_gbs_aggregate"] * 1e9)) / 1e9

    # ---------------------------------------------------- one park + unpark (phase swap)
    if extras:
        swap_ms[0] = swap_ms[1] = 0.0
        _barrier(world)
        park_unpark()  # first one allocates the pinned host buffers
        swap_ms[0] = swap_ms[1] = 0.0
        _barrier(world)
        park_unpark()
        pt = _max_over_ranks(world, dev, swap_ms)
        wsb = working_set_bytes(n_layers)
        swap_info = {"bytes_per_direction": working_set_bytes(model_layers),
                     "park_gbs_per_gpu": round(wsb / (pt[0] / 1e3) / 1e9, 2),
                     "unpark_gbs_per_gpu": round(wsb / (pt[1] / 1e3) / 1e9, 2),
                     "park_ms": round(pt[0], 3), "unpark_ms": round(pt[1], 3),
                     "park_frac": round(wsb / (pt[0] / 1e3) / 1e9 / link["d2h_gbs_per_gpu"], 4),
                     "unpark_frac": round(wsb / (pt[1] / 1e3) / 1e9 / link["h2d_gbs_per_gpu"], 4),
                     "bound": "host link: fractions of the measured pinned copy bandwidth per GPU with every rank "
                              "copying at once", "link": link}
    attend = attend_measure(T, peaks) if extras else None
    gk = T.kernel_figures(kst, args.steps, peaks["hbm_gbs"])
    tiers = None
    if args.archive_device_gb > 0:
        dev_b, host_b = T.bank.archive_usage()
        tiers = {"device_limit_gb": args.archive_device_gb, "archive_device_gb": round(dev_b / 1e9, 2),
                 "archive_host_gb": round(host_b / 1e9, 2),
                 "what": "archive slabs beyond the device limit in pinned, device-mapped host memory; the rebuild "
                         "gather reads those over the host link"}
    T.close()
    del host

    qvg = project = None
    if extras:
        qvg = run_qvg_extra(args, world, rank, dev, peaks)
        project = project_measure(args, world, rank, dev, peaks, steps=3, warmup=3, e2e_steps=0, cpu=False)

    # ---------------------------------------------------- roofline (gather)
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        t = json.load(open(tp)).get(f"{wl}_rebuild_gather")
        if t:
            traffic = int(t["dram_bytes"] / t["layers"] * n_layers)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = min(os.cpu_count() or 1, LAYERS)
        try:
            cpu = cpu_sample(cores, workload=wl, swap=swap)
            one = cpu_sample(1, workload=wl, swap=swap)
            cpu["single_thread_value"] = one["value"]
            cpu["single_thread_sample"] = one["sample"]
            cpu["host_nproc"] = os.cpu_count()
        except Exception as e:  # noqa: BLE001
            cpu = {"value": None, "unit": "GB/s", "cores": 0, "kind": "port", "sample": f"failed: {e}"}
    sec = ms_max / 1e3
    tok = {"commit": round(SEG_TOKENS * args.steps / sec), "rebuild_out": round(rebuild_tokens() * args.steps / sec),
           "newest_segment_out": round(SEG_TOKENS * args.steps / sec), "unit": "segment tokens/s (all layers)"}

    if rank == 0:
        sbytes = step_bytes(n_layers, wl)
        out = {
            "metric": (METRIC_SWAP.format(wl.upper()) if swap else METRIC if wl == "int8" else METRIC_QVG),
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOADS[wl] + (" + park/unpark (phase swap) every turn" if swap else ""),
                       "layers": model_layers, "heads": HEADS, "head_dim": HEAD_DIM, "segment_tokens": SEG_TOKENS,
                       "tokens_per_frame": TPF, "frames_per_segment": FRAMES, "text_tokens": TEXT,
                       "past_frames": PAST, "archived_segments_at_first_timed_step": T.prefill + args.warmup + 1,
                       "phase_swap": swap,
                       "working_set_tokens": rebuild_tokens(), "bytes_per_step": step_bytes(model_layers, wl, swap)["total"],
                       "parallelism": f"layer-sharded x{world} (ShardedKvBank: per-turn NCCL broadcast of the "
                                      f"1 KB turn record on a side stream, no data-path collective)",
                       "l2": "inputs 3.8 GB per step > 126 MB L2"},
            "tokens_per_s": tok,
            "host_policy_latency": host_policy_latency(),
            "phase_swap": swap_info,
            "roofline": {"bound": "hbm", "achieved": gk["rebuild_gather_gbs"],
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gk["rebuild_gather_frac"],
                         "traffic": traffic,
                         "kernel": "k_gather (each commit's one gather launch: the rebuild of the working set and "
                                   "the newest segment decoded in full)",
                         "algorithmic_bytes_per_launch": sbytes["rebuild"] + sbytes["recent"],
                         "peak_src": peaks["src"], **{k: v for k, v in gk.items()
                                                      if k not in ("rebuild_gather_gbs", "rebuild_gather_frac")}},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "result": "the rebuilt working set stays in HBM, where attention reads it; the device-to-host "
                              "read per turn is the commit's status word and the working-set length",
                    "bound_gbs": round(e2e_bound, 1),
                    "bound": f"the K/V upload: {h2d / 1e9:.2f} GB per turn at the measured aggregate pinned H2D "
                             f"{link['h2d_gbs_aggregate']} GB/s with all {world} GPU(s) copying at once"},
            "qvg": qvg,
            "producer": project,
            "archive_tiers": tiers,
            "attend_history": attend,
            "gpu_launches": gk["launches"],
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def attend_measure(T, peaks, reps: int = 3) -> dict:
    """The fused consumer: one segment's queries (6,496 x 24 heads) attending
    to layer 0's history (29,056 keys) straight from the INT8 archive
    (nkv_bank_attend_history), beside torch's scaled_dot_product_attention
    over the materialised bf16 working set (the library path it replaces)."""
    import torch
    import torch.nn.functional as F
    dev = T.dev
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn((SEG_TOKENS, HEADS, HEAD_DIM), generator=g, device=dev).to(torch.bfloat16)
    lay = T.bank.layer(0)
    out, lse = lay.attend_history(q)  # warm-up
    T.bank.kernel_stats(reset=True)
    T.bank.set_timing(True)
    for _ in range(reps):
        lay.attend_history(q, out=out, lse=lse)
    T.bank.set_timing(False)
    n, ms = T.bank.kernel_stats(reset=True)["attend"]
    ms /= max(n, 1)
    k, v = lay.working_set()
    keys = k.shape[1]
    flops = 4.0 * SEG_TOKENS * keys * HEAD_DIM * HEADS
    qt, kt, vt = q.unsqueeze(0).transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    F.scaled_dot_product_attention(qt, kt, vt)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        F.scaled_dot_product_attention(qt, kt, vt)
    b.record()
    torch.cuda.synchronize()
    sdpa_ms = a.elapsed_time(b) / reps
    tf = flops / (ms / 1e3) / 1e12
    return {"kernel": "k_attend_int8 (tcgen05, INT8 K/V dequantized in shared memory)", "queries": SEG_TOKENS,
            "history_keys": keys, "heads": HEADS, "ms": round(ms, 3), "tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4), "peak_tflops": peaks["bf16_tflops"],
            "sdpa_bf16_working_set_ms": round(sdpa_ms, 3),
            "sdpa_tflops": round(flops / (sdpa_ms / 1e3) / 1e12, 1),
            "int8_bytes_read": keys * HEADS * HEAD_DIM * 2 + keys * HEADS * 8,
            "bf16_bytes_read_by_sdpa": keys * HEADS * HEAD_DIM * 4}


def run_qvg_extra(args, world, rank, dev, peaks, steps: int = 3, warmup: int = 3) -> dict:
    """A short QVG turn (config 3: frozen codebooks, 98-block video encode,
    INT8 text, uniform decode-gather rebuild of 16 frames, newest segment)
    after the INT8 bank is closed."""
    import torch
    T = Turns(args, world, rank, dev, "qvg", phase_swap=False, archived=PAST + 1 + warmup,
              max_turns=warmup + steps + 1)
    T.fill_archive(warmup)
    ms, kst = T.timed(steps)
    gk = T.kernel_figures(kst, steps, peaks["hbm_gbs"])
    T.close()
    del T
    torch.cuda.empty_cache()
    total = step_bytes(args.layers, "qvg")["total"]
    return {"metric": METRIC_QVG, "value": round(total * steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "ms_per_step": round(ms / steps, 4), "steps": steps, "warmup": warmup,
            "archived_segments": PAST + 1 + warmup, "peak": peaks["hbm_gbs"], "peak_src": peaks["src"],
            "gpu_launches": gk.pop("launches"), **gk}


# ------------------------------------------------- producer (projection)
METRIC_PROJECT = "captured-K/V commit tokens/s (8B geometry, INT8, fused K/V projection producer)"
DIM = HEADS * HEAD_DIM  # 3072
PROJECT_FLOPS = 2 * SEG_TOKENS * (2 * DIM) * DIM  # one layer's K and V projection of a segment


def project_measure(args, world, rank, dev, peaks, steps: int, warmup: int, e2e_steps: int, cpu: bool,
                    archived: int = PAST + 1) -> dict:
    """The commit with its producer: per layer, the K / V projection of the
    segment's attention input (Lin + bias, RmsNorm and RoPE on K) with the
    INT8 archive rows written by the same tcgen05 kernel (nkv_kv_project),
    then the staged commit (archive + uniform rebuild) and the newest-segment
    gather.  Beside it, the same turn unfused (cuBLAS projection, the bias /
    RmsNorm / RoPE chain in eager PyTorch, then commit_tensors, which
    quantizes) and cuBLAS alone on the same GEMM shape."""
    import torch
    import nomas_kv as nk
    from nomas_kv import synth

    begin, n_layers = nk.partition_layers(args.layers, world, rank)
    stream = torch.cuda.current_stream(dev)
    cfg = nk.CacheConfig(storage=nk.CacheStorage.int8(), sampling=nk.HistorySampling.uniform(), past_frames=PAST)
    bank = nk.KvBank(cfg, n_layers, 1, HEADS, HEAD_DIM, torch.bfloat16, device=dev, layer_begin=begin)
    desc = lambda i: nk._abi.nkv_segment_desc(i, i * FRAMES, FRAMES, FRAMES * TPF, TEXT, 0)  # noqa: E731
    L = SEG_TOKENS
    prefill = max(1, archived - 1 - warmup)
    total = prefill + 2 * (warmup + steps) + e2e_steps + 3
    bank.reserve(bank.segment_bytes(desc(0)) * n_layers * total, rebuild_tokens())

    g = torch.Generator(device=dev)
    g.manual_seed(1234 + begin)
    def randn(*shape, scale=1.0):  # noqa: E306
        return (torch.randn(*shape, device=dev, generator=g) * scale).to(torch.bfloat16)
    wk = [randn(DIM, DIM, scale=DIM ** -0.5) for _ in range(n_layers)]
    wv = [randn(DIM, DIM, scale=DIM ** -0.5) for _ in range(n_layers)]
    bk = [randn(DIM, scale=0.1) for _ in range(n_layers)]
    bv = [randn(DIM, scale=0.1) for _ in range(n_layers)]
    gain = [(1 + randn(HEAD_DIM, scale=0.1).float()).to(torch.bfloat16) for _ in range(n_layers)]
    wkv = [torch.cat([wk[i], wv[i]], 0) for i in range(n_layers)]  # the unfused arm's one GEMM per layer
    xs = [[randn(L, DIM) for _ in range(n_layers)] for _ in range(2)]  # two input sets (each > L2)
    # the segment's 3D RoPE table (rope.rs:115-150 layout: one angle per pair)
    pos = torch.arange(L, device=dev, dtype=torch.float32)[:, None]
    freq = torch.pow(torch.tensor(256.0, device=dev), -torch.arange(0, HEAD_DIM, 2, device=dev) / HEAD_DIM)
    ang = pos * freq[None, :]
    rope = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
    k_out = [torch.empty((1, L, HEADS, HEAD_DIM), dtype=torch.bfloat16, device=dev) for _ in range(n_layers)]
    v_out = [torch.empty_like(t) for t in k_out]
    recent_k = [torch.empty_like(t) for t in k_out]
    recent_v = [torch.empty_like(t) for t in k_out]
    seg = 0
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(n_layers)]
    proj_ms = [0.0, 0]

    def fused(xset, time_launches=False):
        nonlocal seg
        staged = bank.stage_segment(desc(seg))
        for i in range(n_layers):
            if time_launches:
                ev[i][0].record(stream)
            nk.kv_project(xs[xset][i], wk[i], wv[i], bk=bk[i], bv=bv[i], k_gain=gain[i], qk_norm=True, eps=1e-6,
                          rope=rope, k_out=k_out[i].view(L, DIM), v_out=v_out[i].view(L, DIM), codes=staged[i],
                          ranges=[(0, L, 0)], status_ptr=staged[i]["status"], stream=stream)
            if time_launches:
                ev[i][1].record(stream)
        bank.commit_staged()
        bank.decode_segment(seg, recent_k, recent_v)
        seg += 1
        if time_launches:
            torch.cuda.synchronize()
            proj_ms[0] += sum(e[0].elapsed_time(e[1]) for e in ev)
            proj_ms[1] += n_layers

    def unfused(xset):
        nonlocal seg
        for i in range(n_layers):
            kv = torch.matmul(xs[xset][i], wkv[i].T)  # cuBLAS, bf16 out
            k = (kv[:, :DIM] + bk[i]).view(L, HEADS, HEAD_DIM).float()
            v = kv[:, DIM:] + bv[i]
            k = (k * torch.rsqrt((k * k).mean(-1, keepdim=True) + 1e-6) * gain[i].float()).to(torch.bfloat16).float()
            kr, ki = k[..., 0::2], k[..., 1::2]
            c, sn = rope[0][:, None, :], rope[1][:, None, :]
            k = torch.stack([kr * c - ki * sn, ki * c + kr * sn], -1)
            k_out[i].view(L, HEADS, HEAD_DIM).copy_(k.view(L, HEADS, HEAD_DIM))
            v_out[i].view(L, DIM).copy_(v)
        bank.commit_tensors(desc(seg), k_out, v_out)
        bank.decode_segment(seg, recent_k, recent_v)
        seg += 1

    # prefill: the archive through the plain commit of synthetic K / V
    gen = synth.DeviceGen(dev, seed=0, key_sigma=1.0)
    for i in range(n_layers):
        gen.fill(k_out[i], begin + i, 0, 0, nk.NKV_BF16)
        gen.fill(v_out[i], begin + i, 0, 1, nk.NKV_BF16)
    for _ in range(prefill):
        bank.commit_tensors(desc(seg), k_out, v_out)
        seg += 1

    def timed(fn, n):
        for _ in range(warmup):
            fn(seg % 2)
        _barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn(seg % 2)
        b.record(stream)
        torch.cuda.synchronize()
        return _max_over_ranks(world, dev, [a.elapsed_time(b)])[0]

    clocks = ClockSampler(int(dev.index or 0))
    clocks.start()
    ms_fused = timed(fused, steps)
    clk = clocks.stop()
    # per-launch device time of the producer kernel (separate, event-bracketed turns)
    for _ in range(2):
        fused(seg % 2, time_launches=True)
    launch_ms = proj_ms[0] / proj_ms[1]
    ms_unfused = timed(unfused, steps)
    # cuBLAS alone on the same GEMM (x [L, 3072] x [3072, 6144])
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(n_layers):
        torch.matmul(xs[0][i], wkv[i].T)
    a.record(stream)
    reps = 3
    for r in range(reps):
        for i in range(n_layers):
            torch.matmul(xs[r % 2][i], wkv[i].T)
    b.record(stream)
    torch.cuda.synchronize()
    cublas_ms = a.elapsed_time(b) / (reps * n_layers)

    e2e = None
    if e2e_steps:
        # e2e: the attention inputs come from pinned host memory every turn
        host_x = [[t.cpu().pin_memory() for t in xs[s]] for s in range(2)]
        _barrier(world)
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record(stream)
        for st in range(e2e_steps):
            for i in range(n_layers):
                xs[st % 2][i].copy_(host_x[st % 2][i], non_blocking=True)
            fused(st % 2)  # returns after reading the layers' non-finite flags back
        eb.record(stream)
        torch.cuda.synchronize()
        e2e_ms = _max_over_ranks(world, dev, [ea.elapsed_time(eb)])[0]
        e2e = {"value": round(SEG_TOKENS * e2e_steps / (e2e_ms / 1e3), 1), "unit": "segment tokens/s (all layers)",
               "h2d_bytes_per_step": SEG_TOKENS * DIM * 2 * args.layers,
               "d2h_bytes_per_step": 4 * (n_layers + 1) * world, "steps": e2e_steps,
               "result": "the K / V and the rebuilt working set stay in HBM; the device-to-host read per turn is "
                         "the layers' non-finite status words"}

    cpu_line = None
    if cpu and rank == 0 and world == 1:
        try:
            cpu_line = cpu_sample_project(min(os.cpu_count() or 1, LAYERS))
        except Exception as e:  # noqa: BLE001
            cpu_line = {"value": None, "unit": "segment tokens/s (all layers)", "cores": 0, "kind": "port",
                        "sample": f"failed: {e}"}
    bank.close()
    del xs, wk, wv, wkv
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    tflops = PROJECT_FLOPS / (launch_ms / 1e3) / 1e12
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        t = json.load(open(tp)).get("project_kv_project")
        if t:
            traffic = int(t["dram_bytes"] / t["layers"])
    cublas_tflops = PROJECT_FLOPS / (cublas_ms / 1e3) / 1e12
    return {
        "metric": METRIC_PROJECT, "value": round(SEG_TOKENS * steps / (ms_fused / 1e3), 1),
        "unit": "segment tokens/s (all layers)", "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms_fused / steps, 4),
        "unfused": {"ms_per_step": round(ms_unfused / steps, 4),
                    "what": "cuBLAS projection (torch.matmul) + eager bias / RmsNorm / RoPE + commit_tensors",
                    "speedup_fused": round(ms_unfused / ms_fused, 3)},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4), "traffic": traffic,
                     "kernel": "k_kv_project (one launch per layer)", "flops_per_launch": PROJECT_FLOPS,
                     "launch_ms": round(launch_ms, 4), "peak_src": peaks["src"] + " (burst cuBLAS bf16)",
                     "cublas_same_gemm_ms": round(cublas_ms, 4), "cublas_same_gemm_tflops": round(cublas_tflops, 1)},
        "e2e": e2e, "gpu_launches": steps * (n_layers + 3), "clocks": clk, "cpu_baseline": cpu_line,
    }


def run_project(args) -> None:
    import torch.distributed as dist

    world, rank, local, dev = _dist_setup(args)
    peaks = load_peaks()
    r = project_measure(args, world, rank, dev, peaks, steps=args.steps, warmup=args.warmup, e2e_steps=2,
                        cpu=not args.no_cpu, archived=ARCHIVED)
    if rank == 0:
        out = {"metric": r["metric"], "value": r["value"], "unit": r["unit"], "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
               "config": {"workload": "nomas-8B commit with its producer: per layer the K / V projection of a "
                                      "6,496-token segment (Lin + bias, RmsNorm + RoPE on K) with INT8 archive rows "
                                      "in the epilogue, staged commit, uniform rebuild (16 past frames), newest "
                                      "segment", "layers": args.layers, "heads": HEADS, "head_dim": HEAD_DIM,
                          "model_dim": DIM, "segment_tokens": SEG_TOKENS, "parallelism": f"layer-sharded x{world}",
                          "l2": "attention inputs 1.9 GB per step > 126 MB L2"},
               "unfused": r["unfused"], "roofline": r["roofline"], "e2e": r["e2e"],
               "gpu_launches": r["gpu_launches"], "clocks": r["clocks"], "cpu_baseline": r["cpu_baseline"]}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = min(os.cpu_count() or 1, LAYERS)
    wl, swap = args.workload, args.swap
    if wl == "project":
        r = cpu_sample_project(threads)
        out = {"impl": "reference", "metric": METRIC_PROJECT, "value": round(r["value"], 3), "unit": r["unit"],
               "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
               "config": {"workload": "producer chain + quantize (oracle restatement)", "layers_sampled": threads},
               "cpu_baseline": r, "e2e": {"value": round(r["value"], 3), "unit": r["unit"], "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}
        print(json.dumps(out), flush=True)
        return
    r = cpu_sample(threads, warmup=max(0, min(args.warmup, 1)), steps=max(1, min(args.steps, 2)), workload=wl,
                   swap=swap)
    metric = METRIC_SWAP.format(wl.upper()) if swap else METRIC if wl == "int8" else METRIC_QVG
    out = {"impl": "reference", "metric": metric, "value": round(r["value"], 3), "unit": "GB/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": WORKLOADS[wl] + (" + park/unpark (phase swap) every turn" if swap else ""),
                      "layers_sampled": threads},
           "cpu_baseline": r, "e2e": {"value": round(r["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-extras", action="store_true",
                    help="INT8 line only: skip the QVG turn, the park + unpark and the producer turn")
    ap.add_argument("--workload", default="int8", choices=["int8", "qvg", "project"],
                    help="int8 = the headline configuration; qvg = the QVG configuration (frozen codebooks); "
                         "project = the commit with its fused K/V projection producer")
    ap.add_argument("--swap", action="store_true",
                    help="box-run configuration: phase-swapped cache, park + unpark every turn, 64-segment archive")
    ap.add_argument("--archive-device-gb", type=float, default=0.0,
                    help="tiered archive: keep at most this many GB of archive slabs in device memory (0: no limit)")
    ap.add_argument("--verify", default="broadcast", choices=["broadcast", "strict", "off"],
                    help="ShardedKvBank turn-record verification across ranks (N > 1)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="model layers (48 = the 8B geometry; fewer only for small profiling cases)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "project":
        run_project(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
