"""Drive the same cache session through the CPU oracle and the GPU bank and
compare every observable after every operation: status and message, layer
info, layouts, metrics (bank and per layer), working sets (bitwise), and the
archived payload bytes.

Inputs come from nomas_kv.synth: the GPU side fills device tensors with the
counter-based generator, the oracle side gets the identical bits from its
numpy reproduction.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

import nomas_kv as nk
import oracle as orc
from nomas_kv import synth

DT = {"f32": (nk.NKV_F32, orc.F32), "bf16": (nk.NKV_BF16, orc.BF16), "f16": (nk.NKV_F16, orc.F16)}


@dataclass
class Geometry:
    n_layers: int = 2
    batch: int = 1
    heads: int = 4
    head_dim: int = 32
    tpf: int = 64
    frames: int = 3
    text: int = 16
    model_dtype: str = "f32"
    input_dtype: str = "f32"
    seed: int = 0
    key_sigma: float = 0.5


@dataclass
class Spec:
    storage: int = nk.NKV_STORAGE_INT8
    sampling: int = nk.NKV_SAMPLING_UNIFORM
    gamma: float = 2.0
    capacity: int | None = None
    past_frames: int = 6
    phase_swap: bool = False
    qvg: nk.QvgConfig = field(default_factory=nk.QvgConfig)

    def product(self) -> nk.CacheConfig:
        st = nk.CacheStorage(self.storage, self.qvg)
        return nk.CacheConfig(storage=st, sampling=nk.HistorySampling(self.sampling, self.gamma),
                              capacity=self.capacity, past_frames=self.past_frames, phase_swap=self.phase_swap)

    def oracle(self) -> orc.Config:
        q = self.qvg
        return orc.Config(storage=self.storage, sampling=self.sampling, gamma=self.gamma, capacity=self.capacity,
                          past_frames=self.past_frames, phase_swap=self.phase_swap, qvg_stages=q.stages,
                          qvg_bits=q.bits_per_stage, qvg_block=q.block_size, qvg_seed=q.codebook_seed)


def _bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a.view(np.uint16) if a.itemsize == 2 else a


def _nan_mask(a: np.ndarray, kind: str) -> np.ndarray:
    b = _bits(a)
    if b.dtype == np.uint32:
        return (b & 0x7FFFFFFF) > 0x7F800000
    if kind == "f16":
        return (b & 0x7FFF) > 0x7C00
    return (b & 0x7FFF) > 0x7F80


def same_values(a: np.ndarray, b: np.ndarray, kind: str = "bf16") -> np.ndarray:
    """Element-wise equality of bit patterns, NaN == NaN whatever the payload
    (x86 and the GPU propagate NaN payloads differently; positions must match)."""
    return (_bits(a) == _bits(b)) | (_nan_mask(a, kind) & _nan_mask(b, kind))


def torch_to_raw(t) -> np.ndarray:
    import torch
    if t.dtype == torch.float32:
        return t.detach().cpu().numpy()
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class Pair:
    """One oracle bank and one GPU bank with the same configuration."""

    def __init__(self, geo: Geometry, spec: Spec, device="cuda:0", host_from_device: bool = False):
        """host_from_device: the oracle's inputs are the device generator's
        tensors copied back (the same bits as synth.host_values, whose
        equality with the device generator is tested on its own), which is
        far faster than the numpy generator at the 8B geometry."""
        import torch
        self.torch = torch
        self.host_from_device = host_from_device
        self.geo, self.spec = geo, spec
        self.mdt_p, self.mdt_o = DT[geo.model_dtype]
        self.idt_p, self.idt_o = DT[geo.input_dtype]
        self.device = torch.device(device)
        self.gen = synth.DeviceGen(self.device, seed=geo.seed, key_sigma=geo.key_sigma)
        self.err_o = self.err_p = None
        try:
            self.o = orc.Bank(spec.oracle(), geo.n_layers, geo.batch, geo.heads, geo.head_dim, self.mdt_o)
        except orc.OracleError as e:
            self.o, self.err_o = None, e
        try:
            self.p = nk.KvBank(spec.product(), geo.n_layers, geo.batch, geo.heads, geo.head_dim, self.mdt_p,
                               device=self.device)
        except nk.NomasError as e:
            self.p, self.err_p = None, e
        self.next_index = 0
        self.next_frame = 0
        self.sizes: list[tuple[int, int]] = []  # (image, text) per archived segment

    # ------------------------------------------------------------ inputs
    def inputs(self, segment: int, L: int, poison=None):
        """Per-layer (k, v) device tensors and host raw arrays.  `poison`
        is a callable(layer, side, host_array) that may edit the host array
        (the device copy is then uploaded from it)."""
        torch = self.torch
        g = self.geo
        tdt = nk.torch_dtype(self.idt_p)
        kd, vd, kh, vh = [], [], [], []
        for layer in range(g.n_layers):
            for side, (dl, hl) in enumerate(((kd, kh), (vd, vh))):
                h = None
                if poison is not None or not self.host_from_device:
                    h = synth.host_values(g.seed, g.key_sigma, g.batch, L, g.heads, g.head_dim, layer, segment,
                                          side, self.idt_p)
                if poison is not None:
                    h = h.copy()
                    poison(layer, side, h)
                    t = torch.from_numpy(h.view(np.int16) if h.dtype == np.uint16 else h).to(self.device)
                    t = t.view(tdt) if h.dtype == np.uint16 else t
                elif self.host_from_device:
                    t = torch.empty((g.batch, L, g.heads, g.head_dim), dtype=tdt, device=self.device)
                    self.gen.fill(t, layer, segment, side, self.idt_p)
                    h = torch_to_raw(t)
                else:
                    t = torch.empty((g.batch, L, g.heads, g.head_dim), dtype=tdt, device=self.device)
                    self.gen.fill(t, layer, segment, side, self.idt_p)
                dl.append(t)
                hl.append(h)
        return kd, vd, kh, vh

    # ------------------------------------------------------------ operations
    def _both(self, fo, fp):
        eo = ep = None
        try:
            fo()
        except orc.OracleError as e:
            eo = e
        try:
            fp()
        except nk.NomasError as e:
            ep = e
        assert (eo is None) == (ep is None), f"oracle error {eo!r} vs product error {ep!r}"
        if eo is not None:
            assert eo.code == ep.code, (eo.code, ep.code, eo.msg, ep.msg)
            assert eo.msg == ep.msg, (eo.msg, ep.msg)
        return eo

    def commit(self, frames=None, text=None, action_start=-1, segment_index=None, frame_start=None, poison=None,
               image_tokens=None):
        g = self.geo
        frames = g.frames if frames is None else frames
        text = g.text if text is None else text
        image = frames * g.tpf if image_tokens is None else image_tokens
        si = self.next_index if segment_index is None else segment_index
        fs = self.next_frame if frame_start is None else frame_start
        L = image + text
        kd, vd, kh, vh = self.inputs(si, L, poison)
        seg = dict(segment_index=si, frame_start=fs, frame_count=frames, image_tokens=image, text_tokens=text,
                   action_start=action_start)
        desc = nk._abi.nkv_segment_desc(si, fs, frames, image, text, action_start)
        err = self._both(lambda: self.o.commit(seg, self.idt_o, kh, vh),
                         lambda: self.p.commit_tensors(desc, kd, vd))
        if err is None or err.code == orc.ERR_GEOMETRY and "capacity" in err.msg:
            # a rebuild over capacity still archived the segment (history.rs:416-421)
            self.next_index = si + 1
            self.next_frame = fs + frames
            self.sizes.append((image, text))
        return err

    def rollback(self):
        n_before = self.o.info(0)["n_segments"]
        err = self._both(self.o.rollback, self.p.rollback)
        if self.o.info(0)["n_segments"] < n_before:
            self.sizes.pop()
            self.next_frame = self.o.info(0)["total_frames"]
        return err

    def park(self):
        return self._both(self.o.park, self.p.park_all)

    def unpark(self):
        return self._both(self.o.unpark, self.p.unpark_all)

    def set_codebooks(self, cb_per_layer):
        for layer, cb in enumerate(cb_per_layer):
            self.o.set_codebooks(layer, cb)
            self.p.layer(layer).set_qvg_codebooks(cb)

    # ------------------------------------------------------------ checks
    def check(self, working_sets=True, archive=True):
        g = self.geo
        assert self.o.metrics() == self.p.metrics().as_dict(), (self.o.metrics(), self.p.metrics())
        for layer in range(g.n_layers):
            lp = self.p.layer(layer)
            io = self.o.info(layer)
            assert io["valid_len"] == lp.valid_len()
            assert io["capacity"] == lp.capacity()
            assert io["n_segments"] == lp.n_segments()
            assert io["total_frames"] == lp.total_frames()
            assert io["tokens_per_frame"] == lp.tokens_per_frame()
            assert bool(io["parked"]) == lp.is_parked()
            assert self.o.layer_metrics(layer) == lp.metrics().as_dict()
            assert self.o.layout(layer) == [x.as_tuple() for x in lp.working_layout()]
            if working_sets and not io["parked"]:
                ko, vo = self.o.working_set(layer)
                kp, vp = lp.working_set()
                kp, vp = torch_to_raw(kp), torch_to_raw(vp)
                assert kp.shape == ko.shape and vp.shape == vo.shape
                for a, b, name in ((ko, kp, "k"), (vo, vp, "v")):
                    eq = same_values(a, b, self.geo.model_dtype)
                    if not eq.all():
                        bad = np.argwhere(~eq)
                        raise AssertionError(f"layer {layer} working-set {name} differs at {len(bad)} places, "
                                             f"first {bad[:3].tolist()}")
            if archive:
                self.check_archive(layer)
            if self.spec.storage == nk.NKV_STORAGE_QVG:
                cbo, cbp = self.o.codebooks(layer), lp.qvg_codebooks()
                assert (cbo is None) == (cbp is None), f"layer {layer} fitted state differs"
                if cbo is not None:
                    # bitwise, NaN entries by position (payloads are platform-specific)
                    assert same_values(cbo, cbp, "f32").all(), f"layer {layer} codebooks"

    def check_archive(self, layer):
        g = self.geo
        n = self.o.info(layer)["n_segments"]
        sp = self.spec
        for pos in range(n):
            blob = np.asarray(self.p.layer(layer).export_segment(pos))
            # geometry of this segment from the oracle's layouts is not kept:
            # recompute from the committed descriptors
            L_total = blob.size
            if sp.storage == nk.NKV_STORAGE_INT8:
                B, H, D = g.batch, g.heads, g.head_dim
                L = L_total // (2 * B * H * D + 8 * B * H)
                kq, vq, ks, vs = self.o.archive_int8(layer, pos, L)
                ref = np.concatenate([kq.ravel(), vq.ravel(), ks.view(np.uint8).ravel(), vs.view(np.uint8).ravel()])
                assert np.array_equal(ref, blob), f"layer {layer} segment {pos} int8 payload differs"
            elif sp.storage == nk.NKV_STORAGE_QVG:
                self._check_qvg_archive(layer, pos, blob)

    def _check_qvg_archive(self, layer, pos, blob):
        g, q = self.geo, self.spec.qvg
        image, text = self.sizes[pos]
        kc, vc, ksc, vsc = self.o.archive_qvg(layer, pos, image)
        parts = [kc, vc, ksc.view(np.uint8), vsc.view(np.uint8)]
        if text > 0:
            kq, vq, ks, vs = self.o.archive_int8(layer, pos, text)
            parts += [kq.ravel(), vq.ravel(), ks.view(np.uint8).ravel(), vs.view(np.uint8).ravel()]
        ref = np.concatenate([p.ravel() for p in parts])
        assert ref.size == blob.size, (ref.size, blob.size)
        # codes bytewise; the f32 alphas NaN-equivalent
        nc = kc.size + vc.size
        ns = ksc.size + vsc.size
        assert np.array_equal(ref[:nc], blob[:nc]), f"layer {layer} segment {pos} qvg codes differ"
        assert same_values(ref[nc:nc + 4 * ns].view(np.float32), blob[nc:nc + 4 * ns].copy().view(np.float32)).all()
        assert np.array_equal(ref[nc + 4 * ns:], blob[nc + 4 * ns:]), f"layer {layer} segment {pos} text differs"

    def close(self):
        if self.p is not None:
            self.p.close()
        if self.o is not None:
            self.o.close()
