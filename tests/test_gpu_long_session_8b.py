"""Config 4: the long-session rebuild stress at the 8B geometry.

Six layers (one rank's share of 48 layers on 8 GPUs) of 24 heads x 128,
INT8, segments of 4 frames x 1,560 tokens + 256 text tokens, 256 archived
segments (1,024 frames, 63 GB of archive on the device), under
TemporalContext(0.9) and RecentMixUniform with 32 past frames (with 8
interactive rollbacks of 1-4 segments each, re-committed with new content)
and under Recent with a capacity that evicts whole records, video blocks
and head frames (frame-aligned SWA eviction, cache/swa.rs:52-130).

Two checks, both against the oracle:

* after every commit and rollback, the bank's layouts, valid length and
  counters equal those of an oracle bank run in lockstep on the same segment
  descriptors at a tiny head geometry (the sampled frame indices and the trim
  plan depend only on the frame timeline: uniform_history.rs:10-125,
  history.rs:341-446, swa.rs:52-130);
* at checkpoints, a sampled layer's whole working set equals, row for row,
  the oracle's quantize_kv_pair + dequantize (int8.rs:65-155) of exactly the
  source tokens the layout names (quantization is per (token, head) row, so
  this equals the reference's decode of the whole segment followed by
  index_select).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H8, D8, TPF, FRAMES, TEXT = 24, 128, 1560, 4, 256
SEG = FRAMES * TPF + TEXT
LAYERS = 6
SEGMENTS = 256
PAST = 32


class Session:
    def __init__(self, orc, nk, sampling, gamma=2.0, capacity=None):
        import torch
        from nomas_kv import synth
        self.orc, self.nk, self.torch = orc, nk, torch
        self.sampling, self.gamma = sampling, gamma
        cfg = nk.CacheConfig(storage=nk.CacheStorage.int8(), sampling=nk.HistorySampling(sampling, gamma),
                             capacity=capacity, past_frames=PAST)
        self.bank = nk.KvBank(cfg, LAYERS, 1, H8, D8, torch.bfloat16, device="cuda:0")
        self.bank.reserve(self.bank.segment_bytes(self.desc(0, 0)) * LAYERS * (SEGMENTS + 2), 0)
        ocfg = orc.Config(storage=orc.INT8, sampling=sampling, gamma=gamma, capacity=capacity, past_frames=PAST)
        self.tiny = orc.Bank(ocfg, 1, 1, 1, 8, orc.BF16)
        self.tiny_kv = np.zeros((1, SEG, 1, 8), np.uint16)
        self.gen = synth.DeviceGen(torch.device("cuda", 0), seed=0, key_sigma=1.0)
        self.k = [torch.empty((1, SEG, H8, D8), dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
        self.v = [torch.empty_like(t) for t in self.k]
        self.key = {}  # segment_index -> the generator key of its committed content
        self.next_key = 0
        self.n = 0  # segments in the archive

    def desc(self, i, frame_start):
        return self.nk._abi.nkv_segment_desc(i, frame_start, FRAMES, FRAMES * TPF, TEXT, 0)

    def commit(self):
        i, key = self.n, self.next_key
        self.next_key += 1
        for layer in range(LAYERS):
            self.gen.fill(self.k[layer], layer, key, 0, self.nk.NKV_BF16)
            self.gen.fill(self.v[layer], layer, key, 1, self.nk.NKV_BF16)
        self.bank.commit_tensors(self.desc(i, i * FRAMES), self.k, self.v)
        self.tiny.commit(dict(segment_index=i, frame_start=i * FRAMES, frame_count=FRAMES,
                              image_tokens=FRAMES * TPF, text_tokens=TEXT, action_start=0),
                         self.orc.BF16, [self.tiny_kv], [self.tiny_kv])
        self.key[i] = key
        self.n += 1

    def rollback(self):
        self.bank.rollback()
        self.tiny.rollback()
        self.n -= 1
        del self.key[self.n]

    def check_layout(self):
        lay = self.bank.layer(0)
        got = [x.as_tuple() for x in lay.working_layout()]
        want = self.tiny.layout(0)
        assert got == want, (self.n, got[:4], want[:4])
        for layer in range(1, LAYERS):
            assert [x.as_tuple() for x in self.bank.layer(layer).working_layout()] == want
        info = self.tiny.info(0)
        assert lay.valid_len() == info["valid_len"]
        assert lay.total_frames() == info["total_frames"] and lay.n_segments() == info["n_segments"]
        m, mo = lay.metrics().as_dict(), self.tiny.layer_metrics(0)
        for f in ("archived_segments", "rebuilds", "evicted_tokens", "rollbacks", "encode_calls"):
            assert m[f] == mo[f], (f, m[f], mo[f])

    def source_frames(self, seg_index, n_video_tokens):
        """Frames of segment seg_index the rebuild selected: the sampler's
        frame ids inside the segment, or in Recent mode the first ones (the
        reference keeps frames 0..kept of a trimmed record, history.rs:350-358)."""
        if self.sampling == self.orc.RECENT:
            return list(range(n_video_tokens // TPF))
        total = self.tiny.info(0)["total_frames"]
        ids = self.orc.frame_indices("history", total, PAST, self.sampling, self.gamma)
        fs = seg_index * FRAMES
        return [f - fs for f in ids if fs <= f < fs + FRAMES]

    def check_working_set(self, layer):
        torch = self.torch
        kw, vw = self.bank.layer(layer).working_set()
        sk = torch.empty((1, SEG, H8, D8), dtype=torch.bfloat16, device="cuda")
        sv = torch.empty_like(sk)
        for (si, vs, ve, ts, te, _) in self.tiny.layout(0):
            frames = self.source_frames(si, ve - vs)
            assert len(frames) * TPF == ve - vs, (si, frames, vs, ve)
            rows = [f * TPF + t for f in frames for t in range(TPF)] + list(range(FRAMES * TPF, FRAMES * TPF + te - ts))
            self.gen.fill(sk, layer, self.key[si], 0, self.nk.NKV_BF16)
            self.gen.fill(sv, layer, self.key[si], 1, self.nk.NKV_BF16)
            idx = torch.tensor(rows, dtype=torch.long, device="cuda")
            kr = sk.index_select(1, idx).view(torch.int16).cpu().numpy().view(np.uint16)
            vr = sv.index_select(1, idx).view(torch.int16).cpu().numpy().view(np.uint16)
            kq, vq, ks, vsc = self.orc.quantize_kv_pair(kr, vr, self.orc.BF16)
            want_k = self.orc.dequantize(kq, ks, len(rows), self.orc.BF16)
            want_v = self.orc.dequantize(vq, vsc, len(rows), self.orc.BF16)
            sel = torch.cat([torch.arange(vs, ve), torch.arange(ts, te)]).to("cuda")
            got_k = kw.index_select(1, sel).view(torch.int16).cpu().numpy().view(np.uint16)
            got_v = vw.index_select(1, sel).view(torch.int16).cpu().numpy().view(np.uint16)
            assert np.array_equal(got_k, want_k), f"layer {layer} segment {si} K differs"
            assert np.array_equal(got_v, want_v), f"layer {layer} segment {si} V differs"

    def close(self):
        self.bank.close()
        self.tiny.close()
        self.torch.cuda.synchronize()
        self.torch.cuda.empty_cache()


# (after this many segments, roll back this many, then commit them again with new content)
ROLLBACKS = [(40, 1), (80, 2), (120, 3), (160, 4), (200, 1), (230, 2), (245, 3), (256, 4)]
CHECKPOINTS = {64, 128, 192}


def _run(orc, nkv, sampling, gamma=2.0):
    s = Session(orc, nkv, sampling, gamma)
    try:
        plan = dict(ROLLBACKS)
        done = set()
        while s.n < SEGMENTS or SEGMENTS not in done:
            s.commit()
            s.check_layout()
            if s.n in CHECKPOINTS:
                s.check_working_set(s.n % LAYERS)
            if s.n in plan and s.n not in done:
                done.add(s.n)
                for _ in range(plan[s.n]):
                    s.rollback()
                    s.check_layout()
                s.check_working_set(0)
        assert s.n == SEGMENTS and s.bank.layer(0).metrics().rollbacks == sum(r for _, r in ROLLBACKS)
        assert s.bank.layer(LAYERS - 1).n_segments() == SEGMENTS
        s.check_working_set(LAYERS - 1)
    finally:
        s.close()


def test_config4_temporal_context_09_with_rollbacks(orc, nkv):
    _run(orc, nkv, orc.TEMPORAL, 0.9)


def test_config4_recent_mix_uniform_with_rollbacks(orc, nkv):
    _run(orc, nkv, orc.RECENT_MIX)


def test_config4_recent_swa_eviction(orc, nkv):
    """Recent mode with a capacity that is not frame-aligned: the trim drops
    whole records, whole video blocks (keeping text) and head frames."""
    cap = 24 * SEG + 3 * TPF // 2 + 77
    s = Session(orc, nkv, orc.RECENT, capacity=cap)
    try:
        partial = 0
        for _ in range(SEGMENTS):
            s.commit()
            s.check_layout()
            partial += any((ve - vs) % (FRAMES * TPF) != 0 for (_, vs, ve, _, _, _) in s.tiny.layout(0))
            if s.n in CHECKPOINTS:
                s.check_working_set(s.n % LAYERS)
        assert s.bank.layer(0).metrics().evicted_tokens > 0 and partial > 0
        assert s.bank.layer(0).valid_len() <= cap
        # Recent mode rejects rollback, like the reference (history.rs:507-512)
        with pytest.raises(nkv.CacheStateError):
            s.bank.rollback()
        with pytest.raises(orc.OracleError):
            s.tiny.rollback()
        s.check_layout()
        s.check_working_set(LAYERS - 1)
    finally:
        s.close()
