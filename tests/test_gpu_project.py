"""The fused K/V projection + commit producer (nkv_kv_project, tcgen05/TMA on
sm_100a) and the staged commit, against the oracle.

* exact inputs (x and W on small power-of-two grids, every partial sum of
  the product exactly representable): the GEMM is order-independent, so the
  bf16 K / V and the INT8 rows must equal the oracle's bit for bit;
* random inputs: K / V within the f32-accumulation tolerance of the oracle's
  f64 product, and the INT8 rows bit-exact against the oracle's
  quantize_kv_pair (cache/int8.rs:85-134) of the kernel's own K / V;
* the 8B geometry (6,496 tokens, 24 heads): codes bit-exact against the
  device commit quantizer of its own K / V, and oracle rows on a sample;
* non-finite values in and out of the committed ranges;
* the staged commit: a bank fed by the producer equals a bank fed the same
  K / V through nkv_bank_commit, byte for byte.
"""
import ctypes as C

import numpy as np
import pytest

from test_project_oracle import _inputs

pytestmark = pytest.mark.gpu

D = 128
BF16 = 1


def _torch():
    import torch
    return torch


def dev_bf16(bits):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def host_bits(t):
    torch = _torch()
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def run(nkv, a, M, H, bias=True, norm=True, rope=True, ranges=None, code_rows=None, codes=True):
    torch = _torch()
    dim = H * D
    x, wk, wv = dev_bf16(a["x"]), dev_bf16(a["wk"]), dev_bf16(a["wv"])
    bk = dev_bf16(a["bk"]) if bias else None
    bv = dev_bf16(a["bv"]) if bias else None
    gain = dev_bf16(a["gain"])
    tabs = (torch.from_numpy(a["cos"]).cuda(), torch.from_numpy(a["sin"]).cuda()) if rope else None
    k_out = torch.empty((M, dim), dtype=torch.bfloat16, device="cuda")
    v_out = torch.empty_like(k_out)
    rows = code_rows if code_rows is not None else M
    c = None
    if codes:
        c = dict(k_codes=torch.full((rows, dim), 0xAB, dtype=torch.uint8, device="cuda"),
                 v_codes=torch.full((rows, dim), 0xAB, dtype=torch.uint8, device="cuda"),
                 k_scales=torch.full((rows, H), -1.0, dtype=torch.float32, device="cuda"),
                 v_scales=torch.full((rows, H), -1.0, dtype=torch.float32, device="cuda"))
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    nkv.kv_project(x, wk, wv, bk=bk, bv=bv, k_gain=gain, qk_norm=norm, eps=1e-6, rope=tabs, k_out=k_out,
                   v_out=v_out, codes=c, ranges=ranges, status=status)
    torch.cuda.synchronize()
    out = dict(k=host_bits(k_out), v=host_bits(v_out), status=int(status[0].item()) & 0xFFFFFFFF)
    if codes:
        out.update({n: t.cpu().numpy() for n, t in c.items()})
    return out


def oracle_kv(orc, a, bias=True, norm=True, rope=True):
    return orc.kv_project(a["x"], a["wk"], a["wv"], bk=a["bk"] if bias else None, bv=a["bv"] if bias else None,
                          k_gain=a["gain"], qk_norm=norm, eps=1e-6, cos=a["cos"] if rope else None,
                          sin=a["sin"] if rope else None)


def oracle_codes(orc, k_bits, v_bits, H):
    M = k_bits.shape[0]
    kq, vq, ks, vs = orc.quantize_kv_pair(k_bits.reshape(1, M, H, D), v_bits.reshape(1, M, H, D), BF16)
    return kq.reshape(M, H * D), vq.reshape(M, H * D), ks.reshape(M, H), vs.reshape(M, H)


@pytest.mark.parametrize("M,H,opts", [
    (333, 2, (True, True, True)),     # ragged last tile, everything on
    (128, 4, (False, False, False)),  # plain Lin
    (200, 2, (True, False, True)),    # bias + rope, no norm
    (77, 6, (False, True, False)),    # one partial tile, three N tiles per side
])
def test_exact_inputs_bit_exact(nkv, orc, M, H, opts):
    bias, norm, rope = opts
    a = _inputs(orc, M, H, seed=M + H, integer=True)
    got = run(nkv, a, M, H, bias, norm, rope)
    k, v = oracle_kv(orc, a, bias, norm, rope)
    assert got["status"] == 0
    assert np.array_equal(got["k"], k) and np.array_equal(got["v"], v)
    kq, vq, ks, vs = oracle_codes(orc, k, v, H)
    assert np.array_equal(got["k_codes"], kq) and np.array_equal(got["v_codes"], vq)
    assert np.array_equal(got["k_scales"].view(np.uint32), ks.view(np.uint32))
    assert np.array_equal(got["v_scales"].view(np.uint32), vs.view(np.uint32))


def test_row_ranges_map_and_leave_other_rows(nkv, orc):
    M, H = 333, 2
    a = _inputs(orc, M, H, seed=5, integer=True)
    ranges = [(0, 200, 5), (250, 333, 205)]
    got = run(nkv, a, M, H, ranges=ranges, code_rows=300)
    k, v = oracle_kv(orc, a)
    kq, vq, ks, vs = oracle_codes(orc, k, v, H)
    exp_kq = np.full((300, H * D), 0xAB, np.uint8)
    exp_ks = np.full((300, H), -1.0, np.float32)
    exp_kq[5:205], exp_kq[205:288] = kq[0:200], kq[250:333]
    exp_ks[5:205], exp_ks[205:288] = ks[0:200], ks[250:333]
    assert np.array_equal(got["k_codes"], exp_kq)
    assert np.array_equal(got["k_scales"], exp_ks)
    exp_vq = np.full((300, H * D), 0xAB, np.uint8)
    exp_vq[5:205], exp_vq[205:288] = vq[0:200], vq[250:333]
    assert np.array_equal(got["v_codes"], exp_vq)
    assert np.array_equal(got["k"], k)  # the bf16 outputs cover every row


@pytest.mark.parametrize("M,H", [(700, 4), (129, 2)])
def test_random_inputs(nkv, orc, M, H):
    a = _inputs(orc, M, H, seed=99 + M, integer=False)
    got = run(nkv, a, M, H)
    k, v = oracle_kv(orc, a)
    assert got["status"] == 0
    # f32 accumulation on the tensor cores vs the oracle's f64: bf16 results
    # mostly equal; where a rounding flips, the difference is about one bf16
    # unit of the row's O(1) values (a flipped RoPE input moves a nearly
    # cancelling output by that much in absolute terms)
    for g, o in ((got["k"], k), (got["v"], v)):
        gf, of = orc.bf16_to_f32(g), orc.bf16_to_f32(o)
        assert np.mean(g == o) > 0.98
        assert np.max(np.abs(gf - of) / np.maximum(np.abs(of), 1.0)) < 2 ** -5
    # the codes are the quantize of the K / V the kernel wrote: bit-exact
    kq, vq, ks, vs = oracle_codes(orc, got["k"], got["v"], H)
    assert np.array_equal(got["k_codes"], kq) and np.array_equal(got["v_codes"], vq)
    assert np.array_equal(got["k_scales"].view(np.uint32), ks.view(np.uint32))
    assert np.array_equal(got["v_scales"].view(np.uint32), vs.view(np.uint32))


def test_against_torch_fp32_chain(nkv, orc):
    """A plain PyTorch fp32 restatement of the chain, as a loose check."""
    torch = _torch()
    M, H = 256, 2
    a = _inputs(orc, M, H, seed=21)
    got = run(nkv, a, M, H)
    f = lambda b: torch.from_numpy(orc.bf16_to_f32(b)).double()  # noqa: E731
    x, wk, wv, bk, bv, g = (f(a[n]) for n in ("x", "wk", "wv", "bk", "bv", "gain"))
    k = (x @ wk.T + bk).reshape(M, H, D)
    k = k * torch.rsqrt((k * k).mean(-1, keepdim=True) + 1e-6) * g
    c, s = torch.from_numpy(a["cos"]).double()[:, None, :], torch.from_numpy(a["sin"]).double()[:, None, :]
    kr, ki = k[..., 0::2], k[..., 1::2]
    k = torch.stack([kr * c - ki * s, ki * c + kr * s], -1).reshape(M, H * D)
    v = x @ wv.T + bv
    for g_bits, ref in ((got["k"], k), (got["v"], v)):
        gv = torch.from_numpy(orc.bf16_to_f32(g_bits)).double()
        assert torch.allclose(gv, ref, rtol=3e-2, atol=3e-2)


def test_nonfinite_rows(nkv, orc):
    M, H = 160, 2
    a = _inputs(orc, M, H, seed=8, integer=True)
    a["x"] = a["x"].copy()
    a["x"][10, 3] = 0x7F80  # +inf
    got = run(nkv, a, M, H, ranges=[(0, M, 0)])
    assert got["status"] & 3 == 3  # both K and V rows non-finite
    got = run(nkv, a, M, H, ranges=[(11, M, 0)], code_rows=M)
    assert got["status"] == 0  # the bad row is not committed
    got = run(nkv, a, M, H, codes=False)
    assert got["status"] == 0  # no codes, no check


def test_argument_checks(nkv):
    torch = _torch()
    x = torch.zeros((64, 384), dtype=torch.bfloat16, device="cuda")  # H*128 not a multiple of 256
    w = torch.zeros((384, 384), dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    with pytest.raises(nkv.ArgumentError):
        nkv.kv_project(x, w, w, status=st)
    x = torch.zeros((64, 256), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((256, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(nkv.ArgumentError):  # misaligned status word
        nkv.kv_project(x, w, w, status_ptr=st.data_ptr() + 2)
    with pytest.raises(nkv.ArgumentError):  # misaligned input
        nkv.kv_project(x.view(-1)[4:4 + 62 * 256].view(62, 256), w, w, status=st)  # 8-byte offset


def test_8b_geometry_codes_match_commit_quantizer(nkv, orc):
    """6,496 tokens x 24 heads (one segment of one layer): the epilogue's codes
    equal the commit quantizer's codes of the kernel's own K / V, and a row
    sample equals the oracle."""
    torch = _torch()
    M, H = 6496, 24
    dim = H * D
    rng = np.random.default_rng(1)
    b = lambda arr: orc.bf16_bits(np.asarray(arr, np.float32))  # noqa: E731
    a = dict(x=b(rng.standard_normal((M, dim))), wk=b(rng.standard_normal((dim, dim)) / np.sqrt(dim)),
             wv=b(rng.standard_normal((dim, dim)) / np.sqrt(dim)), bk=b(0.1 * rng.standard_normal(dim)),
             bv=b(0.1 * rng.standard_normal(dim)), gain=b(1 + 0.1 * rng.standard_normal(D)))
    ang = rng.uniform(0, 6.3, (M, D // 2)).astype(np.float32)
    a["cos"], a["sin"] = np.cos(ang), np.sin(ang)
    got = run(nkv, a, M, H)
    assert got["status"] == 0
    kq = torch.empty((M, dim), dtype=torch.uint8, device="cuda")
    vq = torch.empty_like(kq)
    ks = torch.empty((M, H), dtype=torch.float32, device="cuda")
    vs = torch.empty_like(ks)
    kb, vb = dev_bf16(got["k"]), dev_bf16(got["v"])
    flag = C.c_uint32()
    assert nkv.lib().nkv_int8_quantize(kb.data_ptr(), vb.data_ptr(), BF16, M * H, D, kq.data_ptr(), vq.data_ptr(),
                                       ks.data_ptr(), vs.data_ptr(), C.byref(flag),
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    assert np.array_equal(got["k_codes"], kq.cpu().numpy()) and np.array_equal(got["v_codes"], vq.cpu().numpy())
    assert np.array_equal(got["k_scales"], ks.cpu().numpy()) and np.array_equal(got["v_scales"], vs.cpu().numpy())
    rows = np.sort(rng.choice(M, 48, replace=False))
    sub = dict(a, x=a["x"][rows], cos=a["cos"][rows], sin=a["sin"][rows])
    k, v = oracle_kv(orc, sub)
    assert np.mean(got["k"][rows] == k) > 0.98 and np.mean(got["v"][rows] == v) > 0.98


# ------------------------------------------------------------ staged commit
def _bank(nkv, n_layers, H):
    cfg = nkv.CacheConfig(storage=nkv.CacheStorage.int8(), sampling=nkv.HistorySampling.uniform(), past_frames=3)
    return nkv.KvBank(cfg, n_layers, 1, H, D, BF16)


def _desc(nkv, i, tpf, frames, text):
    from nomas_kv import _abi
    d = _abi.nkv_segment_desc()
    d.segment_index, d.frame_start, d.frame_count = i, i * frames, frames
    d.image_tokens, d.text_tokens, d.action_start = tpf * frames, text, -1
    return d


def test_staged_commit_equals_tensor_commit(nkv, orc):
    torch = _torch()
    n_layers, H, tpf, frames, text = 2, 2, 64, 2, 16
    L = tpf * frames + text
    produced, fed = _bank(nkv, n_layers, H), _bank(nkv, n_layers, H)
    rng = np.random.default_rng(3)
    b = lambda arr: dev_bf16(orc.bf16_bits(np.asarray(arr, np.float32)))  # noqa: E731
    dim = H * D
    weights = [dict(wk=b(rng.standard_normal((dim, dim)) / 16), wv=b(rng.standard_normal((dim, dim)) / 16),
                    bk=b(0.1 * rng.standard_normal(dim)), bv=b(0.1 * rng.standard_normal(dim)),
                    k_gain=b(1 + 0.1 * rng.standard_normal(D))) for _ in range(n_layers)]
    for seg in range(5):
        xs = [b(rng.standard_normal((L, dim))) for _ in range(n_layers)]
        ang = torch.from_numpy(rng.uniform(0, 6.3, (L, D // 2)).astype(np.float32)).cuda()
        rope = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
        ks = [torch.empty((1, L, H, D), dtype=torch.bfloat16, device="cuda") for _ in range(n_layers)]
        vs = [torch.empty_like(t) for t in ks]
        desc = _desc(nkv, seg, tpf, frames, text)
        produced.commit_projected(desc, xs, weights, rope=rope, k_outs=[t.view(L, dim) for t in ks],
                                  v_outs=[t.view(L, dim) for t in vs])
        fed.commit_tensors(desc, ks, vs)
        torch.cuda.synchronize()
        for i in range(n_layers):
            pk, pv = produced.layer(i).working_set()
            fk, fv = fed.layer(i).working_set()
            assert torch.equal(pk.view(torch.int16), fk.view(torch.int16))
            assert torch.equal(pv.view(torch.int16), fv.view(torch.int16))
            assert [s.as_tuple() for s in produced.layer(i).working_layout()] == \
                [s.as_tuple() for s in fed.layer(i).working_layout()]
            assert np.array_equal(produced.layer(i).export_segment(seg), fed.layer(i).export_segment(seg))
        assert produced.metrics().as_dict() == fed.metrics().as_dict()


def test_staged_commit_rejects_nonfinite_and_guards(nkv, orc):
    torch = _torch()
    n_layers, H, tpf, frames, text = 2, 2, 64, 2, 16
    L = tpf * frames + text
    bank = _bank(nkv, n_layers, H)
    rng = np.random.default_rng(4)
    b = lambda arr: dev_bf16(orc.bf16_bits(np.asarray(arr, np.float32)))  # noqa: E731
    dim = H * D
    weights = [dict(wk=b(rng.standard_normal((dim, dim)) / 16), wv=b(rng.standard_normal((dim, dim)) / 16))
               for _ in range(n_layers)]
    xs = [b(rng.standard_normal((L, dim))) for _ in range(n_layers)]
    bank.commit_projected(_desc(nkv, 0, tpf, frames, text), xs, weights, qk_norm=False)
    k0, v0 = (t.clone() for t in bank.layer(0).working_set())
    m0 = bank.metrics().as_dict()
    bad = [x.clone() for x in xs]
    bad[1][7, 0] = float("inf")
    with pytest.raises(nkv.MsgError, match="non-finite k"):
        bank.commit_projected(_desc(nkv, 1, tpf, frames, text), bad, weights, qk_norm=False)
    k1, v1 = bank.layer(0).working_set()
    assert torch.equal(k0.view(torch.int16), k1.view(torch.int16)) and bank.metrics().as_dict() == m0
    # one staged segment at a time; commit / rollback refused while pending
    staged = bank.stage_segment(_desc(nkv, 1, tpf, frames, text))
    assert len(staged) == n_layers and all(s["status"] for s in staged)
    with pytest.raises(nkv.CacheStateError):
        bank.stage_segment(_desc(nkv, 1, tpf, frames, text))
    with pytest.raises(nkv.CacheStateError):
        bank.rollback()
    bank.discard_staged()
    with pytest.raises(nkv.CacheStateError):
        bank.commit_staged()
    # the bank carries on: the next segment commits normally
    bank.commit_projected(_desc(nkv, 1, tpf, frames, text), xs, weights, qk_norm=False)
    assert bank.layer(0).n_segments() == 2


def test_stage_needs_int8(nkv):
    cfg = nkv.CacheConfig(storage=nkv.CacheStorage.floating(), sampling=nkv.HistorySampling.uniform(), past_frames=3)
    bank = nkv.KvBank(cfg, 1, 1, 2, D, BF16)
    with pytest.raises(nkv.InvalidConfigError):
        bank.stage_segment(_desc(nkv, 0, 64, 2, 16))


def test_chunked_capture_equals_concatenated_commit(nkv, orc):
    """The pipeline's capture (causal_ar.rs:381-420): a segment's video rows
    come from several chunks, its text rows from the last chunk.  Two
    projection calls with row ranges write one staged record; the bank equals
    one fed the concatenated K / V through nkv_bank_commit."""
    torch = _torch()
    H, tpf, text = 2, 64, 16
    dim = H * D
    frames_a, frames_b = 2, 1  # chunk A: 2 frames; chunk B: 1 frame + the text block
    La, Lb = frames_a * tpf + text, frames_b * tpf + text  # every chunk carries its text rows
    L = (frames_a + frames_b) * tpf + text
    produced, fed = _bank(nkv, 1, H), _bank(nkv, 1, H)
    rng = np.random.default_rng(12)
    b = lambda arr: dev_bf16(orc.bf16_bits(np.asarray(arr, np.float32)))  # noqa: E731
    w = dict(wk=b(rng.standard_normal((dim, dim)) / 16), wv=b(rng.standard_normal((dim, dim)) / 16),
             bk=b(0.1 * rng.standard_normal(dim)), bv=b(0.1 * rng.standard_normal(dim)),
             k_gain=b(1 + 0.1 * rng.standard_normal(D)))
    for seg in range(3):
        xa, xb = b(rng.standard_normal((La, dim))), b(rng.standard_normal((Lb, dim)))
        ang = rng.uniform(0, 6.3, (La + Lb, D // 2)).astype(np.float32)
        cos = torch.from_numpy(np.cos(ang)).cuda()
        sin = torch.from_numpy(np.sin(ang)).cuda()
        ka, va = (torch.empty((La, dim), dtype=torch.bfloat16, device="cuda") for _ in range(2))
        kb, vb = (torch.empty((Lb, dim), dtype=torch.bfloat16, device="cuda") for _ in range(2))
        d = _abi_desc(seg, tpf, frames_a + frames_b, text)
        staged = produced.stage_segment(d)[0]
        # chunk A: its video rows -> segment rows [0, 2 tpf)
        nkv.kv_project(xa, w["wk"], w["wv"], bk=w["bk"], bv=w["bv"], k_gain=w["k_gain"],
                       rope=(cos[:La].contiguous(), sin[:La].contiguous()), k_out=ka, v_out=va, codes=staged,
                       ranges=[(0, frames_a * tpf, 0)], status_ptr=staged["status"], stream=produced.stream)
        # chunk B: video rows -> [2 tpf, 3 tpf), text rows -> [3 tpf, L)
        nkv.kv_project(xb, w["wk"], w["wv"], bk=w["bk"], bv=w["bv"], k_gain=w["k_gain"],
                       rope=(cos[La:].contiguous(), sin[La:].contiguous()), k_out=kb, v_out=vb, codes=staged,
                       ranges=[(0, frames_b * tpf, frames_a * tpf), (frames_b * tpf, Lb, (frames_a + frames_b) * tpf)],
                       status_ptr=staged["status"], stream=produced.stream)
        produced.commit_staged()
        k_cat = torch.cat([ka[:frames_a * tpf], kb]).view(1, L, H, D).contiguous()
        v_cat = torch.cat([va[:frames_a * tpf], vb]).view(1, L, H, D).contiguous()
        fed.commit_tensors(d, [k_cat], [v_cat])
        torch.cuda.synchronize()
        assert np.array_equal(produced.layer(0).export_segment(seg), fed.layer(0).export_segment(seg))
        pk, pv = produced.layer(0).working_set()
        fk, fv = fed.layer(0).working_set()
        assert torch.equal(pk.view(torch.int16), fk.view(torch.int16))
        assert torch.equal(pv.view(torch.int16), fv.view(torch.int16))
    assert produced.metrics().as_dict() == fed.metrics().as_dict()


def _abi_desc(i, tpf, frames, text):
    from nomas_kv import _abi
    d = _abi.nkv_segment_desc()
    d.segment_index, d.frame_start, d.frame_count = i, i * frames, frames
    d.image_tokens, d.text_tokens, d.action_start = tpf * frames, text, -1
    return d


@pytest.mark.parametrize("mode", ["recent_capacity", "parked"])
def test_staged_commit_other_modes(nkv, orc, mode):
    """Staged commits keep the plain commit's semantics in Recent mode with SWA
    eviction (history.rs:345-360, swa.rs:52-130) and while parked (a commit
    while parked is overwritten by the stale set on unpark,
    phase_swap.rs:42-92): a producer-fed bank and a tensor-fed twin stay equal."""
    torch = _torch()
    H, tpf, frames, text = 2, 64, 2, 16
    L = tpf * frames + text
    dim = H * D
    if mode == "recent_capacity":
        cfg = nkv.CacheConfig(storage=nkv.CacheStorage.int8(), sampling=nkv.HistorySampling.recent(),
                              capacity=3 * L - 40)
    else:
        cfg = nkv.CacheConfig(storage=nkv.CacheStorage.int8(), sampling=nkv.HistorySampling.uniform(),
                              past_frames=3, phase_swap=True)
    produced, fed = (nkv.KvBank(cfg, 1, 1, H, D, BF16) for _ in range(2))
    rng = np.random.default_rng(31)
    b = lambda arr: dev_bf16(orc.bf16_bits(np.asarray(arr, np.float32)))  # noqa: E731
    w = [dict(wk=b(rng.standard_normal((dim, dim)) / 16), wv=b(rng.standard_normal((dim, dim)) / 16),
              bk=b(0.1 * rng.standard_normal(dim)), k_gain=b(1 + 0.1 * rng.standard_normal(D)))]
    for seg in range(6):
        x = [b(rng.standard_normal((L, dim)))]
        ks = [torch.empty((1, L, H, D), dtype=torch.bfloat16, device="cuda")]
        vs = [torch.empty_like(ks[0])]
        d = _abi_desc(seg, tpf, frames, text)
        park = mode == "parked" and seg in (2, 4)
        if park:
            produced.park_all()
            fed.park_all()
        produced.commit_projected(d, x, w, k_outs=[ks[0].view(L, dim)], v_outs=[vs[0].view(L, dim)])
        fed.commit_tensors(d, ks, vs)
        if park:
            produced.unpark_all()
            fed.unpark_all()
        torch.cuda.synchronize()
        pk, pv = produced.layer(0).working_set()
        fk, fv = fed.layer(0).working_set()
        assert torch.equal(pk.view(torch.int16), fk.view(torch.int16))
        assert torch.equal(pv.view(torch.int16), fv.view(torch.int16))
        assert [s.as_tuple() for s in produced.layer(0).working_layout()] == \
            [s.as_tuple() for s in fed.layer(0).working_layout()]
        assert produced.metrics().as_dict() == fed.metrics().as_dict()
    if mode == "recent_capacity":
        assert produced.metrics().evicted_tokens > 0


def test_staged_commit_8b_geometry(nkv, orc):
    """Full size: 24 heads, 6,496-token segments (4 x 1,560 video + 256 text),
    two layers, three segments; the producer-fed bank equals the tensor-fed
    twin byte for byte."""
    torch = _torch()
    n_layers, H, tpf, frames, text = 2, 24, 1560, 4, 256
    L = tpf * frames + text
    dim = H * D
    cfg = nkv.CacheConfig(storage=nkv.CacheStorage.int8(), sampling=nkv.HistorySampling.uniform(), past_frames=16)
    produced, fed = (nkv.KvBank(cfg, n_layers, 1, H, D, BF16) for _ in range(2))
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    rnd = lambda *shape, scale=1.0: (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)  # noqa: E731
    weights = [dict(wk=rnd(dim, dim, scale=dim ** -0.5), wv=rnd(dim, dim, scale=dim ** -0.5), bk=rnd(dim, scale=0.1),
                    bv=rnd(dim, scale=0.1), k_gain=(1 + rnd(D, scale=0.1).float()).to(torch.bfloat16))
               for _ in range(n_layers)]
    ang = torch.arange(L, device="cuda", dtype=torch.float32)[:, None] * \
        torch.pow(torch.tensor(256.0, device="cuda"), -torch.arange(0, D, 2, device="cuda") / D)[None, :]
    rope = (torch.cos(ang).contiguous(), torch.sin(ang).contiguous())
    for seg in range(3):
        xs = [rnd(L, dim) for _ in range(n_layers)]
        ks = [torch.empty((1, L, H, D), dtype=torch.bfloat16, device="cuda") for _ in range(n_layers)]
        vs = [torch.empty_like(t) for t in ks]
        d = _abi_desc(seg, tpf, frames, text)
        produced.commit_projected(d, xs, weights, rope=rope, k_outs=[t.view(L, dim) for t in ks],
                                  v_outs=[t.view(L, dim) for t in vs])
        fed.commit_tensors(d, ks, vs)
        torch.cuda.synchronize()
        for i in range(n_layers):
            assert np.array_equal(produced.layer(i).export_segment(seg), fed.layer(i).export_segment(seg))
            pk, pv = produced.layer(i).working_set()
            fk, fv = fed.layer(i).working_set()
            assert torch.equal(pk.view(torch.int16), fk.view(torch.int16))
            assert torch.equal(pv.view(torch.int16), fv.view(torch.int16))
    assert produced.metrics().as_dict() == fed.metrics().as_dict()
    produced.close()
    fed.close()


def test_kernel_matches_project_golden(nkv, orc):
    """The device producer on the golden fixture's inputs gives the committed
    digests (tests/golden/project_int8.json)."""
    import json
    import os
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "golden"))
    import make_project as mp

    golden = json.load(open(os.path.join(here, "golden", "project_int8.json")))["cases"]
    for case, want in golden.items():
        c = mp.CASES[case]
        a = mp.inputs(orc, c["M"], c["H"], c["seed"])
        got = run(nkv, a, c["M"], c["H"], bias=c["bias"], norm=c["norm"], rope=c["rope"])
        assert got["status"] == 0
        M, H = c["M"], c["H"]
        for name, arr in (("k", got["k"]), ("v", got["v"]), ("kq", got["k_codes"].reshape(1, M, H, D)),
                          ("vq", got["v_codes"].reshape(1, M, H, D)), ("ks", got["k_scales"].reshape(1, M, H)),
                          ("vs", got["v_scales"].reshape(1, M, H))):
            assert mp.digest(arr) == want[name], (case, name)
