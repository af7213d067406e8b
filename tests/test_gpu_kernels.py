"""GPU parity of the standalone kernels (C ABI) against the oracle:
quantize_kv_pair (int8.rs:85-134), dequantize (int8.rs:139-155),
QvgCodec::encode / decode (qvg.rs:173-300).  Bit-exact."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _dev(torch, a: np.ndarray):
    t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()
    return t


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _quantize(nk, torch, k: np.ndarray, v: np.ndarray, dtype: int, offset: int = 0):
    """Run nkv_int8_quantize on device copies (optionally misaligned by
    `offset` elements)."""
    rows = int(np.prod(k.shape[:-1]))
    D = k.shape[-1]
    kd = _dev(torch, np.concatenate([np.zeros(offset, k.dtype), k.ravel()]))
    vd = _dev(torch, np.concatenate([np.zeros(offset, v.dtype), v.ravel()]))
    esz = k.dtype.itemsize
    kq = torch.empty(rows * D, dtype=torch.uint8, device="cuda")
    vq = torch.empty_like(kq)
    ks = torch.empty(rows, dtype=torch.float32, device="cuda")
    vs = torch.empty_like(ks)
    flag = C.c_uint32()
    lib = nk.lib()
    rc = lib.nkv_int8_quantize(C.c_void_p(kd.data_ptr() + offset * esz), C.c_void_p(vd.data_ptr() + offset * esz),
                               dtype, rows, D, _ptr(kq), _ptr(vq), _ptr(ks), _ptr(vs), C.byref(flag), None)
    msg = lib.nkv_last_error().decode() if rc else ""
    return rc, msg, flag.value, kq.cpu().numpy().reshape(k.shape), vq.cpu().numpy().reshape(k.shape), \
        ks.cpu().numpy().reshape(k.shape[:-1]), vs.cpu().numpy().reshape(k.shape[:-1])


def _to_bf16(orc, raw: np.ndarray, dtype: int) -> np.ndarray:
    """Raw buffer of `dtype` -> bf16 bits of its values (round to nearest even)."""
    if dtype == orc.BF16:
        return raw
    vals = raw if dtype == orc.F32 else raw.view(np.float16).astype(np.float32)
    return orc.bf16_bits(vals)


def _as_dtype(orc, x: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == orc.F32:
        return x.astype(np.float32)
    if dtype == orc.BF16:
        return orc.bf16_bits(x)
    return x.astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("dtype", [0, 1, 2])
@pytest.mark.parametrize("shape", [(1, 64, 4, 128), (2, 33, 3, 32), (1, 17, 2, 64), (1, 9, 5, 16), (1, 8, 2, 256),
                                   (1, 13, 3, 24), (1, 6, 2, 8), (1, 5, 1, 7)])
def test_int8_quantize_matches_oracle(orc, nkv, torch, dtype, shape):
    rng = np.random.default_rng(hash((dtype,) + shape) % 2**32)
    x = rng.standard_normal(shape).astype(np.float32) * rng.choice([1e-6, 1.0, 40.0, 1e4])
    x[..., 0, :] *= 0.0  # an all-zero row -> scale 1
    k = _as_dtype(orc, x, dtype)
    v = _as_dtype(orc, x[::-1].copy(), dtype)
    # the kernel casts to BF16 first, like the bank (history.rs:249-250)
    ref = orc.quantize_kv_pair(_to_bf16(orc, k, dtype), _to_bf16(orc, v, dtype), orc.BF16)
    for offset in (0, 1):
        rc, msg, flag, kq, vq, ks, vs = _quantize(nkv, torch, k, v, dtype, offset)
        assert rc == 0, msg
        assert np.array_equal(kq, ref[0]) and np.array_equal(vq, ref[1])
        assert np.array_equal(ks.view(np.uint32), ref[2].view(np.uint32))
        assert np.array_equal(vs.view(np.uint32), ref[3].view(np.uint32))


def test_int8_quantize_half_integer_ties(orc, nkv, torch):
    """Rows whose quotients x / s land exactly on k + 0.5 (the division path
    inside the kernel's tie band)."""
    rows = []
    for peak in (127.0, 63.5, 254.0, 1.0, 3.0):
        row = [peak] + [np.float32(peak / 127.0) * (k + 0.5) for k in range(-60, 67)]
        rows.append(np.array(row[:128], np.float32))
    x = np.stack(rows).reshape(1, len(rows), 1, 128)
    xb = orc.bf16_bits(x)
    ref = orc.quantize_kv_pair(xb, xb, orc.BF16)
    rc, msg, flag, kq, vq, ks, vs = _quantize(nkv, torch, xb, xb, 1)
    assert rc == 0, msg
    assert np.array_equal(kq, ref[0]) and np.array_equal(ks.view(np.uint32), ref[2].view(np.uint32))


def test_int8_quantize_subnormal_and_extreme_rows(orc, nkv, torch):
    vals = np.array([[1e-40, -3e-41, 9.2e-41, 0.0] * 32, [3.3e38, -1e38, 1.0, 0.0] * 32,
                     [1e-38, 2e-38, -1e-38, 5e-39] * 32], np.float32)
    x = orc.bf16_bits(vals.reshape(1, 3, 1, 128))
    ref = orc.quantize_kv_pair(x, x, orc.BF16)
    rc, msg, flag, kq, vq, ks, vs = _quantize(nkv, torch, x, x, 1)
    assert rc == 0, msg
    assert np.array_equal(kq, ref[0]) and np.array_equal(ks.view(np.uint32), ref[2].view(np.uint32))


@pytest.mark.parametrize("bad,where", [(np.nan, "k"), (np.inf, "v"), (-np.inf, "k"), (3.4e38, "v")])
def test_int8_quantize_rejects_non_finite(orc, nkv, torch, bad, where):
    x = np.ones((1, 4, 2, 128), np.float32)
    y = x.copy()
    (x if where == "k" else y)[0, 2, 1, 77] = bad
    rc, msg, flag, *_ = _quantize(nkv, torch, x, y, 0)
    assert rc == 4 and msg == f"cannot quantize non-finite {where} values"
    assert flag == (1 if where == "k" else 2)


@pytest.mark.parametrize("out_dtype", [0, 1, 2])
def test_int8_dequantize_matches_oracle(orc, nkv, torch, out_dtype):
    rng = np.random.default_rng(3)
    q = rng.integers(1, 256, size=(1, 40, 3, 32), dtype=np.uint8)
    s = (rng.random((1, 40, 3)) * 2.0).astype(np.float32)
    ref = orc.dequantize(q, s, 40, out_dtype)
    qd, sd = _dev(torch, q.ravel()), _dev(torch, s.ravel())
    out = torch.empty(q.size, dtype={0: torch.float32, 1: torch.int16, 2: torch.int16}[out_dtype], device="cuda")
    assert nkv.lib().nkv_int8_dequantize(_ptr(qd), _ptr(sd), 120, 32, out_dtype, _ptr(out), None) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    got = got.view(np.uint16) if out_dtype else got
    assert np.array_equal(got.reshape(ref.shape).view(np.uint32 if out_dtype == 0 else np.uint16),
                          ref.view(np.uint32 if out_dtype == 0 else np.uint16))


def _qvg_pair(orc, nkv, torch, x, cb, side, tokens, block=64, in_dtype=0):
    _, L, H, D = x.shape
    stages, E = cb.shape[2], cb.shape[3]
    bits = E.bit_length() - 1
    xf = x if in_dtype == 0 else orc.bf16_to_f32(x)
    codes_r, scales_r = orc.qvg_encode(cb, side, xf, tokens, block)
    cbd = _dev(torch, np.ascontiguousarray(cb))
    xd = _dev(torch, np.ascontiguousarray(x))
    bpt = (stages * bits + 7) // 8
    nb = -(-tokens // block)
    codes = torch.zeros(max(tokens * H * bpt, 1), dtype=torch.uint8, device="cuda")
    scales = torch.zeros(max(H * nb * stages, 1), dtype=torch.float32, device="cuda")
    rc = nkv.lib().nkv_qvg_encode(_ptr(cbd), side, _ptr(xd), in_dtype, L, H, D, tokens, stages, bits, block,
                                  _ptr(codes), _ptr(scales), None)
    assert rc == 0, nkv.lib().nkv_last_error()
    c = codes.cpu().numpy()[: tokens * H * bpt]
    s = scales.cpu().numpy()[: H * nb * stages]
    assert np.array_equal(c, codes_r), f"codes differ at {np.argwhere(c != codes_r)[:5].ravel().tolist()}"
    assert np.array_equal(s.view(np.uint32), scales_r.view(np.uint32))
    out = torch.zeros((1, tokens, H, D), dtype=torch.float32, device="cuda")
    rc = nkv.lib().nkv_qvg_decode(_ptr(cbd), side, _ptr(codes), _ptr(scales), tokens, H, D, stages, bits, block,
                                  _ptr(out), None)
    assert rc == 0
    torch.cuda.synchronize()
    ref = orc.qvg_decode(cb, side, codes_r, scales_r, tokens, block)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("tokens,H,D,stages,bits,block", [
    (128, 2, 16, 4, 2, 64), (200, 3, 32, 4, 2, 64), (97, 2, 128, 4, 2, 64), (64, 1, 24, 2, 3, 32),
    (70, 2, 16, 3, 4, 16), (33, 2, 8, 1, 8, 64), (150, 1, 64, 8, 2, 50)])
def test_qvg_encode_decode_match_oracle_fitted(orc, nkv, torch, tokens, H, D, stages, bits, block):
    k = orc.randn((1, tokens + 5, H, D), 42 + tokens)
    v = orc.randn((1, tokens + 5, H, D), 43 + tokens)
    cb = orc.qvg_fit(k, v, stages=stages, bits=bits)
    for side, x in ((0, k), (1, v)):
        _qvg_pair(orc, nkv, torch, x, cb, side, tokens, block)


def test_qvg_encode_bf16_input_synthetic_codebooks(orc, nkv, torch):
    rng = np.random.default_rng(5)
    H, D = 4, 128
    cb = np.zeros((2, H, 4, 4, D), np.float32)
    for s, sig in enumerate((1.0, 0.5, 0.25, 0.125)):
        cb[:, :, s] = (rng.standard_normal(cb[:, :, s].shape) * sig).astype(np.float32)
    x = orc.bf16_bits(rng.standard_normal((1, 300, H, D)).astype(np.float32) * 2.0)
    _qvg_pair(orc, nkv, torch, x, cb, 1, 290, 64, in_dtype=1)


def test_qvg_ties_and_degenerate_blocks(orc, nkv, torch):
    H, D = 2, 16
    cb = np.zeros((2, H, 4, 4, D), np.float32)
    cb[:, :, :, 2] = 1.0
    cb[:, :, :, 3] = 1.0  # 2 and 3 identical; 0 and 1 identical (zero -> den 0 -> alpha 1)
    x = np.zeros((1, 70, H, D), np.float32)
    x[0, :35] = 1.0
    _qvg_pair(orc, nkv, torch, x, cb, 0, 70)


def test_qvg_d128_fast_path_ties_nan_and_extremes(orc, nkv, torch):
    """head_dim 128 / 2 bits / block 64 takes the screened encoder; duplicate
    codewords force its exact path, NaN rows and extreme magnitudes its
    fallbacks."""
    H, D = 3, 128
    rng = np.random.default_rng(9)
    cb = (rng.standard_normal((2, H, 4, 4, D)) * 0.5).astype(np.float32)
    cb[:, 0, :, 3] = cb[:, 0, :, 1]  # head 0: entries 1 and 3 identical
    cb[:, 1, 2, :] = 0.25  # head 1, stage 2: all four entries identical
    x = rng.standard_normal((1, 200, H, D)).astype(np.float32)
    x[0, 10, 2, 7] = np.nan
    x[0, 70:75, 2] *= 1e30
    x[0, 80:85, 1] *= 1e-30
    x[0, 130:140, 0] = cb[0, 0, 0, 1] + cb[0, 0, 1, 1]  # exactly on codewords
    for side in (0, 1):
        cbs = np.ascontiguousarray(cb)
        _, L, _, _ = x.shape
        codes_r, scales_r = orc.qvg_encode(cbs, side, x, 196)
        cbd = _dev(torch, cbs)
        xd = _dev(torch, np.ascontiguousarray(x))
        codes = torch.zeros(196 * H, dtype=torch.uint8, device="cuda")
        scales = torch.zeros(H * 4 * 4, dtype=torch.float32, device="cuda")
        rc = nkv.lib().nkv_qvg_encode(_ptr(cbd), side, _ptr(xd), 0, L, H, D, 196, 4, 2, 64, _ptr(codes), _ptr(scales),
                                      None)
        assert rc == 0, nkv.lib().nkv_last_error()
        assert np.array_equal(codes.cpu().numpy(), codes_r)
        s = scales.cpu().numpy()
        same = (s.view(np.uint32) == scales_r.view(np.uint32)) | (np.isnan(s) & np.isnan(scales_r))
        assert same.all()


def test_hardware_pair_converters_equal_integer_rounding_off_nan(tmp_path):
    """The no-NaN fast paths convert with the hardware bf16x2 / f16x2
    converters; they must equal the library's integer round-to-nearest-even
    on every non-NaN f32 (all 2^32 patterns, both lanes)."""
    import os
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "convert_check")
    subprocess.run(["nvcc", "-std=c++17", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-fmad=false",
                    "-I", os.path.join(root, "hy-nomas-rs_b200", "csrc"), os.path.join(root, "tests", "cuda",
                                                                                    "convert_check.cu"),
                    "-o", exe], check=True, capture_output=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=120).stdout
    assert out.split() == ["bf16_mismatches", "0", "f16_mismatches", "0"], out
