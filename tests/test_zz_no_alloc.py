"""The allocation-free quantize entry point (nkv_int8_quantize_layers_noalloc).

Some callers cannot call cudaMalloc — a process whose GPU memory belongs to
another allocator or is capped by a fixed budget, or a latency-critical path
that must avoid cudaMalloc's implicit synchronisation.  For them the library
offers a multi-layer INT8 quantize whose job table and flags live in a
library-wide device array instead of per-call allocations.  This file checks
it through the C ABI against the allocating entry point, nkv_int8_quantize,
bit for bit, on two calls in a row (the shared array keeps the previous call's
contents), and that more layers than the array holds are refused.  It runs
alone in a fresh process or after the whole suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _vp(ts):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _reference(nk, torch, k, v, dtype, rows, D):
    """nkv_int8_quantize (the allocating entry point) on one layer."""
    kq = torch.empty(rows * D, dtype=torch.uint8, device="cuda")
    vq = torch.empty_like(kq)
    ks = torch.empty(rows, dtype=torch.float32, device="cuda")
    vs = torch.empty_like(ks)
    flag = C.c_uint32()
    rc = nk.lib().nkv_int8_quantize(C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), dtype, rows, D,
                                    C.c_void_p(kq.data_ptr()), C.c_void_p(vq.data_ptr()),
                                    C.c_void_p(ks.data_ptr()), C.c_void_p(vs.data_ptr()), C.byref(flag), None)
    assert rc == 0, nk.lib().nkv_last_error()
    return kq, vq, ks, vs


def _call(nk, ks_in, vs_in, dtype, rows, D, outs):
    n = len(ks_in)
    flags = (C.c_uint32 * n)()
    kq, vq, ks, vs = outs
    rc = nk.lib().nkv_int8_quantize_layers_noalloc(_vp(ks_in), _vp(vs_in), n, dtype, rows, D, _vp(kq), _vp(vq),
                                                   _vp(ks), _vp(vs), flags, None)
    return rc, list(flags)


def _check_against_allocating(nk, torch, gen, cases, n_layers, L, H, D):
    """Runs the no-alloc entry point on each (dtype code, torch dtype) case in
    turn, reusing the same outputs, and compares every call with
    nkv_int8_quantize layer by layer."""
    rows = L * H
    outs = ([torch.empty(rows * D, dtype=torch.uint8, device="cuda") for _ in range(n_layers)],
            [torch.empty(rows * D, dtype=torch.uint8, device="cuda") for _ in range(n_layers)],
            [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(n_layers)],
            [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(n_layers)])
    for call, (dtype, tdt) in enumerate(cases):
        ks = [gen.fill(torch.empty((1, L, H, D), dtype=tdt, device="cuda"), layer, call, 0, dtype)
              for layer in range(n_layers)]
        vs = [gen.fill(torch.empty((1, L, H, D), dtype=tdt, device="cuda"), layer, call, 1, dtype)
              for layer in range(n_layers)]
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc, flags = _call(nk, ks, vs, dtype, rows, D, outs)
        free_after = torch.cuda.mem_get_info()[0]
        assert rc == 0, nk.lib().nkv_last_error()
        assert flags == [0] * n_layers
        # the call itself allocated nothing on the device
        assert free_after == free_before, (free_before, free_after)
        for i in range(n_layers):
            ref = _reference(nk, torch, ks[i], vs[i], dtype, rows, D)
            for got, want in zip((outs[0][i], outs[1][i], outs[2][i], outs[3][i]), ref):
                g = got.cpu().numpy()
                w = want.cpu().numpy()
                assert np.array_equal(g.view(np.uint8), w.view(np.uint8)), f"call {call} layer {i} differs"


def test_noalloc_quantize_matches_allocating_entry_point_twice():
    torch = pytest.importorskip("torch")
    import nomas_kv as nk
    from nomas_kv import synth

    assert torch.cuda.is_available(), "needs a CUDA device"
    gen = synth.DeviceGen(torch.device("cuda", 0), seed=5, key_sigma=1.0)
    # one warm-up call so the library's module and the array are resident
    # before the free-memory comparison
    _check_against_allocating(nk, torch, gen, [(nk.NKV_BF16, torch.bfloat16)], 1, 16, 4, 128)
    _check_against_allocating(nk, torch, gen, [(nk.NKV_BF16, torch.bfloat16), (nk.NKV_F32, torch.float32),
                                               (nk.NKV_F16, torch.float16)], 3, 1000, 4, 128)


def test_noalloc_quantize_generic_head_dim_twice():
    """head_dim 96 goes through the generic (non-vectorised) quantize kernel."""
    torch = pytest.importorskip("torch")
    import nomas_kv as nk
    from nomas_kv import synth

    gen = synth.DeviceGen(torch.device("cuda", 0), seed=9, key_sigma=1.0)
    _check_against_allocating(nk, torch, gen, [(nk.NKV_BF16, torch.bfloat16), (nk.NKV_F16, torch.float16)],
                              2, 333, 3, 96)


def test_noalloc_quantize_rejects_more_layers_than_its_array_holds():
    torch = pytest.importorskip("torch")
    import nomas_kv as nk

    n = nk._abi.NKV_NOALLOC_MAX_LAYERS + 1
    t = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    o = torch.zeros(16, dtype=torch.uint8, device="cuda")
    f = torch.zeros(1, dtype=torch.float32, device="cuda")
    rc, _ = _call(nk, [t] * n, [t] * n, nk.NKV_BF16, 1, 16, ([o] * n, [o] * n, [f] * n, [f] * n))
    assert rc == nk._abi.NKV_ERR_ARGUMENT
    assert "n_layers must be in [1, 64]" in nk.lib().nkv_last_error().decode()


def test_noalloc_quantize_reports_first_failing_layer():
    torch = pytest.importorskip("torch")
    import nomas_kv as nk

    n, rows, D = 2, 8, 128
    ks = [torch.ones(rows * D, dtype=torch.bfloat16, device="cuda") for _ in range(n)]
    vs = [torch.ones(rows * D, dtype=torch.bfloat16, device="cuda") for _ in range(n)]
    vs[1][5] = float("nan")
    outs = ([torch.empty(rows * D, dtype=torch.uint8, device="cuda") for _ in range(n)],
            [torch.empty(rows * D, dtype=torch.uint8, device="cuda") for _ in range(n)],
            [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(n)],
            [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(n)])
    rc, flags = _call(nk, ks, vs, nk.NKV_BF16, rows, D, outs)
    assert rc == nk._abi.NKV_ERR_MSG and flags == [0, 2]
    assert nk.lib().nkv_last_error().decode() == "cannot quantize non-finite v values"
    # the next call starts from cleared flags
    vs[1][5] = 1.0
    rc, flags = _call(nk, ks, vs, nk.NKV_BF16, rows, D, outs)
    assert rc == 0 and flags == [0, 0]
