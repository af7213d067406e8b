"""CPU checks of the C ABI: the library loads, exports every entry point
declared in include/nomas_kv.h, and validates configurations exactly like
HistoryCache::new (cache/history.rs:104-156) before touching a device."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "nomas_kv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^(?:int|int32_t|const char\s*\*)\s+(nkv_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "nkv_bank_commit" in names and "nkv_cache_working_set" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol(nkv):
    lib = nkv.lib()
    from nomas_kv import _abi
    for name in _declared():
        assert hasattr(lib, name), f"{name} not exported"
        assert name in _abi.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_abi.SIGNATURES) == set(_declared())
    assert lib.nkv_abi_version() == 1


def test_library_is_the_in_tree_build(nkv):
    from nomas_kv import _abi
    assert _abi.LIB_PATH.startswith(os.path.join(ROOT, "hy-nomas-rs_b200"))


def _create(nk, cfg, batch=1, heads=4, head_dim=32, dtype=0, n_layers=2):
    h = C.c_void_p()
    c = cfg.to_c()
    rc = nk.lib().nkv_bank_create(C.byref(c), n_layers, 0, batch, heads, head_dim, dtype, 0, None, C.byref(h))
    return rc, nk.lib().nkv_last_error().decode(), h


@pytest.mark.parametrize("case,code,msg", [
    ("qvg_batch", 3, "QVG storage requires batch=1 (interactive world-model sessions)"),
    ("qvg_bits0", 3, "invalid QVG stages/bits"),
    ("qvg_bits9", 3, "invalid QVG stages/bits"),
    ("qvg_stages0", 3, "invalid QVG stages/bits"),
    ("gamma0", 3, "invalid temporal_context gamma 0"),
    ("gamma_nan", 3, "invalid temporal_context gamma NaN"),
    ("cap0", 3, "cache capacity must be > 0"),
    ("past0", 3, "past_frames must be > 0"),
])
def test_config_validation_matches_reference(nkv, case, code, msg):
    nk = nkv
    q = nk.QvgConfig
    cfg = {
        "qvg_batch": nk.CacheConfig(storage=nk.CacheStorage.qvg_()),
        "qvg_bits0": nk.CacheConfig(storage=nk.CacheStorage.qvg_(q(bits_per_stage=0))),
        "qvg_bits9": nk.CacheConfig(storage=nk.CacheStorage.qvg_(q(bits_per_stage=9))),
        "qvg_stages0": nk.CacheConfig(storage=nk.CacheStorage.qvg_(q(stages=0))),
        "gamma0": nk.CacheConfig(sampling=nk.HistorySampling.temporal_context(0.0)),
        "gamma_nan": nk.CacheConfig(sampling=nk.HistorySampling.temporal_context(float("nan"))),
        "cap0": nk.CacheConfig(capacity=0),
        "past0": nk.CacheConfig(past_frames=0),
    }[case]
    rc, err, h = _create(nk, cfg, batch=2 if case == "qvg_batch" else 1)
    assert rc == code and err == msg and not h.value


def test_oracle_config_validation_messages_agree(orc, nkv):
    nk = nkv
    pairs = [
        (orc.Config(storage=orc.QVG), nk.CacheConfig(storage=nk.CacheStorage.qvg_()), 2),
        (orc.Config(capacity=0), nk.CacheConfig(capacity=0), 1),
        (orc.Config(past_frames=0), nk.CacheConfig(past_frames=0), 1),
        (orc.Config(sampling=orc.TEMPORAL, gamma=-1.0),
         nk.CacheConfig(sampling=nk.HistorySampling.temporal_context(-1.0)), 1),
    ]
    for oc, pc, batch in pairs:
        with pytest.raises(orc.OracleError) as e:
            orc.Bank(oc, 2, batch, 4, 32, orc.F32)
        rc, err, _ = _create(nk, pc, batch=batch)
        assert rc == e.value.code and err == e.value.msg


def test_null_arguments_are_rejected(nkv):
    lib = nkv.lib()
    assert lib.nkv_bank_commit(None, None, 0, None, None) == 6
    assert lib.nkv_bank_rollback(None) == 6
    assert lib.nkv_bank_destroy(None) == 0


def test_bank_without_gpu_fails_loudly(nkv):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc, err, h = _create(nkv, nkv.CacheConfig(storage=nkv.CacheStorage.int8()))
    assert rc == 5 and "no CUDA device" in err and not h.value


def test_partition_layers():
    import nomas_kv as nk
    assert [nk.partition_layers(48, 8, r) for r in range(8)] == [(6 * r, 6) for r in range(8)]
    assert [nk.partition_layers(48, 1, 0)] == [(0, 48)]
    parts = [nk.partition_layers(10, 4, r) for r in range(4)]
    assert parts == [(0, 3), (3, 3), (6, 2), (8, 2)]


def test_synth_generator_is_deterministic():
    from nomas_kv import synth
    a = synth.host_values(0, 0.5, 1, 7, 4, 32, layer=1, segment=2, side=0, dtype=0)
    b = synth.host_values(0, 0.5, 1, 7, 4, 32, layer=1, segment=2, side=0, dtype=0)
    c = synth.host_values(0, 0.5, 1, 7, 4, 32, layer=1, segment=3, side=0, dtype=0)
    assert a.shape == (1, 7, 4, 32) and (a == b).all() and not (a == c).all()
    t = synth.quantile_table()
    assert t.shape == (65536,) and abs(float(t.mean())) < 1e-6 and abs(float(t.std()) - 1.0) < 1e-3


def test_ctypes_structs_match_the_header(nkv, tmp_path):
    """Every struct the ctypes mirror passes across the ABI has the header's
    size and field offsets (compiled with gcc against include/nomas_kv.h)."""
    import ctypes as C
    import shutil
    import subprocess

    from nomas_kv import _abi

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    structs = {n: getattr(_abi, n) for n in ("nkv_qvg_config", "nkv_cache_config", "nkv_segment_desc",
                                             "nkv_segment_layout", "nkv_metrics", "nkv_cache_info_t",
                                             "nkv_kernel_stat", "nkv_staged_layer", "nkv_row_range",
                                             "nkv_kv_project_args")}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "nomas_kv.h"', "int main(void) {"]
    for name, st in structs.items():
        lines.append(f'  printf("{name} %zu\\n", sizeof({name}));')
        for f, _ in st._fields_:
            lines.append(f'  printf("{name}.{f} %zu\\n", offsetof({name}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run(["gcc", "-std=c11", "-I", inc, str(src), "-o", str(exe)], check=True)
    out = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                               check=True).stdout.splitlines())
    for name, st in structs.items():
        assert int(out[name]) == C.sizeof(st), name
        for f, _ in st._fields_:
            assert int(out[f"{name}.{f}"]) == getattr(st, f).offset, f"{name}.{f}"
