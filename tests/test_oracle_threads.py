"""The oracle's worker-thread count (set_threads) changes no result.

The GPU parity tests at the 8B geometry raise it so the checker finishes in
seconds; here the same small INT8 and QVG sessions run sequentially and on
four threads and must agree byte for byte (working sets, layouts, counters,
archived payloads, codebooks).
"""
import numpy as np
import pytest


def _session(orc, storage, threads):
    from nomas_kv import synth
    orc.set_threads(threads)
    try:
        cfg = orc.Config(storage=storage, sampling=orc.UNIFORM, past_frames=5)
        b = orc.Bank(cfg, 2, 1, 3, 32, orc.BF16)
        out = []
        for s in range(5):
            L = 2 * 40 + 7
            ks = [synth.host_values(3, 0.5, 1, L, 3, 32, layer, s, 0, 2) for layer in range(2)]
            vs = [synth.host_values(3, 0.5, 1, L, 3, 32, layer, s, 1, 2) for layer in range(2)]
            b.commit(dict(segment_index=s, frame_start=2 * s, frame_count=2, image_tokens=80, text_tokens=7),
                     orc.BF16, ks, vs, nthreads=2)
            for layer in range(2):
                k, v = b.working_set(layer)
                out += [k.tobytes(), v.tobytes(), repr(b.layout(layer))]
        out.append(repr(b.metrics()))
        for layer in range(2):
            for pos in range(5):
                if storage == orc.INT8:
                    out += [a.tobytes() for a in b.archive_int8(layer, pos, 87)]
                else:
                    out += [a.tobytes() for a in b.archive_qvg(layer, pos, 80)]
            if storage == orc.QVG:
                out.append(b.codebooks(layer).tobytes())
        b.close()
        return out
    finally:
        orc.set_threads(1)


@pytest.mark.parametrize("storage", ["int8", "qvg"])
def test_oracle_results_do_not_depend_on_thread_count(orc, storage):
    st = orc.INT8 if storage == "int8" else orc.QVG
    a = _session(orc, st, 1)
    b = _session(orc, st, 4)
    assert len(a) == len(b)
    for i, (x, y) in enumerate(zip(a, b)):
        assert x == y, f"item {i} differs"
    assert np.frombuffer(a[0], np.uint16).size > 0
