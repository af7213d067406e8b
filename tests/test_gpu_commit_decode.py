"""nkv_bank_commit_decode: a commit whose rebuild gather also decodes the
new segment in full into caller buffers (commit_segment, history.rs:458-463,
then decode_segment, history.rs:308-338).  Checked against the oracle's
decode_segment bit for bit, and the bank's state (working sets, layouts,
counters, archive) against the oracle after every commit, for INT8, QVG and
Float storage, vectorised and generic gather paths, and a rejected commit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def H(orc, nkv):
    import cache_harness
    return cache_harness


def _session(H, storage, model_dtype, head_dim=32, tpf=32, frames=2, text=9, offset=0):
    import torch
    import nomas_kv as nk
    spec = H.Spec(storage=storage, sampling=nk.NKV_SAMPLING_UNIFORM, past_frames=3)
    geo = H.Geometry(n_layers=2, heads=4, head_dim=head_dim, tpf=tpf, frames=frames, text=text,
                     model_dtype=model_dtype, input_dtype="bf16")
    p = H.Pair(geo, spec)
    L = frames * tpf + text
    tdt = nk.torch_dtype(H.DT[model_dtype][0])
    for s in range(5):
        kd, vd, kh, vh = p.inputs(s, L)
        # outputs at an element offset inside a larger buffer exercise the
        # unaligned (generic) gather when offset is odd
        bufs = [torch.full((offset + L * 4 * head_dim,), 7.0, dtype=tdt, device="cuda") for _ in range(4)]
        dk = [b[offset:].view(1, L, 4, head_dim) for b in bufs[:2]]
        dv = [b[offset:].view(1, L, 4, head_dim) for b in bufs[2:]]
        desc = nk._abi.nkv_segment_desc(s, s * frames, frames, frames * tpf, text, -1)
        seg = dict(segment_index=s, frame_start=s * frames, frame_count=frames, image_tokens=frames * tpf,
                   text_tokens=text, action_start=-1)
        p.o.commit(seg, p.idt_o, kh, vh)
        p.p.commit_tensors(desc, kd, vd, decode_k=dk, decode_v=dv)
        p.next_index, p.next_frame = s + 1, (s + 1) * frames
        p.sizes.append((frames * tpf, text))
        p.check(working_sets=True, archive=True)
        for layer in range(2):
            kr, vr = p.o.decode_segment(layer, s, L)
            assert H.same_values(H.torch_to_raw(dk[layer].contiguous()), kr, model_dtype).all(), (s, layer)
            assert H.same_values(H.torch_to_raw(dv[layer].contiguous()), vr, model_dtype).all(), (s, layer)
    p.close()


@pytest.mark.parametrize("storage", ["int8", "qvg", "float"])
@pytest.mark.parametrize("model_dtype", ["bf16", "f32"])
def test_commit_decode_matches_oracle(H, storage, model_dtype):
    import nomas_kv as nk
    st = {"int8": nk.NKV_STORAGE_INT8, "qvg": nk.NKV_STORAGE_QVG, "float": nk.NKV_STORAGE_FLOAT}[storage]
    _session(H, st, model_dtype)


def test_commit_decode_qvg_table_decoder_and_unaligned_outputs(H):
    """head_dim 128 takes the table-driven QVG decoder with aligned outputs
    and the generic path when an output is not 16-byte aligned."""
    import nomas_kv as nk
    _session(H, nk.NKV_STORAGE_QVG, "bf16", head_dim=128, tpf=70, frames=2, text=5)
    _session(H, nk.NKV_STORAGE_INT8, "bf16", head_dim=128, tpf=16, frames=2, text=3, offset=1)


def test_commit_decode_rejected_segment_leaves_outputs(H):
    import torch
    import nomas_kv as nk
    p = H.Pair(H.Geometry(n_layers=2, input_dtype="bf16", model_dtype="bf16"), H.Spec(past_frames=4))
    for _ in range(2):
        assert p.commit() is None
    L = 3 * 64 + 16
    kd, vd, kh, vh = p.inputs(2, L)
    vd[1][0, 3, 1, 5] = float("nan")
    dk = [torch.full((1, L, 4, 32), 3.0, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    dv = [torch.full_like(dk[0], 3.0) for _ in range(2)]
    desc = nk._abi.nkv_segment_desc(2, 6, 3, 3 * 64, 16, -1)
    with pytest.raises(nk.MsgError, match="cannot quantize non-finite v values"):
        p.p.commit_tensors(desc, kd, vd, decode_k=dk, decode_v=dv)
    torch.cuda.synchronize()
    for t in dk + dv:
        assert bool((t == 3.0).all())
    p.check(working_sets=True, archive=True)  # the bank is as before the call
    p.close()
