"""kd_qkv_projection_noalloc, the entry point for callers that cannot allocate device memory (a plugin host that
owns every allocation and hands the library only inputs and outputs, or a runtime that forbids side allocations on
its devices): it keeps the per-pack rotary scratch in the library's own static device array. Called through the C
ABI, its q, k, v and gate must equal, bit for bit, those of the existing path (kd_rope_gather into a caller buffer,
then kd_qkv_projection) on two calls in a row. The second call has another pack size, and its rows carry other
positions than the first call's rows at the same indices, so a scratch entry left over from the first call could not
pass for a fresh one.

This file is collected last, so a run that stops at the first failure has already run every other test."""

import numpy as np
import pytest
import torch

from karpo_decision_b200 import _lib, ops

DEV = torch.device("cuda")
TABLE_ROWS = 4096


def _case(seed, lengths, offset):
    g = np.random.default_rng(seed)
    t = int(sum(lengths))
    hq, hkv, hd, hidden = 4, 2, 128, 256
    width = hq * hd * 2 + 2 * hkv * hd  # gated queries (Qwen3.5 layout)
    x = torch.from_numpy(g.standard_normal((t, hidden)).astype(np.float32)).to(DEV).bfloat16()
    w = torch.from_numpy((g.standard_normal((width, hidden)) * 0.05).astype(np.float32)).to(DEV).bfloat16()
    seqpos = torch.from_numpy(np.concatenate([np.arange(n) + offset for n in lengths])).to(DEV)
    qn = torch.from_numpy((g.standard_normal(hd) * 0.1).astype(np.float32)).to(DEV).bfloat16()
    kn = torch.from_numpy((g.standard_normal(hd) * 0.1).astype(np.float32)).to(DEV).bfloat16()
    inv = (1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))).to(DEV)
    cos, sin = ops.rope_table(inv, TABLE_ROWS)
    return dict(t=t, x=x, w=w, seqpos=seqpos, qn=qn, kn=kn, cos=cos, sin=sin, hq=hq, hkv=hkv, hd=hd, width=width)


def _outputs(c):
    t = c["t"]
    return (torch.empty(t, c["hq"], c["hd"], dtype=torch.bfloat16, device=DEV),
            torch.empty(t, c["hkv"], c["hd"], dtype=torch.bfloat16, device=DEV),
            torch.empty(t, c["hkv"], c["hd"], dtype=torch.bfloat16, device=DEV),
            torch.empty(t, c["hq"] * c["hd"], dtype=torch.bfloat16, device=DEV))


def _noalloc(c):
    q, k, v, gate = _outputs(c)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("kd_qkv_projection_noalloc", c["x"].data_ptr(), c["x"].stride(0), c["w"].data_ptr(), c["w"].stride(0),
              c["t"], c["width"], c["x"].shape[1], c["seqpos"].data_ptr(), c["hq"], c["hkv"], c["hd"], 1,
              c["qn"].data_ptr(), c["kn"].data_ptr(), ops.NORM_ONE_PLUS, -1, 1e-6, c["cos"].data_ptr(),
              c["sin"].data_ptr(), TABLE_ROWS, c["hd"], q.data_ptr(), k.data_ptr(), v.data_ptr(), gate.data_ptr(),
              ops.status_word(DEV).data_ptr(), stream)
    return q, k, v, gate


def _existing(c):
    q, k, v, gate = _outputs(c)
    t = c["t"]
    cs = torch.empty(c["hd"] // 2, t, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("kd_rope_gather", c["seqpos"].data_ptr(), t, c["cos"].data_ptr(), c["sin"].data_ptr(), TABLE_ROWS,
              c["hd"], cs.data_ptr(), stream)
    _lib.call("kd_qkv_projection", c["x"].data_ptr(), c["x"].stride(0), c["w"].data_ptr(), c["w"].stride(0), t,
              c["width"], c["x"].shape[1], c["seqpos"].data_ptr(), c["hq"], c["hkv"], c["hd"], 1, c["qn"].data_ptr(),
              c["kn"].data_ptr(), ops.NORM_ONE_PLUS, -1, 1e-6, cs.data_ptr(), c["hd"], q.data_ptr(), k.data_ptr(),
              v.data_ptr(), gate.data_ptr(), ops.status_word(DEV).data_ptr(), stream)
    return q, k, v, gate


@pytest.mark.gpu
@pytest.mark.parametrize("call", [0, 1])
def test_noalloc_matches_existing_entry_point(call):
    # Two calls in a row: the second pack is longer and its positions are shifted against the first one's at the same
    # rows, so the second call only matches if its gather refilled every scratch entry it reads.
    for seed, lengths, offset in ((0, [300, 400], 0), (1, [1000, 17, 483], 37)):
        c = _case(seed + 2 * call, lengths, offset)
        got = _noalloc(c)
        want = _existing(c)
        torch.cuda.synchronize()
        for a, b in zip(got, want, strict=True):
            assert torch.equal(a, b)  # the same kernels on the same inputs: equal to the last bit
        ops.check_status(DEV)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """Rejected before any CUDA call, so this also runs without a GPU."""
    lib = _lib.load()
    t = (4 << 20) // 64 + 1  # one row past 4 Mi entries at rot = 128
    rc = lib.kd_qkv_projection_noalloc(None, 256, None, 256, t, 1536, 256, None, 4, 2, 128, 1, None, None, 2, -1,
                                       1e-6, None, None, TABLE_ROWS, 128, None, None, None, None, None, None)
    assert rc == -1  # KD_ERR_ARGUMENT: rejected before anything is looked up or launched
    assert "static scratch" in _lib.last_error()


def test_noalloc_rejects_a_bad_rotary_width_before_launching():
    """A rotary width the projection refuses (48 is not a multiple of 32) is caught before the gather would run, so
    nothing is launched and the shared array keeps its contents; no CUDA call is made, so this runs without a GPU."""
    lib = _lib.load()
    rc = lib.kd_qkv_projection_noalloc(None, 256, None, 256, 100, 1536, 256, None, 4, 2, 128, 1, None, None, 2, -1,
                                       1e-6, None, None, TABLE_ROWS, 48, None, None, None, None, None, None)
    assert rc == -1
    assert "rotary width" in _lib.last_error()
