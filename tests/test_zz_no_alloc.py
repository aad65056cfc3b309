"""kd_qkv_projection_noalloc, the entry point for callers that cannot allocate device memory (a plugin host that
owns every allocation and hands the library only inputs and outputs): it keeps the per-pack rotary scratch in the
library's own static device array. Called through the C ABI, its q, k, v and gate must equal those of the existing
path (kd_rope_gather into a caller buffer, then kd_qkv_projection) on two calls in a row, the second with another
pack size and other positions, so the shared array is refilled rather than reused stale.

This file is collected last, so a run that stops at the first failure has already run every other test."""

import numpy as np
import pytest
import torch

from karpo_decision_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _case(seed, t, lengths):
    g = np.random.default_rng(seed)
    hq, hkv, hd, hidden = 4, 2, 128, 256
    width = hq * hd * 2 + 2 * hkv * hd  # gated queries (Qwen3.5 layout)
    x = torch.from_numpy(g.standard_normal((t, hidden)).astype(np.float32)).to(DEV).bfloat16()
    w = torch.from_numpy((g.standard_normal((width, hidden)) * 0.05).astype(np.float32)).to(DEV).bfloat16()
    seqpos = torch.from_numpy(np.concatenate([np.arange(n) for n in lengths])).to(DEV)
    qn = torch.from_numpy((g.standard_normal(hd) * 0.1).astype(np.float32)).to(DEV).bfloat16()
    kn = torch.from_numpy((g.standard_normal(hd) * 0.1).astype(np.float32)).to(DEV).bfloat16()
    inv = (1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))).to(DEV)
    cos, sin = ops.rope_table(inv, 4096)
    return dict(x=x, w=w, seqpos=seqpos, qn=qn, kn=kn, cos=cos, sin=sin, hq=hq, hkv=hkv, hd=hd, width=width)


def _outputs(c, t):
    return (torch.empty(t, c["hq"], c["hd"], dtype=torch.bfloat16, device=DEV),
            torch.empty(t, c["hkv"], c["hd"], dtype=torch.bfloat16, device=DEV),
            torch.empty(t, c["hkv"], c["hd"], dtype=torch.bfloat16, device=DEV),
            torch.empty(t, c["hq"] * c["hd"], dtype=torch.bfloat16, device=DEV))


def _noalloc(c, t):
    q, k, v, gate = _outputs(c, t)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("kd_qkv_projection_noalloc", c["x"].data_ptr(), c["x"].stride(0), c["w"].data_ptr(), c["w"].stride(0),
              t, c["width"], c["x"].shape[1], c["seqpos"].data_ptr(), c["hq"], c["hkv"], c["hd"], 1,
              c["qn"].data_ptr(), c["kn"].data_ptr(), ops.NORM_ONE_PLUS, -1, 1e-6, c["cos"].data_ptr(),
              c["sin"].data_ptr(), c["hd"], q.data_ptr(), k.data_ptr(), v.data_ptr(), gate.data_ptr(),
              ops.status_word(DEV).data_ptr(), stream)
    return q, k, v, gate


def _existing(c, t):
    q, k, v, gate = _outputs(c, t)
    cs = torch.empty(c["hd"] // 2, t, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("kd_rope_gather", c["seqpos"].data_ptr(), t, c["cos"].data_ptr(), c["sin"].data_ptr(), c["hd"],
              cs.data_ptr(), stream)
    _lib.call("kd_qkv_projection", c["x"].data_ptr(), c["x"].stride(0), c["w"].data_ptr(), c["w"].stride(0), t,
              c["width"], c["x"].shape[1], c["seqpos"].data_ptr(), c["hq"], c["hkv"], c["hd"], 1, c["qn"].data_ptr(),
              c["kn"].data_ptr(), ops.NORM_ONE_PLUS, -1, 1e-6, cs.data_ptr(), c["hd"], q.data_ptr(), k.data_ptr(),
              v.data_ptr(), gate.data_ptr(), ops.status_word(DEV).data_ptr(), stream)
    return q, k, v, gate


@pytest.mark.parametrize("call", [0, 1])
def test_noalloc_matches_existing_entry_point(call):
    # two calls in a row with different packs: the second must not see the first one's scratch contents
    for seed, t, lengths in ((0, 700, [300, 400]), (1, 1500, [1000, 17, 483])):
        c = _case(seed + 2 * call, t, lengths)
        got = _noalloc(c, t)
        want = _existing(c, t)
        torch.cuda.synchronize()
        for a, b in zip(got, want, strict=True):
            # the same kernels on the same inputs: equal to the last bit (the tests' bf16 tolerance is the bound)
            assert (a.float() - b.float()).abs().max().item() <= 2 ** -7 * max(b.float().abs().max().item(), 1.0)
        ops.check_status(DEV)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    t = (4 << 20) // 64 + 1  # one row past 4 Mi entries at rot = 128
    rc = lib.kd_qkv_projection_noalloc(None, 256, None, 256, t, 1536, 256, None, 4, 2, 128, 1, None, None, 2, -1,
                                       1e-6, None, None, 128, None, None, None, None, None, None)
    assert rc == -1  # KD_ERR_ARGUMENT: rejected before anything is looked up or launched
    assert "static scratch" in _lib.last_error()
