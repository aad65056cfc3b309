"""Parity at the benchmark configurations' full widths, and attention at their lengths.

Whole forwards: BASELINE configurations 2-5 at full width with their depth cut to 2 (Qwen-shaped) or 6 (Gemma-shaped:
5 sliding layers with the 1,024-token window and 1 global layer) against the reference's own served path (its bf16
backbone; ``--fp8`` for the FP8 cases) on the same seeded weights and packs (tests/golden/, made by
tests/golden/make_golden.py). The north-star bar: readout logits within 2e-2 (max-abs) of the reference and the same
top answer for every readout. The reference's own bf16-against-float32 gap is printed beside it as the noise floor.

Attention at the configurations' shapes: head 256 with the (1023, 0) window over sequences one short of, at and past
the window (config 4's sliding layers), and one 131,072-token sequence at head 128 with config 5's 32/16 heads,
checked on sampled query rows (its query tensor holds 2^29 elements, 1 GiB, so products of row index and row stride
leave the 32-bit range in bytes)."""

import numpy as np
import pytest
import torch

from golden_cases import WIDE, load
from karpo_decision_b200 import Packed, Readout, from_arrays, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("name", WIDE)
def test_full_width_forward_matches_reference(name):
    spec, weights, arrays, expected = load(name)
    model = Packed(spec, weights, DEV, fp8=name.endswith("_fp8"))
    head = Readout(weights["readout"], spec.logit_cap, DEV)
    del weights
    logits = head(model(from_arrays(arrays, DEV))).cpu().numpy()
    torch.cuda.synchronize()
    ops.check_status(DEV)
    want = expected["logits"]
    err = float(np.abs(logits - want).max())
    err32 = float(np.abs(logits - expected["logits_fp32"]).max())
    floor = float(np.abs(want - expected["logits_fp32"]).max())
    print(f"{name}: readout max-abs vs reference {err:.4f}; vs its float32 run {err32:.4f} "
          f"(the reference's own bf16 vs float32: {floor:.4f}); logits up to {np.abs(want).max():.2f}")
    assert np.isfinite(logits).all()
    assert err <= 2e-2
    assert np.array_equal(logits.argmax(-1), want.argmax(-1))


def _reference_rows(q, kf, vf, rows, start, window, scale):
    """float32 attention of query rows ``rows`` of a sequence starting at pack row ``start`` (causal, or the
    (window, 0) sliding window), GQA by head groups; ``kf``/``vf`` are the keys and values in float32."""
    hq, hkv, hd = q.shape[1], kf.shape[1], q.shape[2]
    out = []
    for r in rows.tolist():
        lo = start if window < 0 else max(start, r - window)
        qg = q[r].float().view(hkv, hq // hkv, hd)
        s = torch.einsum("kgd,nkd->kgn", qg, kf[lo:r + 1]) * scale
        p = torch.softmax(s, dim=-1)
        out.append(torch.einsum("kgn,nkd->kgd", p, vf[lo:r + 1]).reshape(hq, hd))
    return torch.stack(out)


@pytest.mark.parametrize("hq,hkv", [(16, 8), (8, 2)])
def test_attention_head256_window_1024_at_the_window_edges(hq, hkv):
    """Config 4's sliding layers: head 256, window (1023, 0), sequences of 700, 1,023, 1,024, 1,025 and 3,000 tokens;
    every query row of the short ones and sampled rows of the long one against float32."""
    g = torch.Generator(device=DEV).manual_seed(40)
    lengths = [700, 1023, 1024, 1025, 3000]
    t, hd, scale = sum(lengths), 256, 256 ** -0.5
    q, k, v = (torch.randn(t, h, hd, generator=g, device=DEV).bfloat16() for h in (hq, hkv, hkv))
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=DEV)
    got = ops.attention_varlen(q, k, v, cu, cu, max(lengths), scale, (1023, 0)).float().view(t, hq, hd)
    starts = cu[:-1].tolist()
    kf, vf = k.float(), v.float()
    worst = 0.0
    for start, n in zip(starts, lengths, strict=True):
        rows = torch.arange(start, start + n, device=DEV)
        if n > 1100:  # the long sequence: rows inside, at and past the first window, and the last ones
            rows = torch.cat([rows[:8], rows[1016:1032], rows[2040:2056], rows[-16:]])
        want = _reference_rows(q, kf, vf, rows, start, 1023, scale)
        worst = max(worst, (got[rows] - want).abs().max().item())
    assert worst <= 2e-2, worst


@pytest.mark.parametrize("window", [-1, 1023])
def test_attention_one_131072_token_sequence(window):
    """Config 5(a): one 131,072-token sequence, 32 query / 16 key-value heads of 128, causal (global layers) and the
    (1023, 0) window (sliding layers); 512 query rows sampled across the whole sequence against float32."""
    g = torch.Generator(device=DEV).manual_seed(41)
    t, hq, hkv, hd = 131072, 32, 16, 128
    scale = hd ** -0.5
    q = torch.randn(t, hq, hd, generator=g, device=DEV).bfloat16()
    k = torch.randn(t, hkv, hd, generator=g, device=DEV).bfloat16()
    v = torch.randn(t, hkv, hd, generator=g, device=DEV).bfloat16()
    cu = torch.tensor([0, t], dtype=torch.int32, device=DEV)
    got = ops.attention_varlen(q, k, v, cu, cu, t, scale, (window, 0)).view(t, hq, hd)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    pick = torch.Generator().manual_seed(42)
    rows = torch.cat([torch.tensor([0, 1, 127, 128, 65535, 65536, t - 1]),
                      torch.randint(0, t, (505,), generator=pick)]).to(DEV)
    kf, vf = k.float(), v.float()
    worst = 0.0
    for chunk in rows.split(64):
        want = _reference_rows(q, kf, vf, chunk, 0, window, scale)
        worst = max(worst, (got[chunk].float() - want).abs().max().item())
    assert worst <= 2e-2, worst
