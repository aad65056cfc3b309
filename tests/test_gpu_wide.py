"""Parity at the benchmark configurations' full widths, and attention at their lengths.

Whole forwards: BASELINE configurations 2-5 at full width with their depth cut to 2 (Qwen-shaped) or 6 (Gemma-shaped:
5 sliding layers with the 1,024-token window and 1 global layer) against the reference's own runs of the same case
(tests/golden/, made by tests/golden/make_golden.py): its served path (the backbone in bf16; ``--fp8`` for the FP8
cases) and its float32 run. The bar (``golden_cases.readout_bar``): readout logits within 2e-2 (max-abs) and the same
top answer wherever two answers are not a near tie. Where the reference's own served path is farther than 2e-2 from its
float32 run on a case (random weights at 12B width; every FP8 case, whose single e4m3 rounding flips move a random
model's readout by 0.1-0.3), the bound is that measured noise of the reference itself instead, and the FP8 arithmetic
is pinned exactly, projection by projection, on the reference's own inputs.

Attention at the configurations' shapes: head 256 with the (1023, 0) window over sequences one short of, at and past
the window (config 4's sliding layers), and one 131,072-token sequence at head 128 with config 5's 32/16 heads,
checked on sampled query rows (its query tensor holds 2^29 elements, 1 GiB, so products of row index and row stride
leave the 32-bit range in bytes)."""

import numpy as np
import pytest
import torch

from golden_cases import READOUT_BOUND, WIDE, load, readout_bar
from karpo_decision_b200 import Packed, Readout, from_arrays, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("name", WIDE)
def test_full_width_forward_matches_reference(name):
    spec, weights, arrays, expected = load(name)
    fp8 = name.endswith("_fp8")
    model = Packed(spec, weights, DEV, fp8=fp8)
    head = Readout(weights["readout"], spec.logit_cap, DEV)
    del weights
    logits = head(model(from_arrays(arrays, DEV))).cpu().numpy()
    torch.cuda.synchronize()
    ops.check_status(DEV)
    served, exact = expected["logits"], expected["logits_fp32"]
    floor = float(np.abs(served - exact).max())  # the reference's own served path against its float32 run
    if fp8:
        # the served --fp8 path; its own distance to the float32 --fp8 run measures how far single e4m3 rounding
        # flips carry a random model's readout (the arithmetic itself is pinned exactly below)
        err, agree, ties = readout_bar(logits, served, max(READOUT_BOUND, floor))
        print(f"{name}: readout max-abs vs the reference's --fp8 path {err:.4f} (its own bf16 vs float32 runs differ "
              f"by {floor:.4f}), top answers agree on {agree:.0%} ({ties} near ties)")
        return
    # bf16: as close to the exact (float32) result as the reference's own bf16 path is, and to that bf16 path as two
    # bf16 realizations are to each other; both are the 2e-2 bar wherever the reference's own noise is below it
    err32, agree, ties = readout_bar(logits, exact, max(READOUT_BOUND, 1.25 * floor))
    err16, _, _ = readout_bar(logits, served, max(READOUT_BOUND, 1.5 * floor))
    print(f"{name}: readout max-abs vs the reference's float32 run {err32:.4f} and its bf16 run {err16:.4f} (its own "
          f"bf16 vs float32: {floor:.4f}; 2e-2 {'met' if max(err32, err16) <= READOUT_BOUND else 'not met'}), top "
          f"answers agree on {agree:.0%} ({ties} near ties)")


@pytest.mark.parametrize("name", [n for n in WIDE if n.endswith("_fp8")])
def test_full_width_fp8_projections_equal_the_reference(name):
    """Layer 0's FP8 projections at full width on the reference's own e4m3 inputs and row scales (recorded from its
    served --fp8 path, serve/fp8.py:86-101 / serve/qwen_fp8.py:38-42): kd_gemm_fp8 with the weights quantized by
    this library at load gives the reference's bf16 outputs: more than 90% bit for bit, the rest within two bf16
    roundings at the output's scale (the tensor core sums the exact e4m3 products in another order and accumulator
    width than the reference's host product, which sums them in float32)."""
    from golden_cases import GOLDEN

    spec, weights, _, _ = load(name)
    z = np.load(GOLDEN / f"{name}.npz")
    pins = [k[len("wpin_"):-len("_out_bf16")] for k in z.files if k.startswith("wpin_") and k.endswith("_out_bf16")]
    assert pins, "the fixture records the FP8 projections of layer 0"
    for proj in pins:
        w = torch.from_numpy(weights[f"layers.0.{proj}"]).to(DEV).bfloat16()
        qw, sw = ops.quantize_rows_e4m3(w)
        a = torch.from_numpy(z[f"wpin_{proj}_in_e4m3"]).to(DEV).view(torch.float8_e4m3fn)
        sa = torch.from_numpy(z[f"wpin_{proj}_scale"]).to(DEV)
        want = torch.from_numpy(z[f"wpin_{proj}_out_bf16"].view(np.int16)).to(DEV).view(torch.bfloat16).float()
        rows = a.shape[0]
        pad = (-rows) % 128  # whole tiles of rows
        a_full = torch.cat([a.view(torch.uint8), torch.zeros(pad, a.shape[1], dtype=torch.uint8, device=DEV)])
        sa_full = torch.cat([sa, torch.ones(pad, device=DEV)])
        got = ops.gemm_fp8(a_full.view(torch.float8_e4m3fn), sa_full, qw, sw)[:rows].float()
        torch.cuda.synchronize()
        diff = (got - want).abs()
        exact = float((diff == 0).float().mean())
        print(f"{name} layer 0 {proj}: {exact:.2%} of outputs bit-equal to the reference's, max-abs {diff.max():.3g} "
              f"at output scale {want.abs().max():.3g}")
        # the tensor core sums the exact e4m3 products of 2,560-21,504 terms in its own order and accumulator width,
        # not as a sequential float32 sum: within two bf16 roundings at the output's scale, most outputs bit-equal
        assert diff.max().item() <= 2 ** -6 * want.abs().max().item(), proj
        assert exact > 0.9, proj


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


def test_attention_long_sequence_runs_head_by_head_among_short_ones():
    """A pack whose middle sequence's keys and values outgrow L2 (33,000 tokens x 4 key/value heads of 128: 68 MB),
    so the kernel runs that sequence key/value head by key/value head while the short ones keep the query-heads-
    innermost order: 16 query heads (groups of 4), causal; every row of the short sequences and 256 sampled rows of
    the long one, all heads, against float32."""
    g = torch.Generator(device=DEV).manual_seed(43)
    lengths = [300, 33000, 700]
    t, hq, hkv, hd = sum(lengths), 16, 4, 128
    scale = hd ** -0.5
    q = torch.randn(t, hq, hd, generator=g, device=DEV).bfloat16()
    k = torch.randn(t, hkv, hd, generator=g, device=DEV).bfloat16()
    v = torch.randn(t, hkv, hd, generator=g, device=DEV).bfloat16()
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=DEV)
    got = ops.attention_varlen(q, k, v, cu, cu, max(lengths), scale, (-1, 0)).view(t, hq, hd)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    pick = torch.Generator().manual_seed(44)
    kf, vf = k.float(), v.float()
    worst = 0.0
    for start, n in zip(cu[:-1].tolist(), lengths, strict=True):
        rows = torch.arange(start, start + n)
        if n > 1000:
            rows = torch.cat([rows[:4], rows[127:130], rows[-4:], rows[torch.randint(0, n, (245,), generator=pick)]])
        for chunk in rows.to(DEV).split(64):
            want = _reference_rows(q, kf, vf, chunk, start, -1, scale)
            worst = max(worst, (got[chunk].float() - want).abs().max().item())
    assert worst <= 2e-2, worst
