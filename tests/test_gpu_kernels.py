"""Each libkd_b200 kernel on the GPU against a float32 reference of the same op: the numpy oracle (oracle/) for the
reference's pointwise and attention math, plain float32 matmuls for the GEMMs. Inputs are seeded; sizes cover
partial tiles, ragged sequences, GQA ratios and every head size the kernels take."""

import math

import numpy as np
import pytest
import torch

import oracle
from karpo_decision_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def bf16(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(DEV).bfloat16()


def rng(seed=0):
    return np.random.default_rng(seed)


# ------------------------------------------------------------------------------------------------ GEMM


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (128, 256, 64), (255, 256, 64), (256, 256, 64), (257, 512, 128),
                                   (300, 768, 256), (1000, 1024, 1024), (513, 6144, 1024), (77, 96, 200),
                                   (4096, 2560, 2560), (384, 32, 64)])
def test_gemm_bf16_matches_fp32(m, n, k):
    """Single-CTA tiles below 256 rows, CTA pairs from 256 (a pair's second half partly or wholly past M)."""
    g = rng(m + n + k)
    a = bf16(g.standard_normal((m, k)))
    w = bf16(g.standard_normal((n, k)) * 0.05)
    got = ops.gemm(a, w).float()
    want = a.float() @ w.float().T
    torch.cuda.synchronize()
    # fp32 accumulation in another order, one bf16 rounding of the output
    assert (got - want).abs().max().item() <= 2 ** -8 * want.abs().max().item() + 1e-3
    ops.check_status(DEV)


def test_gemm_residual_epilogue_in_place():
    g = rng(1)
    a, w = bf16(g.standard_normal((700, 512))), bf16(g.standard_normal((1024, 512)) * 0.05)
    h = bf16(g.standard_normal((700, 1024)))
    want = h.float() + (a.float() @ w.float().T).bfloat16().float()
    ops.gemm(a, w, out=h, epilogue=ops.EPI_RESIDUAL, residual=h)
    assert (h.float() - want).abs().max().item() <= 2 ** -7 * want.abs().max().item()


@pytest.mark.parametrize("epilogue", [ops.EPI_SWIGLU, ops.EPI_GEGLU])
def test_gemm_gated_epilogues(epilogue):
    from karpo_decision_b200.packed import interleave_gate_up

    g = rng(2)
    m, k, inter = 333, 256, 384
    a = bf16(g.standard_normal((m, k)))
    gate, up = bf16(g.standard_normal((inter, k)) * 0.1), bf16(g.standard_normal((inter, k)) * 0.1)
    got = ops.gemm(a, interleave_gate_up(gate, up).contiguous(), epilogue=epilogue).float()
    gf = (a.float() @ gate.float().T).bfloat16().float()
    uf = (a.float() @ up.float().T).bfloat16().float()
    act = torch.nn.functional.silu(gf) if epilogue == ops.EPI_SWIGLU else \
        torch.nn.functional.gelu(gf, approximate="tanh")
    want = act * uf
    assert got.shape == (m, inter)
    assert (got - want).abs().max().item() <= 2 ** -7 * want.abs().max().item() + 1e-3


@pytest.mark.parametrize("m", [100, 517])
def test_gemm_fp8_matches_dequantized_product(m):
    """Single-CTA tiles (100 rows) and CTA pairs (517 rows)."""
    g = rng(3)
    n, k = 1024, 768
    a = bf16(g.standard_normal((m, k)))
    w = bf16(g.standard_normal((n, k)) * 0.05)
    qa, sa = ops.quantize_rows_e4m3(a)
    qw, sw = ops.quantize_rows_e4m3(w)
    got = ops.gemm_fp8(qa, sa, qw, sw).float()
    want = (qa.float() @ qw.float().T) * sa[:, None] * sw[None, :]
    assert (got - want).abs().max().item() <= 2 ** -8 * want.abs().max().item() + 1e-3


def test_quantize_rows_e4m3_bit_exact():
    """The per-row e4m3 quantization of serve/fp8.py:21-24, bit for bit (same bf16 input, same float32 math)."""
    g = rng(4)
    x = bf16(g.standard_normal((257, 1024)) * 3)
    q, s = ops.quantize_rows_e4m3(x)
    scale = x.float().abs().amax(-1, keepdim=True).clamp(min=1e-12) / 448.0  # torch CUDA: times float(1/448)
    ref = (x.float() / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(s, scale[:, 0])
    assert torch.equal(q.view(torch.uint8), ref.view(torch.uint8))


# ------------------------------------------------------------------------------------------------ pointwise


@pytest.mark.parametrize("mode,one_plus", [(ops.NORM_ONE_PLUS, True), (ops.NORM_WEIGHT, False)])
def test_rmsnorm_matches_oracle(mode, one_plus):
    g = rng(5)
    x = g.standard_normal((301, 1024)).astype(np.float32)
    w = g.standard_normal(1024).astype(np.float32) * 0.1 + (0.0 if one_plus else 1.0)
    xb, wb = bf16(x), bf16(w)
    got = ops.rmsnorm(xb, wb, mode, 1e-6).float().cpu().numpy()
    want = oracle.rms_norm(xb.float().cpu().numpy(), wb.float().cpu().numpy(), 1e-6, one_plus)
    assert np.abs(got - want).max() <= 2 ** -8 * np.abs(want).max()


@pytest.mark.parametrize("cols", [512, 5376])
def test_add_rmsnorm_and_norm_add(cols):
    """Narrow and wide rows against the oracle."""
    g = rng(6)
    h = bf16(g.standard_normal((64, cols)))
    x = bf16(g.standard_normal((64, cols)))
    w = bf16(g.standard_normal(cols) * 0.1)
    hn, xn, wn = (t.float().cpu().numpy() for t in (h, x, w))
    h2 = h.clone()
    y = ops.add_rmsnorm(h2, x, w, ops.NORM_ONE_PLUS, 1e-6)
    s = oracle.bf16(hn + xn)
    assert np.array_equal(h2.float().cpu().numpy(), s)
    assert np.abs(y.float().cpu().numpy() - oracle.rms_norm(s, wn, 1e-6, True)).max() <= 2 ** -8 * 4
    w1 = bf16(1.0 + g.standard_normal(cols) * 0.1)
    out = ops.norm_add(h, x, w1, ops.NORM_WEIGHT, 1e-6)
    want = hn + oracle.rms_norm(xn, w1.float().cpu().numpy(), 1e-6, False)
    assert np.abs(out.float().cpu().numpy() - want).max() <= 2 ** -7 * np.abs(want).max()
    # the layer-end form: (h + bf16(norm(x))) * scalar
    scalar = torch.tensor([0.75], device=DEV).bfloat16()
    out2 = ops.norm_add(h, x, w1, ops.NORM_WEIGHT, 1e-6, scalar=scalar)
    want2 = (hn + oracle.bf16(oracle.rms_norm(xn, w1.float().cpu().numpy(), 1e-6, False))) * 0.75
    assert np.abs(out2.float().cpu().numpy() - want2).max() <= 2 ** -7 * np.abs(want2).max()
    scalar = bf16(np.array([0.875]))
    out = ops.norm_add(h, x, w1, ops.NORM_WEIGHT, 1e-6, scalar=scalar)
    want = (hn + oracle.bf16(oracle.rms_norm(xn, w1.float().cpu().numpy(), 1e-6, False))) * 0.875
    assert np.abs(out.float().cpu().numpy() - want).max() <= 2 ** -7 * np.abs(want).max()


# every positive finite e4m3 value (bias 7, 3 mantissa bits, no infinities, 0x7F is NaN), ascending
E4M3_POS = sorted({(m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
                   for e in range(16) for m in range(8) if (e, m) != (15, 7)})


@pytest.mark.parametrize("cols", [768, 2560, 3072, 3840, 5376, 9728, 21504])
def test_rmsnorm_e4m3_equals_norm_then_quantize(cols):
    """The fused norm + e4m3 cast equals the two ops, on the warp-per-row path (narrow rows) and the block-per-row
    path (3,072 columns and wider), and the wide norm matches the oracle."""
    g = rng(7)
    x = bf16(g.standard_normal((129, cols)))
    w = bf16(1.0 + g.standard_normal(cols) * 0.1)
    y = ops.rmsnorm(x, w, ops.NORM_WEIGHT, 1e-6)
    q1, s1 = ops.quantize_rows_e4m3(y)
    q2, s2 = ops.rmsnorm_e4m3(x, w, ops.NORM_WEIGHT, 1e-6)
    assert torch.equal(s1, s2) and torch.equal(q1.view(torch.uint8), q2.view(torch.uint8))
    want = oracle.rms_norm(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6, False)
    assert np.abs(y.float().cpu().numpy() - want).max() <= 2 ** -8 * np.abs(want).max()
    # the quantization alone (amax per row, x / scale) against the definition
    xf = x.float()
    sw = torch.clamp(xf.abs().amax(1), min=1e-12) * (1.0 / 448.0)
    q3, s3 = ops.quantize_rows_e4m3(x)
    assert torch.equal(s3, sw)
    assert torch.equal(q3.view(torch.uint8), (xf / sw[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8))


def test_quantize_rows_e4m3_near_rounding_midpoints():
    """Rows built so that x / scale lands next to e4m3 rounding midpoints, over many scales (every mantissa pattern of
    the row maximum, all-ones included): the cast equals torch's float division, clamp and cast bit for bit."""
    g = rng(17)
    rows, cols = 512, 1024
    amax = torch.from_numpy(np.ldexp(1.0 + np.arange(rows) / 128.0, g.integers(-20, 20, rows))).float()
    amax[0] = 2.0 - 2.0 ** -7  # the widest bf16 mantissa (all ones)
    scale = amax * (1.0 / 448.0)
    grid = torch.tensor([0.5 * (a + b) for a, b in zip(E4M3_POS[:-1], E4M3_POS[1:])], dtype=torch.float32)
    mid = grid[torch.from_numpy(g.integers(0, len(grid), (rows, cols)))] * torch.from_numpy(
        g.choice([-1.0, 1.0], (rows, cols))).float()
    x = (mid * scale[:, None] * (1.0 + torch.from_numpy(g.uniform(-2e-3, 2e-3, (rows, cols))).float())).bfloat16()
    x[:, 0] = amax.bfloat16()
    x = x.to(DEV)
    q, s = ops.quantize_rows_e4m3(x)
    xf = x.float()
    sw = torch.clamp(xf.abs().amax(1), min=1e-12) * (1.0 / 448.0)
    assert torch.equal(s, sw)
    want = (xf / sw[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(q.view(torch.uint8), want.view(torch.uint8))


def test_embed_and_scaled_embed():
    g = rng(8)
    table = bf16(g.standard_normal((1000, 256)) * 0.02)
    ids = torch.from_numpy(g.integers(0, 1000, 777)).to(DEV)
    assert torch.equal(ops.embed(ids, table), table[ids])
    scaled = ops.embed(ids, table, math.sqrt(256))
    want = table[ids] * torch.tensor(16.0).bfloat16()
    assert torch.equal(scaled, want)


def test_rope_table_matches_transformers_formula():
    """The rotary tables against Transformers' formula evaluated by torch on the same GPU (the reference's rotary
    module runs there: float32 position x inv_freq, cos/sin, cast to bf16). A host-side cos/sin is a different
    float32 implementation whose last-bit differences flip a few bf16 roundings, so it is not the comparison."""
    theta, rot, n = 1e6, 128, 5000
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))
    cos, sin = ops.rope_table(inv.to(DEV), n)
    freqs = torch.arange(n, dtype=torch.float32, device=DEV)[:, None] * inv.to(DEV)[None, :]
    emb = torch.cat([freqs, freqs], -1)
    for got, want in ((cos, emb.cos()), (sin, emb.sin())):
        diff = (got - want.bfloat16().float()).abs()
        assert (diff > 0).float().mean().item() < 1e-4 and diff.max().item() <= 2 ** -8


def test_mrope_tables_match_transformers_rotary_module():
    """M-RoPE tables (one row per token) against Transformers' own Qwen3_5TextRotaryEmbedding (interleaved sections)
    run by torch on the same GPU over the same (3, 1, T) positions, and equal to kd_rope_table's rows where a token's
    three axes hold the same position."""
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding

    from karpo_decision_b200.synthetic import Spec

    spec = Spec("qwen", 1, 256, 2, 1, 256, 512, 1024, partial_rotary=0.25, mrope_section=(11, 11, 10))
    config = Qwen3_5TextConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=256,
                               rope_parameters={"rope_type": "default", "rope_theta": 1e7,
                                                "partial_rotary_factor": 0.25, "mrope_section": [11, 11, 10]})
    module = Qwen3_5TextRotaryEmbedding(config, device=DEV)
    g = rng(31)
    t = 3000
    text = np.arange(t)
    pos = np.stack([text, text, text])
    pos[1, 100:400] = 100 + g.integers(0, 40, 300)  # an image's height and width positions
    pos[2, 100:400] = 100 + g.integers(0, 40, 300)
    positions = torch.from_numpy(pos).to(DEV)
    axis = torch.tensor(spec.pair_axes(), dtype=torch.int32, device=DEV)
    cos, sin = ops.rope_table_axes(module.inv_freq.float().contiguous(), positions, axis)
    want_cos, want_sin = module(torch.zeros(1, dtype=torch.bfloat16, device=DEV), positions[:, None, :])
    for got, want in ((cos, want_cos[0].float()), (sin, want_sin[0].float())):
        diff = (got - want).abs()
        assert (diff > 0).float().mean().item() < 1e-4 and diff.max().item() <= 2 ** -8
    plain_cos, plain_sin = ops.rope_table(module.inv_freq.float().contiguous(), t)
    text_rows = torch.from_numpy(np.r_[0:100, 400:t]).to(DEV)
    assert torch.equal(cos[text_rows], plain_cos[text_rows]) and torch.equal(sin[text_rows], plain_sin[text_rows])


@pytest.mark.parametrize("family,hd,partial", [("qwen", 128, 1.0), ("qwen", 64, 0.5), ("gemma", 256, 1.0),
                                               ("gemma", 128, 1.0), ("gemma", 512, 1.0)])
def test_qkv_norm_rope_matches_oracle(family, hd, partial):
    g = rng(9)
    t, hq, hkv = 97, 4, 2
    gated = family == "qwen"
    width = hq * hd * (2 if gated else 1) + 2 * hkv * hd
    qkv = bf16(g.standard_normal((t, width)))
    seqpos = torch.from_numpy(np.concatenate([np.arange(40), np.arange(57)])).to(DEV)
    one_plus = gated
    qn = bf16(g.standard_normal(hd) * 0.1 + (0 if one_plus else 1))
    kn = bf16(g.standard_normal(hd) * 0.1 + (0 if one_plus else 1))
    mode = ops.NORM_ONE_PLUS if one_plus else ops.NORM_WEIGHT
    rot = int(hd * partial)
    inv = 1.0 / (1e6 ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))
    cos, sin = ops.rope_table(inv.to(DEV), 128)
    q, k, v, gate = ops.qkv_norm_rope(qkv, seqpos, hq, hkv, hd, gated, qn, kn, mode, -1 if gated else ops.NORM_NONE,
                                      1e-6, cos, sin)
    # oracle
    x = qkv.float().cpu().numpy()
    pos = seqpos.cpu().numpy()
    c, s_ = cos.cpu().numpy()[pos], sin.cpu().numpy()[pos]
    qw = hq * hd * (2 if gated else 1)
    qraw = x[:, :qw].reshape(t, hq, -1)
    if gated:
        qraw, graw = qraw[..., :hd], qraw[..., hd:].reshape(t, -1)
    kraw = x[:, qw:qw + hkv * hd].reshape(t, hkv, hd)
    vraw = x[:, qw + hkv * hd:].reshape(t, hkv, hd)
    qnn, knn = qn.float().cpu().numpy(), kn.float().cpu().numpy()
    rq = oracle.rms_norm(qraw, qnn, 1e-6, one_plus)
    rk = oracle.rms_norm(kraw, knn, 1e-6, one_plus)
    if gated:
        rq, rk = oracle.bf16(rq), oracle.bf16(rk)
    want_q = oracle.packed.apply_rope(rq, c, s_)
    want_k = oracle.packed.apply_rope(rk, c, s_)
    want_v = vraw if gated else oracle.rms_norm(vraw, None, 1e-6, False)
    for got, want in ((q, want_q), (k, want_k), (v, want_v)):
        assert np.abs(got.float().cpu().numpy() - want).max() <= 2 ** -7 * max(np.abs(want).max(), 1.0)
    if gated:
        assert np.array_equal(gate.float().cpu().numpy(), graw)


# ------------------------------------------------------------------------------------------------ attention


def attention_case(lengths, hq, hkv, hd, window, scale, gated=False, seed=10):
    g = rng(seed)
    t = sum(lengths)
    q = bf16(g.standard_normal((t, hq, hd)))
    k = bf16(g.standard_normal((t, hkv, hd)))
    v = bf16(g.standard_normal((t, hkv, hd)))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    cu_t = torch.from_numpy(cu).to(DEV)
    gate = bf16(g.standard_normal((t, hq * hd))) if gated else None
    got = ops.attention_varlen(q, k, v, cu_t, cu_t, max(lengths), scale, window, gate=gate)
    want = oracle.attention_varlen(*(x.float().cpu().numpy() for x in (q, k, v)), cu, cu, scale, window)
    want = oracle.bf16(want).reshape(t, hq * hd)
    if gated:
        gn = gate.float().cpu().numpy()
        want = want * (1.0 / (1.0 + np.exp(-gn)))
    return got.float().cpu().numpy(), want


@pytest.mark.parametrize("lengths", [[1], [7, 130, 64, 1, 300], [513], [128, 128]])
@pytest.mark.parametrize("hd,hq,hkv", [(128, 16, 8), (128, 8, 2), (128, 4, 4), (128, 6, 2), (64, 4, 2), (256, 4, 1),
                                       (512, 4, 1)])
def test_attention_causal_matches_oracle(lengths, hd, hq, hkv):
    """Head dims 64-512; at 128, key/value groups of 1, 2, 3 and 4 query heads (the GQA head mapping)."""
    got, want = attention_case(lengths, hq, hkv, hd, (-1, 0), hd ** -0.5)
    # P is rounded to bf16 before the PV product (flash attention); outputs are O(1)
    assert np.abs(got - want).max() <= 2e-2


@pytest.mark.parametrize("window", [(15, 0), (63, 0), (-1, -1)])
def test_attention_window_and_bidirectional(window):
    got, want = attention_case([200, 17, 90], 4, 2, 128, window, 1.0)
    assert np.abs(got - want).max() <= 3e-2


@pytest.mark.parametrize("window", [(15, 0), (-1, -1)])
def test_attention_head512_windows_and_separate_key_bounds(window):
    """Head size 512 (two value slices per head): sliding and bidirectional windows, and queries over longer
    end-aligned key spans (a branch over its shared block's keys, families/gemma/packed.py:196-220)."""
    # scale 512^-0.5 keeps random scores O(1): at scale 1 the softmax is one-hot and compares bf16 ulps of V
    scale = 512 ** -0.5
    got, want = attention_case([200, 17, 90], 8, 2, 512, window, scale)
    assert np.abs(got - want).max() <= 3e-2
    g = rng(15)
    lq, lk = [5, 70, 1], [40, 70, 300]
    q = bf16(g.standard_normal((sum(lq), 4, 512)))
    k, v = (bf16(g.standard_normal((sum(lk), 1, 512))) for _ in range(2))
    cu_q = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)
    got = ops.attention_varlen(q, k, v, torch.from_numpy(cu_q).to(DEV), torch.from_numpy(cu_k).to(DEV), max(lq),
                               scale, window)
    want = oracle.attention_varlen(*(x.float().cpu().numpy() for x in (q, k, v)), cu_q, cu_k, scale, window)
    assert np.abs(got.float().cpu().numpy() - oracle.bf16(want).reshape(sum(lq), -1)).max() <= 3e-2


@pytest.mark.parametrize("hq,hkv", [(16, 8), (4, 4)])
@pytest.mark.parametrize("gated", [False, True])
def test_attention_long_sequences(hq, hkv, gated):
    """Many key tiles per query tile (running-maximum rescales) and several work items per persistent CTA, GQA and
    MHA, with and without Qwen's output gate."""
    got, want = attention_case([1500, 2100, 300, 1], hq, hkv, 128, (-1, 0), 128 ** -0.5, gated=gated, seed=21)
    assert np.abs(got - want).max() <= 2e-2


@pytest.mark.parametrize("window", [(-1, 0), (100, 0), (-1, -1)])
def test_attention_head128_separate_key_bounds(window):
    """Queries end-aligned to longer or shorter key spans at head dim 128 (8 query / 2 key-value heads), including a
    query tile that sees no key at all (its output is 0)."""
    g = rng(16)
    lq, lk = [5, 300, 1, 300], [40, 300, 260, 100]  # the last one's first query tile sees no key
    scale = 128 ** -0.5
    q = bf16(g.standard_normal((sum(lq), 8, 128)))
    k, v = (bf16(g.standard_normal((sum(lk), 2, 128))) for _ in range(2))
    cu_q = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)
    got = ops.attention_varlen(q, k, v, torch.from_numpy(cu_q).to(DEV), torch.from_numpy(cu_k).to(DEV), max(lq),
                               scale, window)
    want = oracle.attention_varlen(*(x.float().cpu().numpy() for x in (q, k, v)), cu_q, cu_k, scale, window)
    want = np.nan_to_num(oracle.bf16(want).reshape(sum(lq), -1))
    assert np.abs(got.float().cpu().numpy() - want).max() <= 2e-2


def test_attention_output_gate():
    got, want = attention_case([100, 60], 4, 2, 128, (-1, 0), 128 ** -0.5, gated=True)
    assert np.abs(got - want).max() <= 2e-2


@pytest.mark.parametrize("hkv", [4, 2])
def test_attention_sequences_do_not_see_each_other(hkv):
    """A sequence's outputs are the same alone and packed with others (tests/gpu/test_packed_qwen.py:114-122), for
    query heads taken one at a time (4/4) and in pairs sharing a key/value head (4/2)."""
    g = rng(11)
    lengths = [50, 90, 70]
    t = sum(lengths)
    q = bf16(g.standard_normal((t, 4, 128)))
    k, v = (bf16(g.standard_normal((t, hkv, 128))) for _ in range(2))
    cu = torch.tensor([0, 50, 140, 210], dtype=torch.int32, device=DEV)
    together = ops.attention_varlen(q, k, v, cu, cu, 90, 0.1, (-1, 0))
    cu1 = torch.tensor([0, 90], dtype=torch.int32, device=DEV)
    alone = ops.attention_varlen(q[50:140], k[50:140], v[50:140], cu1, cu1, 90, 0.1, (-1, 0))
    assert torch.equal(together[50:140], alone)


# ------------------------------------------------------------------------------------------------ head


def test_marker_norm_and_readout():
    g = rng(12)
    h = bf16(g.standard_normal((500, 256)))
    markers = torch.tensor([3, 99, 499, 0], device=DEV)
    w = bf16(g.standard_normal(256) * 0.1)
    out = ops.marker_norm(h, markers, w, ops.NORM_ONE_PLUS, 1e-6)
    want = oracle.rms_norm(h.float().cpu().numpy()[[3, 99, 499, 0]], w.float().cpu().numpy(), 1e-6, True)
    assert np.abs(out.float().cpu().numpy() - want).max() <= 2 ** -8 * np.abs(want).max()
    head = torch.from_numpy(g.standard_normal((5, 256)).astype(np.float32) * 0.02).to(DEV)
    for cap in (None, 30.0, 0.5):
        logits = ops.readout(out, head, cap).cpu().numpy()
        ref = oracle.readout(out.float().cpu().numpy(), head.cpu().numpy(), cap)
        assert np.abs(logits - ref).max() <= 1e-5


@pytest.mark.parametrize("family,hd,partial,fp8", [("qwen", 128, 1.0, False), ("qwen", 64, 0.5, False),
                                                   ("gemma", 256, 1.0, False), ("gemma", 128, 1.0, False),
                                                   ("qwen", 256, 0.25, False), ("gemma", 64, 1.0, False),
                                                   ("qwen", 128, 1.0, True), ("gemma", 128, 1.0, True),
                                                   ("gemma", 256, 1.0, True)])
def test_qkv_projection_equals_gemm_then_norm_rope(family, hd, partial, fp8):
    """The fused QKV epilogue against the stored projection followed by kd_qkv_norm_rope (one bf16 ulp: the sums of
    squares run in another order)."""
    g = rng(13)
    t, hq, hkv, hidden = 301, 4, 2, 256
    gated = family == "qwen"
    width = hq * hd * (2 if gated else 1) + 2 * hkv * hd
    x = bf16(g.standard_normal((t, hidden)))
    w = bf16(g.standard_normal((width, hidden)) * 0.05)
    seqpos = torch.from_numpy(np.concatenate([np.arange(200), np.arange(101)])).to(DEV)
    one_plus = gated
    mode = ops.NORM_ONE_PLUS if one_plus else ops.NORM_WEIGHT
    qn = bf16(g.standard_normal(hd) * 0.1 + (0 if one_plus else 1))
    kn = bf16(g.standard_normal(hd) * 0.1 + (0 if one_plus else 1))
    rot = int(hd * partial)
    inv = 1.0 / (1e6 ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))
    cos, sin = ops.rope_table(inv.to(DEV), 256)
    v_mode = -1 if gated else ops.NORM_NONE
    if fp8:
        xq, xs = ops.quantize_rows_e4m3(x)
        wq, ws = ops.quantize_rows_e4m3(w)
        qkv = ops.gemm_fp8(xq, xs, wq, ws)
        cs = ops.rope_gather(seqpos, cos, sin)
        fused = ops.qkv_projection(xq, wq, seqpos, hq, hkv, hd, gated, qn, kn, mode, v_mode, 1e-6, cs, rot,
                                   scale_a=xs, scale_w=ws)
    else:
        qkv = ops.gemm(x, w)
        cs = ops.rope_gather(seqpos, cos, sin)
        fused = ops.qkv_projection(x, w, seqpos, hq, hkv, hd, gated, qn, kn, mode, v_mode, 1e-6, cs, rot)
    split = ops.qkv_norm_rope(qkv, seqpos, hq, hkv, hd, gated, qn, kn, mode, v_mode, 1e-6, cos, sin)
    for a_, b_ in zip(fused, split, strict=True):
        if a_ is None:
            assert b_ is None
            continue
        diff = (a_.float() - b_.float()).abs().max().item()
        assert diff <= 2 ** -7 * max(b_.float().abs().max().item(), 1.0), diff
    ops.check_status(DEV)


def test_gather_rows():
    g = rng(14)
    src = bf16(g.standard_normal((300, 8, 64)))
    rows = torch.from_numpy(g.integers(0, 300, 517)).to(DEV)
    assert torch.equal(ops.gather_rows(src, rows), src[rows])


# ------------------------------------------------------------------------------------------------ Gated DeltaNet


def test_conv_silu_matches_oracle_and_restarts_at_sequence_starts():
    g = rng(21)
    lengths = [1, 2, 37, 300, 5]
    t, c = sum(lengths), 384
    x = bf16(g.standard_normal((t, c + 64)))  # a wider buffer: the convolution reads its first c columns
    w = bf16(g.standard_normal((c, 4)) * 0.3)
    seqpos = np.concatenate([np.arange(n) for n in lengths])
    got = ops.conv_silu(x, w, torch.from_numpy(seqpos).to(DEV), channels=c)
    want = oracle.packed.causal_conv_silu(x[:, :c].float().cpu().numpy(), w.float().cpu().numpy(), seqpos)
    assert np.abs(got.float().cpu().numpy() - oracle.bf16(want)).max() <= 2 ** -7 * max(np.abs(want).max(), 1.0)


@pytest.mark.parametrize("nk,nv,dk,dv,lengths", [(2, 4, 64, 64, [1, 17, 200, 33]), (2, 2, 128, 64, [1, 17, 200, 33]),
                                                  (1, 2, 128, 128, [1, 17, 200, 33]),
                                                  (2, 4, 128, 128, [127, 128, 129, 1, 300, 700])])
def test_gated_delta_rule_matches_oracle(nk, nv, dk, dv, lengths):
    """The gated delta rule against the oracle's recurrent rule (Transformers' torch_recurrent_gated_delta_rule), over
    packed sequences of ragged lengths (the state restarts at each). Heads of 128 run the chunked tensor-core form, whose
    128-token chunks the lengths straddle (one short of, at and one past a chunk, several chunks): its products take
    bf16 operands (normalized q and k, W, U, the inverse T, D and the state S, as flash-linear-attention's chunked
    kernels do) with float32 accumulation, so it is held to 2e-2 of the output scale; the recurrent form (float32
    throughout) to one bf16 rounding."""
    g = rng(22)
    t = sum(lengths)
    width = 2 * nk * dk + nv * dv
    qkv = bf16(g.standard_normal((t, width)))
    ab = bf16(g.standard_normal((t, 2 * nv)))
    a_log = bf16(np.log(g.uniform(1, 16, nv)))
    dt = np.exp(g.uniform(np.log(1e-3), np.log(1e-1), nv))
    dt_bias = bf16(dt + np.log(-np.expm1(-dt)))
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    got = ops.gated_delta_rule(qkv, ab, a_log, dt_bias, torch.from_numpy(cu).to(DEV), nk, nv, dk, dv)
    x = qkv.float().cpu().numpy()
    q = x[:, :nk * dk].reshape(t, nk, dk).repeat(nv // nk, axis=1)
    k = x[:, nk * dk:2 * nk * dk].reshape(t, nk, dk).repeat(nv // nk, axis=1)
    v = x[:, 2 * nk * dk:].reshape(t, nv, dv)
    abn = ab.float().cpu().numpy()
    b, a = abn[:, :nv], abn[:, nv:]
    gg = -np.exp(a_log.float().cpu().numpy()) * oracle.packed.softplus(a + dt_bias.float().cpu().numpy())
    beta = oracle.bf16(1.0 / (1.0 + np.exp(-b)))
    want = oracle.packed.gated_delta_rule(q, k, v, gg, beta, cu).reshape(t, nv * dv)
    ops.check_status(DEV)
    bound = 2e-2 if dk == dv == 128 else 2 ** -7
    err = np.abs(got.float().cpu().numpy() - want).max()
    print(f"delta rule {nk}/{nv} heads of {dk}/{dv}: max-abs {err:.3g} at output scale {np.abs(want).max():.3g}")
    assert err <= bound * max(np.abs(want).max(), 1.0)


def test_gated_norm_matches_oracle():
    g = rng(23)
    t, heads, dv = 77, 4, 128
    x = bf16(g.standard_normal((t, heads * dv)))
    z = bf16(g.standard_normal((t, heads * dv)))
    w = bf16(1 + 0.1 * g.standard_normal(dv))
    got = ops.gated_norm(x, z, w, heads, dv, 1e-6).float().cpu().numpy()
    xn = x.float().cpu().numpy().reshape(t, heads, dv)
    normed = oracle.bf16(xn / np.sqrt((xn * xn).mean(-1, keepdims=True) + 1e-6))
    normed = oracle.bf16(w.float().cpu().numpy() * normed)
    want = oracle.bf16(normed * oracle.packed.silu(z.float().cpu().numpy().reshape(t, heads, dv)))
    assert np.abs(got - want.reshape(t, -1)).max() <= 2 ** -7 * max(np.abs(want).max(), 1.0)
