"""The CPU oracle (oracle/, a numpy restatement) against golden fixtures made by running the reference's own packed
forward and readout (tests/golden/make_golden.py): the pin that makes the oracle a trustworthy checker."""

import numpy as np
import pytest

import oracle
from golden_cases import CASES, GOLDEN, load

PLAIN = [c for c in CASES if not c.endswith("_fp8")]
FP8 = [c for c in CASES if c.endswith("_fp8")]


def forward(spec):
    return oracle.qwen_forward if spec.family == "qwen" else oracle.gemma_forward


@pytest.mark.parametrize("name", PLAIN)
def test_oracle_matches_reference_fixture(name):
    spec, weights, pack, expected = load(name)
    hidden = forward(spec)(weights, spec.as_dict(), pack, mode="fp32")
    logits = oracle.readout(hidden, weights["readout"], spec.logit_cap)
    scale = np.abs(expected["hidden"]).max()
    # float32 restatement vs float32 reference: only the summation order differs.
    assert np.abs(hidden - expected["hidden"]).max() <= 2e-4 * scale, name
    assert np.abs(logits - expected["logits"]).max() <= 2e-4, name
    assert (logits.argmax(-1) == expected["logits"].argmax(-1)).all()


@pytest.mark.parametrize("name", FP8)
def test_oracle_fp8_projection_matches_reference(name):
    """Layer 0's quantized projections, given the reference's own e4m3 inputs and scales: the oracle's weight
    quantization and rowwise-scaled product reproduce the reference's outputs (float32 summation order only)."""
    spec, weights, _, _ = load(name)
    z = np.load(GOLDEN / f"{name}.npz")
    pinned = [k[len("pin_"):-len("_out")] for k in z.files if k.startswith("pin_") and k.endswith("_out")]
    assert pinned, "fixture has no pinned projections"
    for proj in pinned:
        w = weights[f"layers.0.{proj}"]
        qw, sw = oracle.e4m3_rows(w)
        got = (z[f"pin_{proj}_in"] @ qw.T) * z[f"pin_{proj}_scale"][:, None] * sw.reshape(1, -1)
        want = z[f"pin_{proj}_out"]
        assert np.abs(got - want).max() <= 1e-5 * max(np.abs(want).max(), 1e-6), proj


@pytest.mark.parametrize("name", FP8)
def test_oracle_fp8_forward_tracks_reference(name):
    """The whole FP8 forward: a deep random model turns single e4m3 rounding flips (from float32 summation-order
    differences in the norms) into visible output changes, so this is a loose check, like the reference's own
    comparison of its FP8 path (cosine, tests/gpu/test_cuda_qwen_fast.py:60-72)."""
    spec, weights, pack, expected = load(name)
    hidden = forward(spec)(weights, spec.as_dict(), pack, mode="fp32", fp8=True)
    a, b = hidden.ravel(), expected["hidden"].ravel()
    cosine = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    assert cosine > 0.9, cosine


def test_bf16_rounding_is_nearest_even():
    import torch

    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.140625, 1e-30], dtype=np.float32)
    assert np.array_equal(oracle.bf16(x), torch.from_numpy(x).bfloat16().float().numpy())


def test_e4m3_matches_torch_cast():
    import torch

    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 100,
                        np.array([0.0, 448.0, -448.0, 1e-4, 0.0009765625, 240.0, 232.0], dtype=np.float32)])
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(oracle.packed.e4m3(x), ref)


def test_unit_lower_inverse_by_blocks():
    """The blocked triangular inverse of the chunked delta rule equals a dense inverse, block multiples or not."""
    g = np.random.default_rng(3)
    for c in (64, 100, 7):
        a = np.tril(g.standard_normal((c, c)) * 0.3, -1)
        want = np.linalg.inv(np.eye(c) + a)
        assert np.abs(oracle.packed.unit_lower_inverse(a) - want).max() <= 1e-9 * max(1.0, np.abs(want).max())


def test_chunked_delta_rule_equals_recurrent():
    """The chunked (WY) gated delta rule, the form flash-linear-attention evaluates for the reference, equals the
    recurrent rule the kernels and goldens follow: sequences shorter than, equal to and longer than a chunk, state
    restarting at each sequence start, decays and write strengths in their real ranges."""
    g = np.random.default_rng(4)
    lengths = [1, 63, 64, 65, 200]
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    t, heads, dk, dv = cu[-1], 2, 16, 24
    q, k = (g.standard_normal((t, heads, dk)).astype(np.float32) for _ in range(2))
    v = g.standard_normal((t, heads, dv)).astype(np.float32)
    decay = -np.exp(g.uniform(-3.0, 0.5, (t, heads))).astype(np.float32)  # g = -exp(A_log) softplus(.) < 0
    beta = (1.0 / (1.0 + np.exp(-g.standard_normal((t, heads))))).astype(np.float32)
    want = oracle.packed.gated_delta_rule(q, k, v, decay, beta, cu)
    for chunk in (64, 16):
        got = oracle.packed.gated_delta_rule_chunked(q, k, v, decay, beta, cu, chunk=chunk)
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())  # measured 7e-7 at 0.4


@pytest.mark.parametrize("name", ["qwen_tiny", "qwen_partial", "gemma_tiny"])
def test_cpu_reference_matches_golden(name):
    """The torch restatement timed as the CPU baseline (oracle/cpu_reference.py) gives the reference's float32
    readouts, layer by layer composed as the full forward."""
    import torch

    from oracle.cpu_reference import Model

    spec, weights, arrays, expected = load(name)
    torch.set_num_threads(4)
    logits = Model(weights, spec.as_dict()).forward(arrays).numpy()
    assert np.abs(logits - expected["logits"]).max() <= 2e-4 * max(1.0, np.abs(expected["logits"]).max())


@pytest.mark.parametrize("name", ["qwen_tiny_fp8_served", "gemma_tiny_fp8_served"])
def test_oracle_fp8_bf16_within_the_served_fp8_noise(name):
    """The oracle's FP8 forward with the reference's bf16 rounding points lies as close to the reference's served
    ``--fp8`` readout as the reference's own float32 ``--fp8`` run does (e4m3 rounding flips set that distance)."""
    spec, weights, pack, expected = load(name)
    logits = oracle.readout(forward(spec)(weights, spec.as_dict(), pack, mode="bf16", fp8=True), weights["readout"],
                            spec.logit_cap)
    floor = np.abs(expected["logits"] - expected["logits_fp32"]).max()
    assert np.abs(logits - expected["logits"]).max() <= max(2e-2, floor)
