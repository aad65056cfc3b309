"""Loading the golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py from the reference itself)."""

from __future__ import annotations

import ast
import hashlib
from pathlib import Path

import numpy as np

from karpo_decision_b200.synthetic import Spec, numpy_weights

GOLDEN = Path(__file__).resolve().parent / "golden"
IMAGE_TOKEN = 4095  # the image cases' soft-token id
CASES = ["qwen_tiny", "qwen_partial", "gemma_tiny", "gemma_blocks", "qwen_tiny_fp8", "gemma_tiny_fp8", "qwen_bidir",
         "gemma_bidir", "gemma_blocks_bidir", "gemma_global512", "qwen_hybrid", "gemma_images", "qwen_hybrid128",
         "qwen_images"]
#: BASELINE configurations 2-5 at full width (depth cut), from the reference's bf16 path (float32 run beside it).
WIDE = ["qwen_0p8b", "qwen_4b_fp8", "gemma_12b", "gemma_12b_fp8", "gemma_31b_fp8"]


def load(name: str) -> tuple[Spec, dict, dict, dict]:
    """(spec, weights, pack arrays, expected outputs) of golden case ``name``; the regenerated weights are checked
    against the digest recorded with the fixture."""
    z = np.load(GOLDEN / f"{name}.npz")
    spec = Spec(**ast.literal_eval(str(z["spec"])))
    weights = numpy_weights(spec, int(z["seed"]))
    h = hashlib.sha256()
    for key in sorted(weights):
        h.update(key.encode())
        h.update(np.ascontiguousarray(weights[key], dtype=np.float32).tobytes())
    if h.hexdigest() != str(z["weights_sha256"]):
        raise AssertionError(f"{name}: regenerated weights differ from the ones the fixture was made with")
    pack = {k: z[k] for k in ("input_ids", "seqpos", "cu", "markers", "marker_cu", "segment_ids", "image_features",
                              "rope") if k in z.files}
    if "image_features" in pack:  # the image cases' soft-token id (tests/golden/make_golden.py IMAGE_TOKEN)
        pack["image_token"] = IMAGE_TOKEN
    expected = {k: z[k] for k in ("hidden", "logits", "hidden_fp32", "logits_fp32") if k in z.files}
    expected["dtype"] = str(z["dtype"]) if "dtype" in z.files else "fp32"
    return spec, weights, pack, expected


#: The north-star readout bound: max-abs difference of the readout logits.
READOUT_BOUND = 2e-2


def readout_bar(got: np.ndarray, want: np.ndarray, bound: float = READOUT_BOUND) -> tuple[float, float, int]:
    """Asserts the readout bar: every logit within ``bound`` of ``want`` (max-abs), and the same top answer for every
    readout whose top-two margin in ``want`` exceeds 2 * bound. A readout whose two best answers lie closer than that
    can change its top answer within the bound (a near tie); there the top answer must be one of the answers within
    2 * bound of ``want``'s best, which the bound implies and which is checked too. Returns (max-abs error, top-answer
    agreement over all readouts, number of near ties)."""
    err = float(np.abs(got - want).max())
    assert np.isfinite(got).all()
    assert err <= bound, f"readout max-abs {err:.4f} above {bound:.4f}"
    ordered = np.sort(want, axis=-1)
    margin = ordered[:, -1] - ordered[:, -2]
    clear = margin > 2 * bound
    ours, theirs = got.argmax(-1), want.argmax(-1)
    assert np.array_equal(ours[clear], theirs[clear]), "a top answer changed on a readout with a clear margin"
    rows = np.arange(len(ours))
    assert (want[rows, ours] >= want.max(-1) - 2 * bound).all()
    return err, float((ours == theirs).mean()), int((~clear).sum())
