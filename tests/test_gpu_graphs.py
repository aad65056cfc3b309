"""The CUDA-graph path (karpo_decision_b200.graphs) against the eager forward: a replay must give the eager result bit
for bit for any pack its bucket covers (padding rows are separate sequences, so the real rows see exactly what they
see eagerly), and uncovered packs run the plain path (the reference's tests/gpu/test_cuda_graphs.py:31-79)."""

import numpy as np
import pytest
import torch

from golden_cases import load
from karpo_decision_b200 import Packed, from_arrays
from karpo_decision_b200.graphs import Graphs
from karpo_decision_b200.synthetic import synthetic_pack_arrays

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("name", ["qwen_tiny", "gemma_tiny", "qwen_bidir", "gemma_bidir", "qwen_hybrid"])
def test_replay_equals_eager_for_any_covered_pack(name):
    spec, weights, _, _ = load(name)
    model = Packed(spec, weights, DEV)
    graphs = Graphs(model, buckets=(512, 1024, 2048), max_sequences=16)
    for seed, lengths in enumerate([[100], [37, 211, 64, 130], [512], [300, 400, 9, 1, 250], [2000, 48]]):
        # Gemma reads out one marker per block, at its last token (families/gemma/packed.py:136-143)
        arrays = synthetic_pack_arrays(lengths, spec.vocab, seed=seed,
                                       markers_per_seq=(1, 3) if spec.family == "qwen" else (1, 1))
        p = from_arrays(arrays, DEV)
        eager = model(p).clone()
        replay = graphs(p)
        torch.cuda.synchronize()
        assert graphs.bucket_for(p) is not None
        assert torch.equal(replay, eager), (name, lengths, (replay.float() - eager.float()).abs().max().item())
    graphs.release()


def test_uncovered_packs_run_the_plain_path():
    spec, weights, _, _ = load("qwen_tiny")
    model = Packed(spec, weights, DEV)
    graphs = Graphs(model, buckets=(512,), max_sequences=4)
    too_long = from_arrays(synthetic_pack_arrays([600], spec.vocab, seed=1), DEV)
    too_many = from_arrays(synthetic_pack_arrays([10] * 6, spec.vocab, seed=2), DEV)
    for p in (too_long, too_many):
        assert graphs.bucket_for(p) is None
        assert torch.equal(graphs(p), model(p))
    # a covered pack after the plain ones still replays correctly
    p = from_arrays(synthetic_pack_arrays([120, 33], spec.vocab, seed=3), DEV)
    assert torch.equal(graphs(p), model(p))
