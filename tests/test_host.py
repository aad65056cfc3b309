"""Host-side logic of the B200 path that needs no GPU: weight repacking, workspace layout, packing, shapes."""

import numpy as np
import pytest
import torch

from karpo_decision_b200.pack import from_arrays, pack
from karpo_decision_b200.packed import GATE_BLOCK, Workspace, interleave_gate_up
from karpo_decision_b200.synthetic import CONFIGS, Spec, numpy_weights, synthetic_lengths, synthetic_pack_arrays


def test_interleave_gate_up_blocks_and_padding():
    gate = torch.arange(300 * 4, dtype=torch.float32).view(300, 4)
    up = -gate
    w = interleave_gate_up(gate, up)
    assert w.shape == (2 * 384, 4)  # 300 padded to 3 blocks of 128
    assert torch.equal(w[:128], gate[:128]) and torch.equal(w[128:256], up[:128])
    assert torch.equal(w[512:512 + 44], gate[256:300]) and w[512 + 44:640].abs().sum() == 0
    assert torch.equal(w[640:640 + 44], up[256:300]) and w[640 + 44:].abs().sum() == 0
    assert GATE_BLOCK == 128


def test_workspace_views_are_contiguous():
    spec = CONFIGS["tiny"]
    ws = Workspace(spec, 1000, torch.device("cpu"), fp8=True, inter_pad=1024, stored_qkv=False)
    cs = ws.cs("full_attention", 700)
    assert cs.shape == (32, 700) and cs.is_contiguous()
    q, s = ws.e4m3(700, 256)
    assert q.shape == (700, 256) and q.is_contiguous() and s.shape == (700,)
    q, k, v, gate = ws.heads(spec, "full_attention", 700)
    assert q.shape == (700, 4, 64) and k.shape == v.shape == (700, 2, 64) and gate.shape == (700, 256)
    assert q.is_contiguous() and ws.o(spec, "full_attention", 700).shape == (700, 256) and ws._qkv is None


def test_workspace_sizes_for_gemma_global_heads():
    """Gemma 4 global layers with their own head size and shared key/value heads: buffers sized for the widest kind,
    viewed per layer kind."""
    from karpo_decision_b200.packed import rotary_width

    spec = Spec("gemma", 6, 256, 4, 2, 64, 512, 100, global_head_dim=512, global_kv_heads=1, k_eq_v=True,
                global_rope="proportional")
    assert spec.attn_dims("full_attention") == (512, 1) and spec.attn_dims("sliding_attention") == (64, 2)
    assert spec.qkv_width_of("full_attention") == 4 * 512 + 2 * 512 and spec.shares_kv("full_attention")
    assert rotary_width(spec, "full_attention") == 512 and rotary_width(spec, "sliding_attention") == 64
    ws = Workspace(spec, 100, torch.device("cpu"), fp8=False, inter_pad=512, stored_qkv=True)
    q, k, v, gate = ws.heads(spec, "full_attention", 90)
    assert q.shape == (90, 4, 512) and k.shape == (90, 1, 512) and gate is None
    q, k, v, _ = ws.heads(spec, "sliding_attention", 90)
    assert q.shape == (90, 4, 64) and v.shape == (90, 2, 64)
    assert ws.qkv(spec, "full_attention", 90).shape == (90, 3072) and ws.cs("full_attention", 90).shape == (256, 90)
    # the weights: no v_proj in the shared-key global layer, per-kind shapes elsewhere
    w = numpy_weights(spec, 0)
    assert "layers.5.v_proj" not in w and w["layers.5.q_proj"].shape == (2048, 256)
    assert w["layers.5.k_proj"].shape == (512, 256) and w["layers.0.v_proj"].shape == (128, 256)


def test_synthetic_lengths_fill_exactly():
    lengths = synthetic_lengths(65536, 128, 8192, seed=3)
    assert sum(lengths) == 65536 and min(lengths) >= 1 and max(lengths) <= 8192


def test_pack_arrays_and_from_arrays_agree_with_pack():
    arrays = synthetic_pack_arrays([5, 9, 3], 100, seed=1, markers_per_seq=(1, 3))
    assert arrays["cu"].tolist() == [0, 5, 14, 17]
    assert (np.diff(arrays["marker_cu"]) >= 1).all()
    # the last token of every sequence is a marker
    ends = set((arrays["cu"][1:] - 1).tolist())
    assert ends <= set(arrays["markers"].tolist())
    p = from_arrays(arrays, torch.device("cpu"))
    assert p.cu.dtype == torch.int32 and p.markers.dtype == torch.int64 and p.max_length == 9

    class Seq:
        def __init__(self, ids, markers):
            self.input_ids, self.markers = ids, markers

    seqs = [Seq(torch.from_numpy(arrays["input_ids"][a:b]), torch.from_numpy(
        arrays["markers"][arrays["marker_cu"][i]:arrays["marker_cu"][i + 1]] - a))
        for i, (a, b) in enumerate(zip(arrays["cu"][:-1], arrays["cu"][1:]))]
    q = pack(seqs, torch.device("cpu"))
    assert torch.equal(q.markers, p.markers) and torch.equal(q.cu, p.cu) and torch.equal(q.seqpos, p.seqpos)


def test_spec_flops_and_gemma_layer_pattern():
    spec = CONFIGS["qwen-0.8b"]
    assert spec.qkv_width == 6144
    # QKV 1024x6144, o 2048x1024, gate-up 1024x6144, down 3072x1024 -> ~1 GFLOP per token (28 layers)
    assert abs(spec.gemm_flops_per_token() / 1e9 - 0.998) < 0.01
    g = Spec("gemma", 62, 64, 2, 1, 64, 64, 10)
    types = g.layer_types()
    assert types[5] == "full_attention" and types[4] == "sliding_attention" and types[-1] == "full_attention"


def test_numpy_weights_are_bf16_exact_and_seeded():
    spec = CONFIGS["tiny"]
    a, b = numpy_weights(spec, 3), numpy_weights(spec, 3)
    for key in a:
        assert np.array_equal(a[key], b[key])
    w = a["layers.0.q_proj"]
    assert np.array_equal(torch.from_numpy(w).bfloat16().float().numpy(), w)


def test_block_plan_matches_oracle_and_refuses_bad_segments():
    import pytest

    import oracle
    from karpo_decision_b200.plan import block_plan
    from karpo_decision_b200.synthetic import synthetic_block_arrays

    arrays = synthetic_block_arrays([(5, []), (6, [2, 3]), (2, [4])], 50, seed=0)
    cu, seg = torch.from_numpy(arrays["cu"]), torch.from_numpy(arrays["segment_ids"])
    plan = block_plan(cu, seg, window=4, device=torch.device("cpu"))
    want = oracle.packed.block_plan(arrays["cu"], arrays["segment_ids"], 4)
    assert plan.q_cu.tolist() == want["q_cu"].tolist() == [0, 5, 11, 13, 16, 18, 22]
    assert plan.g_rows.tolist() == want["g_rows"].tolist()
    assert plan.s_rows.tolist() == want["s_rows"].tolist()
    # the second sequence's first branch sees its whole shared block globally, its last 3 rows in sliding layers
    assert plan.g_rows[11:19].tolist() == [5, 6, 7, 8, 9, 10, 11, 12]
    assert plan.s_rows[11:16].tolist() == [8, 9, 10, 11, 12]
    bad = seg.clone()
    bad[5:11] = 1  # a sequence starting with branch 1 has no shared block
    with pytest.raises(ValueError):
        block_plan(cu, bad, 4, torch.device("cpu"))


def test_marker_bounds_plan_markers_per_virtual_sequence_and_refuse_bad_ones():
    """The reference's readout rule for block layouts (families/gemma/packed.py:136-143): per block or branch at most
    one marker, at its last token; the shared block of a branched sequence reads out none."""
    import pytest

    from karpo_decision_b200.plan import block_plan, marker_bounds
    from karpo_decision_b200.synthetic import synthetic_block_arrays

    arrays = synthetic_block_arrays([(5, []), (6, [2, 3]), (2, [4])], 50, seed=0)
    cu, seg = torch.from_numpy(arrays["cu"]), torch.from_numpy(arrays["segment_ids"])
    plan = block_plan(cu, seg, window=4, device=torch.device("cpu"), markers_cpu=arrays["markers"])
    # virtual sequences [0,5) [5,11) [11,13) [13,16) [16,18) [18,22): markers 4, 12, 15, 21
    assert arrays["markers"].tolist() == [4, 12, 15, 21]
    assert plan.m_cu.tolist() == [0, 1, 1, 2, 3, 3, 4]
    assert marker_bounds([0, 5, 9], np.array([4, 8])) == [0, 1, 2]
    assert marker_bounds([0, 5, 9], np.array([8])) == [0, 0, 1]  # a block may read out nothing
    with pytest.raises(ValueError):
        marker_bounds([0, 5, 9], np.array([3, 8]))  # not the block's last token
    with pytest.raises(ValueError):
        marker_bounds([0, 5, 9], np.array([4, 7, 8]))  # two markers in one block


def test_packed_plan_refuses_what_the_reference_refuses():
    """``Packed.plan`` on the host (no kernel runs): Qwen refuses block layouts (families/qwen/packed.py:180-181),
    Gemma refuses a sequence with several markers or one before its last token."""
    import pytest

    from karpo_decision_b200.packed import Packed

    cpu = torch.device("cpu")
    qwen = Spec("qwen", 1, 256, 4, 2, 64, 256, 64)
    model = Packed(qwen, numpy_weights(qwen, 0), cpu)
    arrays = synthetic_pack_arrays([5, 7], qwen.vocab, seed=0, markers_per_seq=(1, 3))
    assert model.plan(from_arrays(arrays, cpu)) is None
    with pytest.raises(ValueError):
        model.plan(from_arrays({**arrays, "segment_ids": np.zeros(12, dtype=np.int64)}, cpu))
    gemma = Spec("gemma", 1, 256, 4, 2, 64, 256, 64, window=4, attention="bidirectional")
    model = Packed(gemma, numpy_weights(gemma, 0), cpu)
    assert model.prune_last and model.full_window == (-1, -1)
    good = synthetic_pack_arrays([5, 7], gemma.vocab, seed=0)
    assert model.plan(from_arrays(good, cpu)) is None
    two = dict(good, markers=np.array([3, 4, 11]), marker_cu=np.array([0, 2, 3]))
    with pytest.raises(ValueError):
        model.plan(from_arrays(two, cpu))
    early = dict(good, markers=np.array([2, 11]))
    with pytest.raises(ValueError):
        model.plan(from_arrays(early, cpu))


def test_image_plan_matches_oracle_and_refuses_what_the_reference_refuses():
    """Image rows and key rows (families/gemma/vision.py:160-196) against the oracle's plan, and the refusals: a pack
    with images but no soft token, an image longer than the sliding window."""
    import pytest

    import oracle
    from karpo_decision_b200.plan import image_plan
    from karpo_decision_b200.synthetic import synthetic_block_arrays

    arrays = synthetic_block_arrays([(40, []), (30, [12, 20]), (25, [])], 100, seed=0)
    ids = arrays["input_ids"].copy()
    ids[ids == 99] = 0
    for row, length in [(10, 13), (45, 10), (85, 12), (102, 9)]:
        ids[row:row + length] = 99
    plan = image_plan(ids, arrays["cu"].tolist(), arrays["segment_ids"], arrays["seqpos"], 99, 16,
                      torch.device("cpu"))
    spans = oracle.packed.image_spans(dict(arrays, input_ids=ids, image_token=99), 16)
    assert plan.q_cu.tolist() == [0, 13, 23, 35, 44] and plan.max_q == 13
    assert plan.keys.tolist() == np.concatenate([seen for _, _, seen in spans]).tolist()
    # the branch image (rows 85..96, positions 33..44) sees shared positions 18..29 and its branch rows 82..96
    assert plan.keys[plan.k_cu[2]:plan.k_cu[3]].tolist() == [*range(58, 70), *range(82, 97)]
    with pytest.raises(ValueError):
        image_plan(arrays["input_ids"] % 50, arrays["cu"].tolist(), arrays["segment_ids"], arrays["seqpos"], 99, 16,
                   torch.device("cpu"))
    long = ids.copy()
    long[0:17] = 99
    with pytest.raises(ValueError):
        image_plan(long, arrays["cu"].tolist(), arrays["segment_ids"], arrays["seqpos"], 99, 16, torch.device("cpu"))


def test_smoke_packs_pass_the_host_plan():
    """The packs of ``__graft_entry__.smoke`` satisfy the host planning rules the forward enforces before any kernel
    is queued (a Gemma block's readout marker is its last token, one per block)."""
    import __graft_entry__
    from karpo_decision_b200.plan import marker_bounds

    for spec, arrays in __graft_entry__.smoke_cases():
        cu = np.asarray(arrays["cu"], dtype=np.int64)
        assert len(arrays["markers"]) >= len(cu) - 1
        if spec.family == "gemma":
            marker_bounds(cu.tolist(), np.asarray(arrays["markers"]))


def test_microbench_work_counts():
    """The micro-benchmark's algorithmic work: visible query-key pairs under the varlen contract's windows."""
    from karpo_decision_b200.microbench import parse_lengths, visible_pairs
    assert visible_pairs([4], (-1, 0)) == 10           # causal: L(L+1)/2
    assert visible_pairs([4], (1, 0)) == 1 + 2 + 2 + 2  # sliding window of 2
    assert visible_pairs([3, 2], (-1, -1)) == 9 + 4     # bidirectional: L^2
    assert visible_pairs([5], (0, 1)) == 2 + 2 + 2 + 2 + 1
    assert sum(parse_lengths("mix:65536")) == 65536 and parse_lengths("8192,4096") == [8192, 4096]


def test_fine_buckets_cover_every_size_with_bounded_padding():
    """The graph buckets (the reference's fine bands, serve/qwen_graphs.py:171): the first bucket holding a pack
    pads it by at most 64 tokens up to 2,048 and by at most a sixteenth beyond; the list stops at that bucket."""
    from karpo_decision_b200.graphs import DEFAULT_BUCKETS, fine_buckets
    assert len(DEFAULT_BUCKETS) == 112 and DEFAULT_BUCKETS[0] == 64 and DEFAULT_BUCKETS[-1] == 65536
    for n in (1, 63, 64, 65, 2047, 2048, 2049, 5000, 32769, 65536):
        b = fine_buckets(n)
        assert b[-1] >= n and (len(b) == 1 or b[-2] < n)
        assert b[-1] - n < 64 if n <= 2048 else (b[-1] - n) * 16 <= n
    with pytest.raises(ValueError):
        fine_buckets(65537)


def test_block_and_image_plans_match_oracle_on_random_layouts():
    """Random block layouts (1-5 sequences, 0-3 branches each, windows 1..49) and random image runs inside them:
    the vectorized host plans equal the oracle's sequence-by-sequence restatement row for row."""
    import oracle
    from karpo_decision_b200.plan import block_plan, image_plan
    from karpo_decision_b200.synthetic import synthetic_block_arrays

    rng = np.random.default_rng(0)
    cpu = torch.device("cpu")
    checked_images = 0
    for trial in range(200):
        layouts = [(int(rng.integers(1, 40)), [int(rng.integers(1, 30)) for _ in range(int(rng.integers(0, 4)))])
                   for _ in range(int(rng.integers(1, 6)))]
        a = synthetic_block_arrays(layouts, 100, seed=trial)
        window = int(rng.integers(1, 50))
        plan = block_plan(torch.from_numpy(a["cu"]), torch.from_numpy(a["segment_ids"]), window, cpu,
                          markers_cpu=a["markers"])
        want = oracle.packed.block_plan(a["cu"], a["segment_ids"], window)
        assert plan.q_cu.tolist() == want["q_cu"].tolist()
        assert plan.g_rows.tolist() == want["g_rows"].tolist() and plan.s_rows.tolist() == want["s_rows"].tolist()
        # one image run starting at a random row, cut at its block's end and at the window
        ids, seg, cu = a["input_ids"].copy(), a["segment_ids"], set(a["cu"].tolist())
        ids[ids == 99] = 0
        w_img = int(rng.integers(8, 40))
        s = int(rng.integers(0, len(ids)))
        e = s + 1
        while e < len(ids) and e - s < int(rng.integers(1, w_img + 1)) and seg[e] == seg[s] and e not in cu:
            e += 1
        ids[s:e] = 99
        plan = image_plan(ids, a["cu"].tolist(), seg, a["seqpos"], 99, w_img, cpu)
        spans = oracle.packed.image_spans(dict(a, input_ids=ids, image_token=99), w_img)
        assert plan.keys.tolist() == np.concatenate([seen for _, _, seen in spans]).tolist()
        checked_images += 1
    assert checked_images == 200


def test_mrope_pair_axes_and_oracle_tables_follow_transformers():
    """Spec.pair_axes (the axis each rotary pair reads, which kd_rope_table_axes takes) and the oracle's M-RoPE tables
    against Transformers' own Qwen3_5TextRotaryEmbedding on the host, over positions whose three axes differ."""
    import torch
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding

    import oracle

    for head_dim, partial, sections in ((256, 0.25, (11, 11, 10)), (64, 1.0, (12, 10, 10))):
        spec = Spec("qwen", 1, 256, 2, 1, head_dim, 512, 1024, partial_rotary=partial, mrope_section=sections)
        config = Qwen3_5TextConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=head_dim,
                                   rope_parameters={"rope_type": "default", "rope_theta": 1e7,
                                                    "partial_rotary_factor": partial,
                                                    "mrope_section": list(sections)})
        module = Qwen3_5TextRotaryEmbedding(config)
        rng = np.random.default_rng(3)
        pos = rng.integers(0, 500, size=(3, 200))
        # which axis each pair reads: positions that differ on one axis only move exactly that axis's pairs
        axes = spec.pair_axes()
        for axis in range(3):
            shifted = pos.copy()
            shifted[axis] += 1
            def freqs(p):  # the module's own layout: (3, batch, tokens, pairs), then its interleaving
                f = (module.inv_freq[None, None, :, None].expand(3, 1, -1, 1).float()
                     @ torch.from_numpy(p)[:, None, None, :].float()).transpose(2, 3)
                return module.apply_interleaved_mrope(f, list(sections))

            moved = (freqs(pos) != freqs(shifted)).any(dim=1).reshape(-1).numpy()  # per frequency pair
            assert moved.tolist() == [x == axis for x in axes], (head_dim, axis)
        cos, sin = module(torch.zeros(1), torch.from_numpy(pos)[:, None, :])
        want_cos, want_sin = oracle.packed.mrope_tables(pos, head_dim, 1e7, partial, sections, "fp32")
        # float32 angles up to position 500: the two inv_freq computations may differ in the last bit
        assert np.abs(cos[0].numpy() - want_cos).max() < 1e-4 and np.abs(sin[0].numpy() - want_sin).max() < 1e-4


def test_bench_latency_of_one_sequence_configurations_is_the_step():
    """Configuration 5(a)'s requests (one 131,072-token sequence) are longer than the largest graph bucket: the bench
    reports the step as their latency instead of building graphs for them; the other configurations' request lengths
    all fit a bucket."""
    import types

    import bench
    from karpo_decision_b200.graphs import fine_buckets

    model = types.SimpleNamespace(spec=CONFIGS["gemma-31b"])
    out = bench.request_latency(model, None, "gemma-31b@131k", torch.device("cpu"), 4)
    assert out["requests"] == 0 and "step" in out["note"]
    for config, (_, (low, high), _) in bench.WORKLOADS.items():
        if "@" not in config:
            assert high <= fine_buckets(65536)[-1], config
