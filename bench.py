"""Packed prefill throughput of the B200 path (and of the reference's CPU path with ``--impl reference``).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config qwen-0.8b] [--fp8] [--graphs]
                    [--impl ours|reference] [--no-extra] [--no-routed]

A step is one packed forward + readout over one pack of the configuration's token count (BASELINE config 2 by
default: the 0.8B-class Qwen-shaped decoder, packs of 65,536 tokens, lengths log-uniform in [128, 8192], 1-4 readout
markers per sequence; random-init bf16 weights and synthetic token ids). Under torchrun every rank runs its own
stream of packs (replicas: one model per GPU, no collective on the data path), so per-GPU work is fixed as N grows.
``value`` is all ranks' tokens over the slowest rank's device time with the pack resident; ``e2e`` is the same through
the public API in wall-clock time per step: the pack built from host arrays (pinned, copied to the device), forward,
readout, logits read back, a synchronize per step. Rank 0 prints one JSON line, which also carries:

- ``roofline``: the single kernel with the largest share of the step's device time, its algorithmic FLOPs over its
  CUDA-event time against the measured peak; ``roofline_families`` sums the GEMM and attention kernels;
- ``extra_configs`` (N = 1): BASELINE configs 3-5 (qwen-4b FP8, gemma-12b bf16, gemma-31b FP8, 32,768-token packs)
  with their own rooflines and clocks, and per-request p50/p90 latency on the 12B and 31B shapes, plain and graphs;
- ``routed`` (every N): BASELINE config 5(b), a stream of requests (lengths log-uniform in [256, 32768], 1-4
  questions each) dispatched from rank 0 to the replica with the fewest in flight (``karpo_decision_b200.replicas``);
- ``cpu_baseline`` (N = 1): the reference's algorithm on the host cores (``--impl reference`` below).

``--impl reference`` times the reference's plain path on the host cores (oracle/cpu_reference.py, its layers restated
in torch, float32, every host thread) on this configuration's real pack: each step runs the embedding, one layer of
each kind and the head over the whole pack; ``value`` scales the layer times by the layer counts.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "packed prefill tokens/s"
WORKLOADS = {
    # config: (tokens per pack, length range, log-uniform); the model is the configuration's name up to any "@"
    "tiny": (2048, (32, 512), False),
    "qwen-0.8b": (65536, (128, 8192), True),
    "qwen-4b": (32768, (256, 16384), True),
    "gemma-12b": (32768, (512, 32768), True),
    "gemma-31b": (32768, (256, 32768), True),
    "gemma-31b@131k": (131072, (131072, 131072), False),  # one 131,072-token sequence
}
#: BASELINE configs 3-5 measured beside the headline (model, FP8, latency requests or 0)
EXTRA = (("qwen-4b", True, 0), ("gemma-12b", False, 12), ("gemma-31b", True, 12))
#: The routed stream (config 5(b)): model, FP8, request lengths, questions per request
ROUTED = ("gemma-31b", True, (256, 32768), (1, 4))


def model_of(config: str) -> str:
    """The synthetic model a bench configuration runs."""
    return config.split("@")[0]


def parse() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="qwen-0.8b", choices=sorted(WORKLOADS))
    ap.add_argument("--fp8", action="store_true")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--graphs", action="store_true", help="time the CUDA-graph path (one bucket at the pack size)")
    ap.add_argument("--requests", type=int, default=16, help="single requests timed for the latency figures")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per pack (default: the configuration's; smaller "
                                                          "packs are for profiling captures)")
    ap.add_argument("--no-extra", action="store_true", help="skip the BASELINE configs 3-5 block")
    ap.add_argument("--no-routed", action="store_true", help="skip the routed request stream")
    ap.add_argument("--routed-requests", type=int, default=16, help="routed requests per GPU")
    ap.add_argument("--cpu-layers", type=int, default=1, help="reference arm: layers of each kind timed per step")
    return ap.parse_args()


def workload(config: str, seed: int, tokens: int = 0) -> dict:
    from karpo_decision_b200.synthetic import CONFIGS, synthetic_lengths, synthetic_pack_arrays

    default, (low, high), log = WORKLOADS[config]
    tokens = tokens or default
    spec = CONFIGS[model_of(config)]
    lengths = synthetic_lengths(tokens, low, high, seed, log_uniform=log)
    return synthetic_pack_arrays(lengths, spec.vocab, seed + 1, markers_per(spec))


def markers_per(spec) -> tuple[int, int]:
    """Readout markers per sequence: 1-4 (Qwen's joint layouts, tests/gpu/test_packed_qwen.py:52-60); Gemma reads
    out one marker per block, at its last token (families/gemma/packed.py:136-143)."""
    return (1, 4) if spec.family == "qwen" else (1, 1)


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def config_block(args: argparse.Namespace, world: int) -> dict:
    tokens, (low, high), log = WORKLOADS[args.config]
    tokens = args.tokens or tokens
    from karpo_decision_b200.synthetic import CONFIGS

    lo, hi = markers_per(CONFIGS[model_of(args.config)])
    return {"workload": f"{args.config} packed prefill, packs of {tokens} tokens, lengths "
                        f"{'log-uniform' if log else 'uniform'} [{low},{high}], {lo}-{hi} markers/sequence, causal"
                        + (", FP8 projections" if args.fp8 else ""),
            "tokens_per_pack": tokens, "parallelism": f"replicas x{world}",
            "path": "graphs" if getattr(args, "graphs", False) else "plain",
            "l2": "working set (weights and per-layer activations) larger than L2 between steps"}


# ------------------------------------------------------------------------------------------------ CPU baseline


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference_sample(config: str, layers_per_kind: int = 1, seed: int = 1000) -> dict:
    """One step of the reference's plain path on the host cores over the configuration's real pack: the embedding,
    ``layers_per_kind`` layers of each layer kind and the head, timed separately. Returns the timed milliseconds and
    the whole-model time estimate (layer times scaled by the layer counts)."""
    import torch

    from karpo_decision_b200.synthetic import CONFIGS, numpy_weights, small
    from oracle.cpu_reference import Model

    torch.set_num_threads(host_cores())
    spec = CONFIGS[model_of(config)]
    kinds = spec.layer_types()
    counts = {k: kinds.count(k) for k in set(kinds)}
    # the first layers of each kind: Qwen's first layers, Gemma's first 5 sliding and its first global (layer 5)
    needed = max(kinds.index(k) for k in counts) + 1 if layers_per_kind == 1 else min(spec.layers, 6 * layers_per_kind)
    key = (config, needed)
    if key not in _CPU_MODELS:
        _CPU_MODELS.clear()
        sub = small(spec, layers=needed)
        _CPU_MODELS[key] = Model(numpy_weights(sub, 0), sub.as_dict())
    model = _CPU_MODELS[key]
    arrays = workload(config, seed)
    tokens = len(arrays["input_ids"])
    ids = torch.from_numpy(arrays["input_ids"])
    seqpos = torch.from_numpy(arrays["seqpos"])
    cu = [int(x) for x in arrays["cu"]]
    markers = torch.from_numpy(arrays["markers"])
    with torch.inference_mode():
        t0 = time.perf_counter()
        tables = model.tables(seqpos)
        h = model.embed(ids)
        t_rest = time.perf_counter() - t0
        per_kind: dict[str, list[float]] = {k: [] for k in counts}
        sub_kinds = model.layer_kinds()
        for i in range(needed):
            if len(per_kind[sub_kinds[i]]) >= layers_per_kind:
                continue
            t0 = time.perf_counter()
            h = model.layer(i, h, tables, cu)
            per_kind[sub_kinds[i]].append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        model.head(h, markers)
        t_rest += time.perf_counter() - t0
    timed = t_rest + sum(sum(v) for v in per_kind.values())
    whole = t_rest + sum(counts[k] * statistics.mean(v) for k, v in per_kind.items())
    return {"tokens": tokens, "timed_s": timed, "model_s": whole,
            "layers_timed": {k: len(v) for k, v in per_kind.items()}, "layer_counts": counts}


_CPU_MODELS: dict = {}


def cpu_baseline_block(config: str, samples: list[dict]) -> dict:
    tokens = samples[0]["tokens"]
    model_s = statistics.median(s["model_s"] for s in samples)
    timed = ", ".join(f"{n} of {samples[0]['layer_counts'][k]} {k}" for k, n in samples[0]["layers_timed"].items())
    import torch

    return {"value": tokens / model_s, "unit": "tokens/s", "cores": host_cores(), "threads": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{len(samples)} step(s), each the embedding, {timed} layer(s) and the head over the real "
                      f"{tokens}-token {config} pack (the bench's workload) through oracle/cpu_reference.py (the "
                      f"reference's layers restated in torch, float32, {torch.get_num_threads()} threads); the "
                      f"whole-model time scales the layer times by the layer counts ({model_s:.1f} s per pack)"}


def run_reference(args: argparse.Namespace) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_reference_sample(args.config, args.cpu_layers)
    samples = [cpu_reference_sample(args.config, args.cpu_layers) for _ in range(args.steps)]
    block = cpu_baseline_block(args.config, samples)
    timed_ms = statistics.mean(s["timed_s"] for s in samples) * 1000.0
    cfg = config_block(args, world=1)
    cfg["workload"] += (f"; reference arm: per step the embedding, {args.cpu_layers} layer(s) of each kind and the "
                        f"head over the whole pack, value scaled to all {samples[0]['layer_counts']} layers")
    line = {
        "impl": "reference", "metric": METRIC, "value": block["value"], "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": timed_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": cfg, "cpu_baseline": block,
        "e2e": {"value": block["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ clocks


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.lines: list[str] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8], strict=False):
                if flag.lower() in ("active", "1", "yes"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ rooflines

#: Kernels whose work is a GEMM (FLOPs from each launch's M, N, K) and the attention kernel (FLOPs of the pack's
#: visible pairs).
GEMM_KERNELS = ("kd_gemm_bf16", "kd_qkv_projection", "kd_gemm_fp8", "kd_qkv_projection_fp8")
ATTENTION = "kd_attention_varlen"

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from ncu captures of the same kernels on an
# 8,192-token pack of the same configuration, scaled to the bench's pack by tokens (every operand moves once per
# launch): attention (one layer's launch), and the GEMM family as the mean of one layer's four launches (QKV + norm +
# RoPE, o_proj + residual, gate/up + SwiGLU, down + residual).
TRAFFIC_CAPTURES = {("qwen-0.8b", ATTENTION): (8192, 100.882432e6 + 14.541056e6),
                    ("qwen-0.8b", "gemm"): (8192, (31.640064e6 + 52.296192e6 + 54.548992e6 + 0.698880e6 + 29.403648e6 +
                                                   6.410752e6 + 73.426176e6 + 3.883264e6) / 4)}


def traffic(config: str, fp8: bool, kernel: str, tokens: int) -> float | None:
    capture = TRAFFIC_CAPTURES.get((config, kernel))
    if capture is None or fp8:
        return None
    captured_tokens, nbytes = capture
    return nbytes * tokens / captured_tokens


def peak_numbers() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        if "bf16_tflops_sustained" in data:
            return float(data["bf16_tflops_sustained"]), "MEASURED_PEAKS.json bf16_tflops_sustained (of measured)"
    return 1400.0, "fallback 1.4 PFLOP/s sustained (of fallback)"


def attention_flops(spec, lengths) -> float:
    """FLOPs of one forward's attention over a pack: per layer, 4 * head_dim * heads per visible (query, key) pair;
    causal pairs L (L + 1) / 2 per sequence, sliding-window pairs sum_i min(i + 1, W)."""
    total = 0.0
    lengths = [int(n) for n in lengths]
    causal = sum(n * (n + 1) / 2 for n in lengths)
    w = spec.window
    sliding = sum((min(n, w) * (min(n, w) + 1)) / 2 + max(0, n - w) * w for n in lengths)
    for kind in spec.layer_types():
        total += 4.0 * spec.head_dim * spec.heads * (causal if kind == "full_attention" else sliding)
    return total


def rooflines(prof, spec, lengths, steps: int, fp8: bool, config: str, tokens: int) -> tuple[dict, dict]:
    """(roofline of the single kernel with the largest device time, per-family sums). Tensor kernels against the
    measured sustained bf16 peak; FP8 GEMMs against twice it (dense e4m3 runs at twice the bf16 rate on tcgen05 and
    MEASURED_PEAKS.json holds no FP8 figure)."""
    peak, source = peak_numbers()
    times = prof.times()
    a_flops = attention_flops(spec, lengths) * steps

    def entry(names, flops, fp8_gemm):
        ms = sum(ms for n in names for ms, _ in times.get(n, []))
        p = peak * (2.0 if fp8_gemm else 1.0)
        achieved = flops / (ms / 1000.0) / 1e12 if ms else None
        return {"kernel": " + ".join(n for n in names if n in times), "bound": "tensor", "achieved": achieved,
                "peak": p, "unit": "TFLOP/s", "frac": achieved / p if achieved else None,
                "ms_per_step": ms / steps, "peak_source": ("2 x " if fp8_gemm else "") + source}

    gemm_names = [n for n in GEMM_KERNELS if n in times]
    g_flops = sum(f for n in gemm_names for _, f in times[n])
    families = {
        "attention": dict(entry([ATTENTION], a_flops, False), traffic=traffic(config, fp8, ATTENTION, tokens)),
        "gemm": dict(entry(gemm_names, g_flops, fp8), traffic=traffic(config, fp8, "gemm", tokens)),
    }
    total = {n: sum(ms for ms, _ in rs) for n, rs in times.items()}
    top = max(total, key=total.get)
    if top == ATTENTION:
        single = dict(families["attention"])
    elif top in GEMM_KERNELS:
        single = entry([top], sum(f for _, f in times[top]), fp8 and top.endswith("fp8"))
        single["traffic"] = None
    else:  # a memory-bound kernel: reported without a FLOP roofline
        single = {"kernel": top, "bound": "hbm", "achieved": None, "frac": None, "ms_per_step": total[top] / steps}
    single["share"] = round(total[top] / sum(total.values()), 4)
    return single, families


# ------------------------------------------------------------------------------------------------ GPU arm


def build_model(config: str, fp8: bool, dev):
    import torch

    from karpo_decision_b200 import Packed, Readout
    from karpo_decision_b200.synthetic import CONFIGS, device_weights

    spec = CONFIGS[model_of(config)]
    weights = device_weights(spec, 0, dev)
    model = Packed(spec, weights, dev, fp8=fp8)
    head = Readout(weights["readout"].float(), spec.logit_cap, dev)
    del weights
    torch.cuda.empty_cache()
    return spec, model, head


def measure(config: str, fp8: bool, steps: int, warmup: int, dev, local: int, group, world: int, *,
            graphs: bool = False, tokens: int = 0, model=None, e2e: bool = True) -> tuple[dict, tuple]:
    """Device-timed steps (pack resident) and wall-clock end-to-end steps of one configuration on this rank; the
    times are the max over ranks. Returns the result block and (spec, model, head) for reuse."""
    import torch

    from karpo_decision_b200 import from_arrays, ops, profile

    rank = int(os.environ.get("RANK", 0))
    spec, model_, head = model if model is not None else build_model(config, fp8, dev)
    arrays = workload(config, seed=1000 + rank, tokens=tokens)
    n_tokens = len(arrays["input_ids"])
    p = from_arrays(arrays, dev)
    forward = model_
    graph_path = None
    if graphs:
        from karpo_decision_b200.graphs import Graphs

        graph_path = Graphs(model_, buckets=(n_tokens,), max_sequences=len(arrays["cu"]) + 8)
        forward = graph_path

    def step():
        return head(forward(p))

    def barrier():
        if group is not None:
            group.barrier()
        torch.cuda.synchronize()

    for _ in range(warmup):
        step()
    ops.check_status(dev)
    barrier()
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks, profile.kernels(stream) as prof:
        start.record(stream)
        for _ in range(steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    ops.check_status(dev)
    launches = prof.launches // steps
    single, families = rooflines(prof, spec, np.diff(arrays["cu"]), steps, fp8, config, n_tokens)

    e2e_ms = float("nan")
    h2d = d2h = 0
    if e2e:
        # wall clock per step through the public API: pack from host arrays (pinned, copied), forward, readout,
        # logits read back (the read synchronizes the step)
        h2d = sum(np.asarray(v).nbytes for k, v in arrays.items() if k in ("input_ids", "seqpos", "cu", "markers",
                                                                          "marker_cu"))
        d2h = len(arrays["markers"]) * spec.codes * 4
        for _ in range(2):
            head(forward(from_arrays(arrays, dev, pinned=True))).cpu()
        barrier()
        walls = []
        for _ in range(steps):
            t0 = time.perf_counter()
            head(forward(from_arrays(arrays, dev, pinned=True))).cpu()
            walls.append(time.perf_counter() - t0)
        e2e_ms = sum(walls) / len(walls) * 1000.0
    ms, e2e_ms, value, e2e_value = aggregate([ms, e2e_ms], n_tokens, world, dev, group)
    if graph_path is not None:
        graph_path.release()
    block = {"value": value, "unit": "tokens/s", "ms_per_step": ms, "tokens_per_pack": n_tokens,
             "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d,
                     "d2h_bytes_per_step": d2h, "timing": "wall clock per step, synchronized"},
             "gpu_launches": launches, "roofline": single, "roofline_families": families,
             "kernel_shares": prof.shares(), "clocks": clocks.summary()}
    return block, (spec, model_, head)


def aggregate(times_ms: list[float], tokens: int, world: int, device, group=None) -> tuple[float, float, float, float]:
    """The slowest rank's times (a MAX all-reduce over the ranks; identity on one rank) and the whole-job
    throughputs: every rank processed ``tokens`` per step, so tokens * world / slowest time."""
    import torch

    t = torch.tensor(times_ms, dtype=torch.float64, device=device)
    if group is not None and world > 1:
        group.all_reduce(t, op=group.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    return ms, e2e_ms, tokens * world / (ms / 1000.0), tokens * world / (e2e_ms / 1000.0)


def request_arrays(spec, lengths: list[int], questions: list[int], seed: int) -> list[dict]:
    """One request per length: Qwen a joint sequence with its questions' markers; Gemma one block with one marker,
    or for k > 1 questions a shared block followed by k branches of 16-64 tokens, one marker each (blocks.py)."""
    from karpo_decision_b200.synthetic import synthetic_block_arrays, synthetic_pack_arrays

    rng = np.random.default_rng(seed)
    out = []
    for i, (n, k) in enumerate(zip(lengths, questions, strict=True)):
        if spec.family == "qwen":
            out.append(synthetic_pack_arrays([n], spec.vocab, seed + i, (k, k)))
            continue
        if k == 1:
            out.append(synthetic_block_arrays([(n, [])], spec.vocab, seed + i))
            continue
        branches = [int(x) for x in rng.integers(16, 65, size=k)]
        out.append(synthetic_block_arrays([(max(n - sum(branches), 1), branches)], spec.vocab, seed + i))
    return out


def draw_requests(spec, count: int, low: int, high: int, questions: tuple[int, int], seed: int) -> list[dict]:
    rng = np.random.default_rng(seed)
    lengths = [int(round(math.exp(rng.uniform(math.log(low), math.log(high))))) for _ in range(count)]
    ks = [int(rng.integers(questions[0], questions[1] + 1)) for _ in range(count)]
    return request_arrays(spec, lengths, ks, seed)


def request_latency(model, head, config: str, dev, n: int) -> dict:
    """Per-request latency of single requests (one sequence each, length drawn from the configuration's range, one
    question): host arrays -> pinned -> device -> forward -> readout -> host logits, device-synchronized wall time per
    request (the reference's latency definition, serve/engine.py:53-55, from the packed pass on), on the plain path
    and on the CUDA-graph path (the fine buckets that hold the requests)."""
    import torch

    from karpo_decision_b200 import from_arrays
    from karpo_decision_b200.graphs import Graphs, fine_buckets

    spec = model.spec
    _, (low, high), log = WORKLOADS[config]
    every = fine_buckets(65536)
    if low > every[-1]:  # one sequence per pack (config 5(a)): the request is the step
        return {"requests": 0, "note": f"single requests of {low} tokens are this configuration's step (ms_per_step); "
                                       f"the graph buckets end at {every[-1]} tokens"}
    rng = np.random.default_rng(7)
    lengths = [int(round(math.exp(rng.uniform(math.log(low), math.log(high))))) if log else
               int(rng.integers(low, high + 1)) for _ in range(n)]
    requests = request_arrays(spec, lengths, [1] * n, seed=7)
    # requests longer than the largest bucket run the plain path inside the graph wrapper, as in the reference
    needed = sorted({min(b for b in every if b >= len(r["input_ids"])) for r in requests
                     if len(r["input_ids"]) <= every[-1]})
    graphs = Graphs(model, buckets=tuple(needed), max_sequences=1)
    out = {"requests": n, "lengths": f"one sequence each, {'log-uniform' if log else 'uniform'} [{low},{high}], "
                                      f"one question", "graph_buckets": len(needed)}
    for name, fwd in (("plain", model), ("graphs", graphs)):
        times = []
        for arrays in requests[:2] + requests:  # the first two once more first: warm-up, excluded
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            head(fwd(from_arrays(arrays, dev, pinned=True))).cpu()
            times.append((time.perf_counter() - t0) * 1000.0)
        times = times[2:]
        out[name] = {"p50_ms": round(float(np.median(times)), 3), "p90_ms": round(float(np.percentile(times, 90)), 3),
                     "mean_ms": round(float(np.mean(times)), 3)}
    graphs.release()
    return out


class TimedRunner:
    """``PackRunner`` that also sums each forward's device time (CUDA events on the current stream)."""

    def __init__(self, model, head, dev) -> None:
        from karpo_decision_b200.replicas import PackRunner

        self.inner = PackRunner(model, head, dev)
        self.device_ms = 0.0
        self.tokens = 0

    def run(self, arrays):
        import torch

        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        out = self.inner.run(arrays)  # reads the logits back: the step is complete
        end.record()
        end.synchronize()
        self.device_ms += start.elapsed_time(end)
        self.tokens += len(arrays["input_ids"])
        return out


def routed_stream(per_gpu: int, rank: int, world: int, dev, group, model=None) -> dict | None:
    """BASELINE config 5(b) on every rank: the gemma-31b FP8 model on each GPU, a stream of requests from rank 0 routed
    to the replica with the fewest in flight (karpo_decision_b200.replicas), 2 clients per GPU in a closed loop.
    Throughput is the stream's tokens over rank 0's wall time (the routing and hand-over are host work); each
    replica's device time is summed from CUDA events and its maximum over ranks reported beside it."""
    import torch

    from karpo_decision_b200 import replicas

    config, fp8, (low, high), questions = ROUTED
    spec, m, head = model if model is not None else build_model(config, fp8, dev)
    runner = TimedRunner(m, head, dev)
    for arrays in draw_requests(spec, 2, 2048, 2048, (1, 2), seed=99):  # warm-up on every replica
        runner.run(arrays)
    runner.device_ms, runner.tokens = 0.0, 0
    dispatcher = None
    port = torch.zeros(1, dtype=torch.int64, device=dev)
    if rank == 0:
        dispatcher = replicas.Dispatcher(runner, world, "127.0.0.1", 0)
        port.fill_(dispatcher.port)
    if group is not None and world > 1:
        group.broadcast(port, src=0)
    result = None
    if rank == 0:
        requests = draw_requests(spec, per_gpu * world, low, high, questions, seed=2024)
        dispatcher.wait_ready()
        clients = 2 * world
        lock = threading.Lock()
        queue = list(range(len(requests)))
        latency = [0.0] * len(requests)

        def client():
            while True:
                with lock:
                    if not queue:
                        return
                    i = queue.pop(0)
                t0 = time.perf_counter()
                dispatcher.run(requests[i])
                latency[i] = (time.perf_counter() - t0) * 1000.0

        t0 = time.perf_counter()
        threads = [threading.Thread(target=client) for _ in range(clients)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        wall = time.perf_counter() - t0
        stats = dispatcher.stats()
        dispatcher.close()
        tokens = sum(len(r["input_ids"]) for r in requests)
        result = {"model": config, "fp8": fp8, "requests": len(requests), "tokens": tokens, "clients": clients,
                  "lengths": f"log-uniform [{low},{high}], {questions[0]}-{questions[1]} questions each (Gemma: one "
                             f"block, or a shared block and one 16-64-token branch per question)",
                  "wall_s": round(wall, 4), "value": tokens / wall, "unit": "tokens/s",
                  "timing": "wall clock on the dispatching rank, first submit to last reply",
                  "p50_ms": round(float(np.median(latency)), 3), "p90_ms": round(float(np.percentile(latency, 90)), 3),
                  "served": stats["served"], "failed": stats["failed"], "handover_ms": stats["handover_ms"],
                  "busy_s": stats["busy_s"]}
    else:
        replicas.serve(runner, "127.0.0.1", int(port.item()), rank)
    busy = torch.tensor([runner.device_ms], dtype=torch.float64, device=dev)
    if group is not None and world > 1:
        group.all_reduce(busy, op=group.ReduceOp.MAX)
    if result is not None:
        result["device_busy_s_max"] = round(busy.item() / 1000.0, 4)
        result["device_value"] = result["tokens"] / (busy.item() / 1000.0)
    return result


def run_ours(args: argparse.Namespace) -> None:
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
        group = dist

    block, (spec, model, head) = measure(args.config, args.fp8, args.steps, args.warmup, dev, local, group, world,
                                         graphs=args.graphs, tokens=args.tokens)
    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": block["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": block["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3" if args.fp8 else "bf16", "data": "synthetic",
            "config": config_block(args, world), "e2e": block["e2e"], "gpu_launches": block["gpu_launches"],
            "roofline": block["roofline"], "roofline_families": block["roofline_families"],
            "kernel_shares": block["kernel_shares"], "clocks": block["clocks"],
        }
        if args.requests > 0:
            line["latency"] = request_latency(model, head, args.config, dev, args.requests)
    del model, head
    torch.cuda.empty_cache()

    big = None
    if world == 1 and not args.no_extra and args.config == "qwen-0.8b" and not args.tokens:
        extra = {}
        for config, fp8, latency_n in EXTRA:
            b, built = measure(config, fp8, 3, 2, dev, local, None, 1, e2e=False)
            entry = {k: b[k] for k in ("value", "unit", "ms_per_step", "tokens_per_pack", "gpu_launches", "roofline",
                                       "roofline_families", "clocks")}
            entry["dtype"] = "e4m3" if fp8 else "bf16"
            entry["workload"] = (f"{config} packed prefill, packs of {b['tokens_per_pack']} tokens, lengths "
                                 f"log-uniform {list(WORKLOADS[config][1])}, causal" + (", FP8 projections" if fp8
                                                                                        else ""))
            if latency_n:
                entry["latency"] = request_latency(built[1], built[2], config, dev, latency_n)
            extra[f"{config}{' fp8' if fp8 else ''}"] = entry
            if (config, fp8) == ROUTED[:2]:
                big = built  # the routed stream's model, already on this GPU
            else:
                del built
            torch.cuda.empty_cache()
        line["extra_configs"] = extra

    if not args.no_routed:
        routed = routed_stream(args.routed_requests, rank, world, dev, group, model=big)
        if rank == 0:
            line["routed"] = routed
    big = None
    torch.cuda.empty_cache()

    if rank == 0:
        if world == 1 and os.environ.get("KD_BENCH_NO_CPU") != "1":
            line["cpu_baseline"] = cpu_baseline_block(args.config, [cpu_reference_sample(args.config)])
        print(json.dumps(line), flush=True)
    if group is not None:
        group.barrier()
        group.destroy_process_group()


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
