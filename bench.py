"""Packed prefill throughput of the B200 path (and of the reference's CPU path with ``--impl reference``).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config qwen-0.8b] [--fp8] [--impl ours|reference]

A step is one packed forward + readout over one pack of the configuration's token count (BASELINE config 2 by
default: the 0.8B-class Qwen-shaped decoder, packs of 65,536 tokens, lengths log-uniform in [128, 8192], 1-4 readout
markers per sequence; random-init bf16 weights and synthetic token ids). Rank r of N runs its own stream of packs
(replicas: one model per GPU, no collective on the data path; the routing of the reference's server is host-side),
so per-GPU work is fixed as N grows. ``value`` is all ranks' tokens over the slowest rank's device time with the
pack already resident; ``e2e`` is the same through the public API with the pack copied from pinned host memory and
the logits read back inside the timed region. Rank 0 prints one JSON line.
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
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="target CPU time of the baseline sample")
    ap.add_argument("--graphs", action="store_true", help="time the CUDA-graph path (one bucket at the pack size)")
    ap.add_argument("--requests", type=int, default=16, help="single requests timed for the latency figures")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per pack (default: the configuration's; smaller "
                                                          "packs are for profiling captures)")
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


# ------------------------------------------------------------------------------------------------ CPU baseline


_CPU_WEIGHTS: dict = {}


def cpu_sample_rate(config: str, seconds: float, fp8: bool = False) -> dict:
    """The reference algorithm on the host cores (the oracle port, float32, all BLAS threads): packs of a few short
    sequences of the same model until about ``seconds`` of CPU work; returns tokens/s and what the sample was."""
    import oracle
    from karpo_decision_b200.synthetic import CONFIGS, numpy_weights, synthetic_lengths, synthetic_pack_arrays

    spec = CONFIGS[model_of(config)]
    if config not in _CPU_WEIGHTS:  # drawn once per process: a full-size draw takes seconds
        _CPU_WEIGHTS[config] = numpy_weights(spec, 0)
    weights = _CPU_WEIGHTS[config]
    forward = oracle.qwen_forward if spec.family == "qwen" else oracle.gemma_forward
    tokens_done, elapsed, packs = 0, 0.0, 0
    seed = 100
    while elapsed < seconds or packs == 0:
        lengths = synthetic_lengths(256, 32, 256, seed, log_uniform=True)
        arrays = synthetic_pack_arrays(lengths, spec.vocab, seed + 1, markers_per(spec))
        start = time.perf_counter()
        hidden = forward(weights, spec.as_dict(), arrays, mode="fp32", fp8=fp8)
        oracle.readout(hidden, weights["readout"], spec.logit_cap)
        elapsed += time.perf_counter() - start
        tokens_done += len(arrays["input_ids"])
        packs += 1
        seed += 1
    threads = _blas_threads()
    return {"value": tokens_done / elapsed, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{packs} packs of 256 tokens (lengths log-uniform [32,256]) through the full {config} model "
                      f"({spec.layers} layers), numpy float32 oracle, {elapsed:.1f} s"}


def _blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        return max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        return os.cpu_count() or 1


def run_reference(args: argparse.Namespace) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    per_step = max(args.cpu_seconds / max(args.steps, 1), 1.0)
    for _ in range(args.warmup):
        cpu_sample_rate(args.config, 0.0, args.fp8)
    rates = [cpu_sample_rate(args.config, per_step, args.fp8) for _ in range(args.steps)]
    value = statistics.median(r["value"] for r in rates)
    tokens, _, _ = WORKLOADS[args.config]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": tokens / value * 1000.0,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32" if not args.fp8 else "e4m3",
        "data": "synthetic", "config": config_block(args, world=1),
        "cpu_baseline": {**rates[0], "value": value},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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


# ------------------------------------------------------------------------------------------------ GPU arm


def run_ours(args: argparse.Namespace) -> None:
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        group = dist

    from karpo_decision_b200 import Packed, Readout, from_arrays, ops, profile
    from karpo_decision_b200.synthetic import CONFIGS, device_weights

    spec = CONFIGS[model_of(args.config)]
    weights = device_weights(spec, 0, dev)
    model = Packed(spec, weights, dev, fp8=args.fp8)
    head = Readout(weights["readout"].float(), spec.logit_cap, dev)
    del weights
    arrays = workload(args.config, seed=1000 + rank, tokens=args.tokens)
    tokens = len(arrays["input_ids"])
    p = from_arrays(arrays, dev)
    torch.cuda.synchronize()

    forward = model
    if args.graphs:
        from karpo_decision_b200.graphs import Graphs

        forward = Graphs(model, buckets=(tokens,), max_sequences=len(arrays["cu"]) + 8)

    def step():
        return head(forward(p))

    def barrier():
        if group is not None:
            group.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    ops.check_status(dev)
    barrier()

    # ---- device-timed steps (pack resident), per-kernel events on the launching stream
    stream = torch.cuda.current_stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks, profile.kernels(stream) as prof:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    ops.check_status(dev)

    # ---- end to end through the public API: pinned host pack -> device -> forward -> readout -> host logits
    pinned = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in arrays.items()}
    h2d = sum(t.numel() * t.element_size() for t in pinned.values())
    out_host = torch.empty(len(arrays["markers"]), spec.codes, dtype=torch.float32).pin_memory()
    d2h = out_host.numel() * 4

    def e2e_step():
        q = from_pinned(pinned, dev, arrays)
        logits = head(forward(q))
        out_host.copy_(logits, non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps

    ms, e2e_ms, value, e2e_value = aggregate([ms, e2e_ms], tokens, world, dev, group)

    if rank == 0:
        peaks = peak_numbers()
        launches = prof.launches // args.steps
        # GEMMs (projections, the fused QKV one included): FLOPs from each launch's M, N, K
        gemm = prof.summary("gemm")
        qkv = prof.summary("qkv_projection")
        g_ms = (gemm["mean_ms"] or 0) * gemm["launches"] + (qkv["mean_ms"] or 0) * qkv["launches"]
        g_flops = gemm["flops_per_launch"] * gemm["launches"] + qkv["flops_per_launch"] * qkv["launches"]
        gemm_tf = g_flops / (g_ms / 1000.0) / 1e12 if g_ms else None
        # attention: algorithmic FLOPs of the pack's visible (query, key) pairs, 4 * head_dim per pair and head
        attn = prof.summary("attention")
        a_ms = (attn["mean_ms"] or 0) * attn["launches"]
        a_flops = attention_flops(spec, np.diff(arrays["cu"])) * args.steps
        attn_tf = a_flops / (a_ms / 1000.0) / 1e12 if a_ms else None
        kernels = {
            "attention": {"kernel": "kd_attention_varlen", "bound": "tensor", "achieved": attn_tf,
                          "ms_per_step": a_ms / args.steps, "traffic": traffic("attention", args, tokens)},
            "gemm": {"kernel": "kd_gemm_bf16 + kd_qkv_projection" if not args.fp8 else
                     "kd_gemm_fp8 + kd_qkv_projection_fp8", "bound": "tensor", "achieved": gemm_tf,
                     "ms_per_step": g_ms / args.steps, "traffic": traffic("gemm", args, tokens)},
        }
        # Each family against its own dense peak: bf16 for attention and bf16 GEMMs; e4m3 GEMMs run at twice the bf16
        # rate on tcgen05 (MEASURED_PEAKS.json holds no FP8 figure, so theirs is twice the measured bf16 one).
        for k, v in kernels.items():
            fp8_family = args.fp8 and k == "gemm"
            v["peak"] = peaks[0] * (2.0 if fp8_family else 1.0)
            v["peak_source"] = ("2 x " if fp8_family else "") + peaks[1]
            v["frac"] = v["achieved"] / v["peak"] if v["achieved"] else None
        dominant = max(kernels, key=lambda k: kernels[k]["ms_per_step"])
        top = kernels[dominant]
        achieved = top["achieved"]
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3" if args.fp8 else "bf16", "data": "synthetic",
            "config": config_block(args, world),
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "roofline": {"bound": "tensor", "kernel": top["kernel"], "achieved": achieved, "peak": top["peak"],
                         "unit": "TFLOP/s", "frac": top["frac"], "traffic": top["traffic"],
                         "peak_source": top["peak_source"]},
            "roofline_kernels": kernels,
            "kernel_shares": prof.shares(),
            "clocks": clocks.summary(),
        }
        if args.requests > 0:
            line["latency"] = request_latency(model, head, args, dev, args.requests)
        if world == 1 and os.environ.get("KD_BENCH_NO_CPU") != "1":
            line["cpu_baseline"] = cpu_sample_rate(args.config, args.cpu_seconds, args.fp8)
        print(json.dumps(line), flush=True)
    if group is not None:
        group.destroy_process_group()


def aggregate(times_ms: list[float], tokens: int, world: int, device, group=None) -> tuple[float, float, float, float]:
    """The slowest rank's device times (a MAX all-reduce over the ranks; identity on one rank) and the whole-job
    throughputs: every rank processed ``tokens`` per step, so tokens * world / slowest time."""
    import torch

    t = torch.tensor(times_ms, dtype=torch.float64, device=device)
    if group is not None and world > 1:
        group.all_reduce(t, op=group.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    return ms, e2e_ms, tokens * world / (ms / 1000.0), tokens * world / (e2e_ms / 1000.0)


def request_latency(model, head, args, dev, n: int) -> dict:
    """Per-request latency of single requests (one sequence each, length drawn from the configuration's range,
    1-4 questions): pinned host pack -> device -> forward -> readout -> host logits, device-synchronized wall time
    per request (the reference's latency definition, serve/engine.py:53-55, from the packed pass on), on the plain
    path and on the CUDA-graph path (the fine buckets up to the longest request)."""
    import torch

    from karpo_decision_b200.graphs import Graphs, fine_buckets
    from karpo_decision_b200.synthetic import CONFIGS, synthetic_lengths, synthetic_pack_arrays

    spec = CONFIGS[model_of(args.config)]
    _, (low, high), log = WORKLOADS[args.config]
    rng = np.random.default_rng(7)
    requests = []
    for i in range(n):
        length = synthetic_lengths(high, low, high, seed=int(rng.integers(1 << 30)), log_uniform=log)[0]
        requests.append(synthetic_pack_arrays([length], spec.vocab, seed=i, markers_per_seq=markers_per(spec)))
    longest = max(len(r["input_ids"]) for r in requests)
    graphs = Graphs(model, buckets=fine_buckets(longest), max_sequences=1)
    out = {"requests": n, "lengths": f"one sequence each, {'log-uniform' if log else 'uniform'} [{low},{high}]"}
    for name, fwd in (("plain", model), ("graphs", graphs)):
        times = []
        for arrays in requests + requests[:2]:  # the first two again: warm-up excluded below
            pinned = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in arrays.items()}
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            logits = head(fwd(from_pinned(pinned, dev, arrays))).cpu()
            torch.cuda.synchronize()
            times.append((time.perf_counter() - t0) * 1000.0)
            del logits
        times = times[2:]
        out[name] = {"p50_ms": round(float(np.median(times)), 3), "p90_ms": round(float(np.percentile(times, 90)), 3),
                     "mean_ms": round(float(np.mean(times)), 3)}
    graphs.release()
    return out


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


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from ncu captures of the same kernels on an
# 8,192-token pack of the same configuration, scaled to the bench's pack by tokens (every operand moves once per
# launch): attention (one layer's launch), and the GEMM family as the mean of one layer's four launches (QKV + norm +
# RoPE, o_proj + residual, gate/up + SwiGLU, down + residual).
TRAFFIC_CAPTURES = {("qwen-0.8b", "attention"): (8192, 100.882432e6 + 14.541056e6),
                    ("qwen-0.8b", "gemm"): (8192, (31.640064e6 + 52.296192e6 + 54.548992e6 + 0.698880e6 + 29.403648e6 +
                                                   6.410752e6 + 73.426176e6 + 3.883264e6) / 4)}


def traffic(kernel: str, args, tokens: int) -> float | None:
    capture = TRAFFIC_CAPTURES.get((args.config, kernel))
    if capture is None or args.fp8:
        return None
    captured_tokens, nbytes = capture
    return nbytes * tokens / captured_tokens


def from_pinned(pinned: dict, dev, arrays: dict):
    import torch

    from karpo_decision_b200.pack import Pack

    cu = arrays["cu"]
    counts = np.diff(arrays["marker_cu"])
    return Pack(
        input_ids=pinned["input_ids"].to(dev, non_blocking=True),
        seqpos=pinned["seqpos"].to(dev, non_blocking=True),
        cu=pinned["cu"].to(dev, torch.int32, non_blocking=True),
        cu_cpu=torch.from_numpy(np.asarray(cu, dtype=np.int64)),
        max_length=int(np.diff(cu).max()),
        markers=pinned["markers"].to(dev, non_blocking=True),
        marker_cu=pinned["marker_cu"].to(dev, torch.int32, non_blocking=True),
        max_markers=int(counts.max()),
    )


def peak_numbers() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        if "bf16_tflops_sustained" in data:
            return float(data["bf16_tflops_sustained"]), "MEASURED_PEAKS.json bf16_tflops_sustained (of measured)"
    return 1400.0, "fallback 1.4 PFLOP/s sustained (of fallback)"


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
