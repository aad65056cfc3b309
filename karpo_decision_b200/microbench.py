"""One libkd_b200 op at a chosen shape on seeded synthetic inputs, timed with CUDA events on the current stream.
Kernel profiles are captured on it, so that a capture holds one kernel at a small size instead of a whole model:

    python -m karpo_decision_b200.microbench attention --lengths 8192 --hq 16 --hkv 8 --hd 256 --window=1023,0
    python -m karpo_decision_b200.microbench gemm --m 8192 --n 6144 --k 1024 --fp8 --epilogue swiglu
    python -m karpo_decision_b200.microbench qkv --lengths mix:8192 --k 1024 --hq 16 --hkv 8 --gate
    python -m karpo_decision_b200.microbench rmsnorm_e4m3 --rows 16384 --cols 5376
    python -m karpo_decision_b200.microbench delta_rule --lengths 8192,4096,2048,2048 --hk 16 --hv 32
    python -m karpo_decision_b200.microbench attention --lengths mix:65536 --lib fa2    # a library kernel, same inputs

``--window=left,right`` takes its value after ``=`` (``-1`` is unbounded; ``-1,0``, the default, is causal).
``--lengths`` is a comma-separated list of sequence lengths, or ``mix:T`` for T tokens of lengths log-uniform in
[128, 8192] (the bench's packs). Prints one JSON line: the op, its shape, the mean time per launch over ``--iters``
launches after two untimed ones, and the launch's algorithmic work (FLOPs for tensor-core ops, bytes read once and
written once for memory-bound ones) with the rate achieved.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import ops
from .synthetic import synthetic_lengths

EPILOGUES = {"store": ops.EPI_STORE, "swiglu": ops.EPI_SWIGLU, "geglu": ops.EPI_GEGLU, "residual": ops.EPI_RESIDUAL}


def parse_lengths(spec: str) -> list[int]:
    if spec.startswith("mix:"):
        return synthetic_lengths(int(spec[4:]), 128, 8192, 0)
    return [int(x) for x in spec.split(",")]


def visible_pairs(lengths: list[int], window: tuple[int, int]) -> int:
    """Query-key pairs the varlen contract lets attend (queries and keys of equal length per sequence)."""
    left, right = window
    total = 0
    for n in lengths:
        i = np.arange(n, dtype=np.int64)
        lo = np.maximum(0, i - left) if left >= 0 else np.zeros_like(i)
        hi = np.minimum(n - 1, i + right) if right >= 0 else np.full_like(i, n - 1)
        total += int(np.maximum(hi - lo + 1, 0).sum())
    return total


def bf16(g: torch.Generator, *shape: int, device: torch.device, scale: float = 1.0) -> torch.Tensor:
    return (torch.randn(*shape, generator=g, device="cpu") * scale).to(device=device, dtype=torch.bfloat16)


def build(args: argparse.Namespace, dev: torch.device):
    """(the launch as a closure, work per launch, the work's unit, a description of the shape)."""
    g = torch.Generator().manual_seed(args.seed)
    op = args.op
    if op == "attention":
        lengths = parse_lengths(args.lengths)
        t = sum(lengths)
        q = bf16(g, t, args.hq, args.hd, device=dev)
        k = bf16(g, t, args.hkv, args.hd, device=dev)
        v = bf16(g, t, args.hkv, args.hd, device=dev)
        gate = bf16(g, t, args.hq * args.hd, device=dev) if args.gate else None
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
        window = tuple(int(x) for x in args.window.split(","))
        out = torch.empty(t, args.hq * args.hd, dtype=torch.bfloat16, device=dev)
        scale = args.hd ** -0.5

        def run():
            ops.attention_varlen(q, k, v, cu, cu, max(lengths), scale, window, gate=gate, out=out)

        if args.lib:
            run = library_attention(args.lib, q, k, v, cu, lengths, scale, window)
        flops = 4 * args.hd * args.hq * visible_pairs(lengths, window)
        return run, flops, "FLOP", {"sequences": len(lengths), "tokens": t, "hq": args.hq, "hkv": args.hkv,
                                    "hd": args.hd, "window": list(window), "gate": bool(args.gate)}
    if op == "gemm":
        m, n, kk = args.m, args.n, args.k
        epi = EPILOGUES[args.epilogue]
        a = bf16(g, m, kk, device=dev)
        w = bf16(g, n, kk, device=dev, scale=kk ** -0.5)
        width = n // 2 if epi in (ops.EPI_SWIGLU, ops.EPI_GEGLU) else n
        res = bf16(g, m, width, device=dev) if epi == ops.EPI_RESIDUAL else None
        out = torch.empty(m, width, dtype=torch.bfloat16, device=dev)
        if args.fp8:
            qa, sa = ops.quantize_rows_e4m3(a)
            qw, sw = ops.quantize_rows_e4m3(w)

            def run():
                ops.gemm_fp8(qa, sa, qw, sw, out=out, epilogue=epi, residual=res)
        else:
            def run():
                ops.gemm(a, w, out=out, epilogue=epi, residual=res)

        if args.lib == "cublas":  # the library product alone, no epilogue: torch.matmul / rowwise torch._scaled_mm
            full = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            if args.fp8:
                sa2, sw2 = sa.view(-1, 1).contiguous(), sw.view(1, -1).contiguous()

                def run():
                    torch._scaled_mm(qa, qw.t(), scale_a=sa2, scale_b=sw2, out_dtype=torch.bfloat16, out=full)
            else:
                def run():
                    torch.matmul(a, w.t(), out=full)
        elif args.lib:
            raise SystemExit("gemm --lib takes cublas")
        return run, 2 * m * n * kk, "FLOP", {"m": m, "n": n, "k": kk, "fp8": bool(args.fp8),
                                             "epilogue": args.epilogue}
    if op == "qkv":
        # Qwen's fused projection: [q | gate] per head, k, v; q/k norms (1 + w) and RoPE over the full head in the
        # epilogue; rows are the sequences of --lengths, K = --k
        lengths = parse_lengths(args.lengths)
        t, kk, hq, hkv, hd = sum(lengths), args.k, args.hq, args.hkv, args.hd
        n = (hq * (2 if args.gate else 1) + 2 * hkv) * hd
        a = bf16(g, t, kk, device=dev)
        w = bf16(g, n, kk, device=dev, scale=kk ** -0.5)
        q_norm, k_norm = (bf16(g, hd, device=dev, scale=0.1) for _ in range(2))
        seqpos = torch.cat([torch.arange(x, dtype=torch.int64) for x in lengths]).to(dev)
        inv_freq = (1e6 ** (-torch.arange(0, hd, 2, dtype=torch.float32) / hd)).to(dev)
        cos, sin = ops.rope_table(inv_freq, max(lengths))
        cs = ops.rope_gather(seqpos, cos, sin)
        sa = sw = None
        if args.fp8:
            (a, sa), (w, sw) = ops.quantize_rows_e4m3(a), ops.quantize_rows_e4m3(w)
        heads = (torch.empty(t, hq, hd, dtype=torch.bfloat16, device=dev),
                 torch.empty(t, hkv, hd, dtype=torch.bfloat16, device=dev),
                 torch.empty(t, hkv, hd, dtype=torch.bfloat16, device=dev),
                 torch.empty(t, hq * hd, dtype=torch.bfloat16, device=dev) if args.gate else None)

        def run():
            ops.qkv_projection(a, w, seqpos, hq, hkv, hd, args.gate, q_norm, k_norm, ops.NORM_ONE_PLUS, -1, 1e-6, cs,
                               hd, out=heads, scale_a=sa, scale_w=sw)

        return run, 2 * t * n * kk, "FLOP", {"m": t, "n": n, "k": kk, "hq": hq, "hkv": hkv, "hd": hd,
                                             "gate": bool(args.gate), "fp8": bool(args.fp8)}
    if op in ("rmsnorm", "rmsnorm_e4m3", "quantize", "norm_add"):
        rows, cols = args.rows, args.cols
        x = bf16(g, rows, cols, device=dev)
        w = bf16(g, cols, device=dev, scale=0.1) + 1
        if op == "rmsnorm":
            out = torch.empty_like(x)

            def run():
                ops.rmsnorm(x, w, ops.NORM_WEIGHT, 1e-6, out=out)

            nbytes = rows * cols * 4
        elif op == "norm_add":
            h = bf16(g, rows, cols, device=dev)
            out = torch.empty_like(x)

            def run():
                ops.norm_add(h, x, w, ops.NORM_WEIGHT, 1e-6, out=out)

            nbytes = rows * cols * 6
        else:
            norm = op == "rmsnorm_e4m3"

            def run():
                ops.rmsnorm_e4m3(x, w if norm else None, ops.NORM_WEIGHT if norm else -1, 1e-6 if norm else 0.0)

            nbytes = rows * cols * 3 + rows * 4
        return run, nbytes, "B", {"rows": rows, "cols": cols}
    if op in ("delta_rule", "conv_silu", "gated_norm"):
        lengths = parse_lengths(args.lengths)
        t = sum(lengths)
        hk, hv, dk, dv = args.hk, args.hv, args.dk, args.dv
        width = 2 * hk * dk + hv * dv
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=dev)
        if op == "delta_rule":
            qkv = bf16(g, t, width, device=dev)
            ab = bf16(g, t, 2 * hv, device=dev)
            a_log = bf16(g, hv, device=dev, scale=0.5)
            dt_bias = bf16(g, hv, device=dev, scale=0.5)
            out = torch.empty(t, hv * dv, dtype=torch.bfloat16, device=dev)

            def run():
                ops.gated_delta_rule(qkv, ab, a_log, dt_bias, cu, hk, hv, dk, dv, out=out)

            if args.lib == "fla":
                run = library_delta_rule(qkv, ab, a_log, dt_bias, cu, hk, hv, dk, dv)
            elif args.lib:
                raise SystemExit("delta_rule --lib takes fla")

            return run, 6 * t * hv * dk * dv, "FLOP", {"sequences": len(lengths), "tokens": t, "hk": hk, "hv": hv,
                                                        "dk": dk, "dv": dv}
        if op == "conv_silu":
            x = bf16(g, t, width, device=dev)
            taps = bf16(g, width, 4, device=dev, scale=0.5)
            seqpos = torch.cat([torch.arange(n, dtype=torch.int64) for n in lengths]).to(dev)
            out = torch.empty(t, width, dtype=torch.bfloat16, device=dev)

            def run():
                ops.conv_silu(x, taps, seqpos, out=out)

            return run, 2 * t * width * 2 + t * 8, "B", {"tokens": t, "channels": width, "taps": 4}
        x = bf16(g, t, hv * dv, device=dev)
        z = bf16(g, t, hv * dv, device=dev)
        w = bf16(g, dv, device=dev, scale=0.1) + 1
        out = torch.empty(t, hv * dv, dtype=torch.bfloat16, device=dev)

        def run():
            ops.gated_norm(x, z, w, hv, dv, 1e-6, out=out)

        return run, 3 * t * hv * dv * 2, "B", {"tokens": t, "heads": hv, "head_dim": dv}
    raise SystemExit(f"unknown op {op}")


def library_attention(lib: str, q, k, v, cu, lengths, scale, window):
    """The same attention by a library kernel on the same tensors (no output gate): ``fa2`` flash-attention 2's
    flash_attn_varlen_func (GQA native), ``flashinfer[:backend]`` its ragged-KV prefill (``auto``: the backend it
    picks for this GPU; ``cutlass``: its sm100 kernel), ``torch[:backend]``
    F.scaled_dot_product_attention per sequence with the key/value heads repeated to the query heads outside the timed
    launch (whatever backend torch selects, or the one named: ``cudnn``, ``flash``, ``efficient``; ``cudnn`` is the
    library the reference's head-512 global layers call). Causal and sliding windows (left, 0) only."""
    left, right = window
    if right != 0 and not (left < 0 and right < 0):
        raise SystemExit("library attention: causal, sliding or bidirectional windows")
    causal = right == 0
    t, hq, hd = q.shape
    hkv = k.shape[1]
    max_len = max(lengths)
    if lib == "fa2":
        from flash_attn import flash_attn_varlen_func

        def run():
            flash_attn_varlen_func(q, k, v, cu, cu, max_len, max_len, softmax_scale=scale, causal=causal,
                                   window_size=(left if left >= 0 else -1, -1 if not causal else 0))
        return run
    if lib.split(":")[0] == "flashinfer":  # flashinfer[:backend], e.g. flashinfer:cutlass for its sm100 FMHA
        import flashinfer

        ws = torch.empty(256 << 20, dtype=torch.uint8, device=q.device)
        backend = lib.split(":")[1] if ":" in lib else "auto"
        wrapper = flashinfer.BatchPrefillWithRaggedKVCacheWrapper(ws, "NHD", backend=backend)
        wrapper.plan(cu, cu, hq, hkv, hd, causal=causal, window_left=left if left >= 0 else -1, sm_scale=scale,
                     q_data_type=torch.bfloat16)

        def run():
            wrapper.run(q, k, v)
        return run
    if lib.split(":")[0] == "torch":
        import contextlib

        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        backends = {"cudnn": SDPBackend.CUDNN_ATTENTION, "flash": SDPBackend.FLASH_ATTENTION,
                    "efficient": SDPBackend.EFFICIENT_ATTENTION}
        name = lib.split(":")[1] if ":" in lib else None
        if name is not None and name not in backends:
            raise SystemExit(f"torch SDPA backend {name}: one of {sorted(backends)}")
        group = hq // hkv
        kx, vx = k.repeat_interleave(group, dim=1), v.repeat_interleave(group, dim=1)
        bounds = cu.tolist()
        mask = None
        if left >= 0:
            raise SystemExit("torch SDPA comparison: causal or bidirectional only")

        def run():
            with sdpa_kernel(backends[name]) if name else contextlib.nullcontext():
                for a, b in zip(bounds[:-1], bounds[1:]):
                    F.scaled_dot_product_attention(q[a:b].transpose(0, 1)[None], kx[a:b].transpose(0, 1)[None],
                                                   vx[a:b].transpose(0, 1)[None], attn_mask=mask, is_causal=causal,
                                                   scale=scale)
        return run
    raise SystemExit(f"unknown attention library {lib}")


def library_delta_rule(qkv, ab, a_log, dt_bias, cu, hk, hv, dk, dv):
    """The reference's own Gated DeltaNet kernel on the same inputs: flash-linear-attention's chunk_gated_delta_rule
    with use_qk_l2norm_in_kernel and cu_seqlens, as families/qwen/packed.py:88-103 calls it; the query/key heads
    repeated to the value heads, the decay and write strength computed (families/qwen/fused.py:42-44) outside the timed
    launch."""
    import torch.nn.functional as F
    from fla.ops.gated_delta_rule import chunk_gated_delta_rule

    t = qkv.shape[0]
    kd = hk * dk
    q = qkv[:, :kd].reshape(1, t, hk, dk).repeat_interleave(hv // hk, dim=2).contiguous()
    k = qkv[:, kd:2 * kd].reshape(1, t, hk, dk).repeat_interleave(hv // hk, dim=2).contiguous()
    v = qkv[:, 2 * kd:].reshape(1, t, hv, dv).contiguous()
    b, a = ab[:, :hv].float(), ab[:, hv:].float()
    g = (-a_log.float().exp() * F.softplus(a + dt_bias.float()))[None].contiguous()
    beta = b.sigmoid().to(torch.bfloat16)[None].contiguous()
    cu64 = cu.long()

    def run():
        chunk_gated_delta_rule(q, k, v, g=g, beta=beta, initial_state=None, output_final_state=False,
                               use_qk_l2norm_in_kernel=True, cu_seqlens=cu64)
    return run


def main(argv: list[str] | None = None) -> dict:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("op", choices=["attention", "gemm", "qkv", "rmsnorm", "rmsnorm_e4m3", "quantize", "norm_add",
                                  "delta_rule", "conv_silu", "gated_norm"])
    p.add_argument("--lengths", default="mix:8192")
    p.add_argument("--hq", type=int, default=16)
    p.add_argument("--hkv", type=int, default=8)
    p.add_argument("--hd", type=int, default=128)
    p.add_argument("--window", default="-1,0", help="left,right (-1: unbounded); -1,0 is causal")
    p.add_argument("--gate", action="store_true", help="Qwen's sigmoid output gate")
    p.add_argument("--m", type=int, default=8192)
    p.add_argument("--n", type=int, default=6144)
    p.add_argument("--k", type=int, default=1024)
    p.add_argument("--fp8", action="store_true")
    p.add_argument("--epilogue", choices=sorted(EPILOGUES), default="store")
    p.add_argument("--rows", type=int, default=16384)
    p.add_argument("--cols", type=int, default=5376)
    p.add_argument("--hk", type=int, default=16)
    p.add_argument("--hv", type=int, default=32)
    p.add_argument("--dk", type=int, default=128)
    p.add_argument("--dv", type=int, default=128)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--lib", default="", help="time a library kernel on the same inputs instead: attention fa2, "
                                             "flashinfer[:backend] or torch[:cudnn|flash|efficient]; gemm cublas; "
                                             "delta_rule fla")
    args = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("microbench needs a CUDA device")
    dev = torch.device("cuda", torch.cuda.current_device())
    run, work, unit, shape = build(args, dev)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    ops.check_status(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.iters):
        run()
    end.record()
    torch.cuda.synchronize()
    ops.check_status(dev)
    us = start.elapsed_time(end) * 1e3 / args.iters
    rate = work / (us * 1e-6)
    line = {"op": args.op, "impl": args.lib or "libkd_b200", "shape": shape, "iters": args.iters,
            "us_per_launch": round(us, 2),
            "work_per_launch": work, "unit": unit,
            "achieved": round(rate / 1e12, 2) if unit == "FLOP" else round(rate / 1e9, 1),
            "achieved_unit": "TFLOP/s" if unit == "FLOP" else "GB/s"}
    print(json.dumps(line))
    return line


if __name__ == "__main__":
    main()
