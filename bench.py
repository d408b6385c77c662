#!/usr/bin/env python
"""Benchmark of the fused QK-RMSNorm + RoPE + non-causal attention op.

Workload (the metric's config): Flux.1 joint
attention at 1024x1024, B1 H24 S4608 D128, bf16, QK-RMSNorm + 3-axis RoPE.
A step is one fused call over one batch element's (b, h) units. With N GPUs
each rank runs its own batch element (batch x head partition, no
collective): weak scaling, global batch N.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the reference's algorithm on the host cores: the
C++ restatement of the shader sequence (oracle/, the reference itself cannot
be built or run here), on a bounded row sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-runner_b200"))

METRIC = "Flux joint-attn TFLOP/s per GPU (B1 H24 D128 S4608 bf16); % of BF16 peak"
FALLBACK_PEAK_TFLOPS = 1590.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="flux_1024")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-strong", action="store_true",
                    help="with N > 1 GPUs: skip the Qwen-Edit strong-scaling block")
    ap.add_argument("--profile-run", action="store_true",
                    help="only W + K fused calls, nothing else (for ncu captures)")
    ap.add_argument("--mode", choices=["batch", "headsplit", "ring"], default="batch",
                    help="batch: one batch element per rank (default, weak scaling); "
                         "headsplit / ring: one attention over all ranks (strong scaling)")
    ap.add_argument("--matrix", default="",
                    help="strong-scaling runs in one process group: comma-separated "
                         "config:mode[:transport] entries, e.g. "
                         "qwen_edit_2048:ring:copy,flux_1024:headsplit")
    ap.add_argument("--copy-streams", type=int, default=1,
                    help="ring copy transport: side streams (copy engines) per pull")
    ap.add_argument("--transport", choices=["copy", "nccl"], default="copy",
                    help="ring mode: K/V blocks pulled from their owners on the copy engines "
                         "(copy) or passed around the ring by NCCL P2P (nccl)")
    ap.add_argument("--qkv", action="store_true",
                    help="the QKV projection with the prologue in its epilogue "
                         "(llmr_qkv_project) on the configuration's shapes, against a cuBLAS "
                         "GEMM (torch.matmul) followed by the standalone prologue")
    ap.add_argument("--proj", action="store_true",
                    help="the output projection with the gated residual in its epilogue "
                         "(llmr_out_project, txt/img weight sets) against cuBLAS GEMMs per "
                         "stream followed by torch's bias / gate / residual ops")
    ap.add_argument("--varlen", action="store_true",
                    help="the CFG pair with different text lengths (Z-Image shapes: 256 + 4096 "
                         "and 0 + 4096 tokens, H30 D128 bf16, norm + RoPE) as one packed "
                         "llmr_attention_varlen call against two llmr_attention_fused calls")
    ap.add_argument("--vae", action="store_true",
                    help="the VAE mid-block attention (vae_attention: one head, fp32 [S, C], "
                         "128x128 latent = 16384 tokens, D = 512 and 384) on the wide-head "
                         "kernel, end to end through the mirror, and the oracle on the host")
    ap.add_argument("--cpu-table", action="store_true",
                    help="only the CPU baseline: the oracle on all host cores and on 1 core, "
                         "every configuration, a bounded row sample each")
    ap.add_argument("--heads", type=int, default=0,
                    help="with --profile-run: use this many heads (a smaller capture)")
    return ap.parse_args()


def profile_run(args):
    """Exactly W + K fused calls of the configuration on cuda:0 and nothing
    else, so that an ncu launch list or capture sees only the op's kernels.
    --config depth_fp32: the spatial_attention mirror on the Depth-shaped fp32
    case (H16 S1370 D64) on the tensor cores instead."""
    import torch

    import llmr_attn as L
    if args.config == "depth_fp32":
        import numpy as np
        H, S, D = 16, 1370, 64
        rng = np.random.default_rng(1)
        q, k, v = (torch.from_numpy(rng.standard_normal((H, S, D), dtype=np.float32) * 0.5)
                   .cuda() for _ in range(3))
        o = torch.empty((H, S, D), device="cuda")
        ctx = L.Context(0, workspace_bytes=4 * H * D * (4 * S + 2 * ((S + 3) // 4 * 4)))
        for _ in range(args.warmup + args.steps):
            L.spatial_attention(ctx, q, k, v, None, o, D, H, S, 0.125)
        ctx.sync()
        torch.cuda.synchronize()
        print(json.dumps({"profile_run": "depth_fp32 spatial_attention mirror",
                          "calls": args.warmup + args.steps, "launches": ctx.launches}))
        return
    from llmr_attn import configs as C
    from llmr_attn.runner import to_device
    case = C.CASES[args.config]
    prep = C.prepare(case, L.rope_tables, n_heads=args.heads or None)
    dc = to_device(prep)
    ctx = L.Context(0)
    ctx.reserve(L.workspace_bytes(dc.desc()))
    for _ in range(args.warmup + args.steps):
        dc.run(ctx)
    ctx.sync()
    torch.cuda.synchronize()
    print(json.dumps({"profile_run": case.name, "heads": dc.cfg.n_heads,
                      "calls": args.warmup + args.steps, "launches": ctx.launches}))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d.get("hbm_gbs", 0.0)), "measured"
    return FALLBACK_PEAK_TFLOPS, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", str(device_index), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons, power = [], [], set(), []
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # "under load": samples drawing more than 40% of the highest power seen
        pmax = max(power)
        loaded = [s for s, p in zip(sm, power) if p >= 0.4 * pmax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def host_cores() -> int:
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(case, prep, budget_s=12.0, rows_per_chunk=512, threads=0):
    """The oracle (reference algorithm restated) on host cores (`threads`, 0 =
    all) over a bounded row sample of one batch element. Returns (TFLOP/s,
    rows, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.set_threads(threads if threads > 0 else host_cores())
    S, H, D = case.seq_len, case.n_heads, case.head_dim

    def run(rows):
        t0 = time.perf_counter()
        O.attention_block(prep.q[0], prep.k[0], prep.v[0], H, D, case.scale, eps=case.eps,
                          q_gain=prep.q_gain, k_gain=prep.k_gain,
                          split_row=min(case.split_row, S), cos=prep.cos, sin=prep.sin,
                          exact=case.exact, rows=(0, rows), threads=threads)
        return time.perf_counter() - t0

    # A short probe sizes one timed call to about `budget_s` seconds.
    probe = min(S, 128)
    dt = run(probe)
    rows = int(min(S, max(probe, probe * budget_s / max(dt, 1e-3))) // 16 * 16) or 16
    dt = run(rows)
    flops = 4.0 * H * rows * S * D
    return flops / dt / 1e12, rows, dt


def config_block(case, n):
    return {"workload": f"{case.name}: B{case.batch} H{case.n_heads} S{case.seq_len} "
                        f"D{case.head_dim} {case.dtype}, QK-RMSNorm + RoPE + non-causal attention",
            "batch_per_gpu": case.batch, "global_batch": case.batch * n,
            "n_heads": case.n_heads, "seq_len": case.seq_len, "head_dim": case.head_dim,
            "parallelism": f"batch x head partition over {n} GPU(s), no collective",
            "l2": "flushed (256 MiB write) between timed steps"}


def qkv_bench(args):
    """Hidden = H*D (the model width of the reference's blocks): x [B*S, hidden]
    and W [3*H*D, hidden] in the configuration's dtype, QK-RMSNorm + RoPE as
    the configuration has them. Times (a) llmr_qkv_project and (b) cuBLAS
    x @ W^T into a [B*S, 3*H*D] buffer followed by llmr_attention_prologue
    reading it as three strided views; both produce the attention kernel's
    fp16 [3][B][H][S][D] input. CUDA events, L2 flushed between steps."""
    import numpy as np
    import torch

    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.runner import attn_config, torch_dtype
    case = C.CASES[args.config]
    prep = C.prepare(case, L.rope_tables)
    B, S, H, D = prep.q.shape
    hidden = H * D
    dt = torch_dtype(case.dtype)
    if dt == torch.float32:
        raise SystemExit("--qkv needs a 16-bit configuration")
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn((B * S, hidden), device="cuda", generator=g).to(dt)
    w = (torch.randn((3 * hidden, hidden), device="cuda", generator=g) * hidden ** -0.5).to(dt)
    cfg = attn_config(case, S)
    g32 = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    qg, kg, cos, sin = g32(prep.q_gain), g32(prep.k_gain), g32(prep.cos), g32(prep.sin)
    ctx = L.Context(0)
    out = torch.empty((3, B, H, S, D), device="cuda", dtype=torch.float16)
    y = torch.empty((B * S, 3 * hidden), device="cuda", dtype=dt)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    st = {"q_row_stride": 3 * hidden, "k_row_stride": 3 * hidden, "v_row_stride": 3 * hidden,
          "q_batch_stride": S * 3 * hidden, "k_batch_stride": S * 3 * hidden,
          "v_batch_stride": S * 3 * hidden}

    def fused():
        L.qkv_project(ctx, x, w, out, cfg, batch=B, seq_len=S, q_gain=qg, k_gain=kg, cos=cos,
                      sin=sin)

    def unfused():
        torch.matmul(x, w.t(), out=y)
        L.attention_prologue(ctx, y[:, :hidden], y[:, hidden:2 * hidden], y[:, 2 * hidden:],
                             out, cfg, batch=B, seq_len=S, q_gain=qg, k_gain=kg, cos=cos,
                             sin=sin, strides=st)

    res = {}
    for name, fn in (("fused", fused), ("cublas_plus_prologue", unfused)):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        res[name] = sum(ts) / len(ts)
    flops = 2.0 * B * S * hidden * 3 * hidden
    peak, _, kind = peaks()
    print(json.dumps({
        "qkv_projection": case.name, "M": B * S, "N": 3 * hidden, "K": hidden,
        "dtype": case.dtype, "fused_ms": res["fused"],
        "fused_tflops": flops / (res["fused"] / 1e3) / 1e12,
        "cublas_plus_prologue_ms": res["cublas_plus_prologue"],
        "speedup": res["cublas_plus_prologue"] / res["fused"],
        "peak": peak, "peak_source": kind, "steps": args.steps}), flush=True)
    ctx.close()


def proj_bench(args):
    """o [B*S, H*D] (the attention output) and two weight sets [H*D, H*D] in the
    configuration's dtype, split at the configuration's txt/img row, fp32
    hidden: (a) llmr_out_project; (b) per stream a cuBLAS GEMM, bias add and
    gated residual with torch ops. CUDA events, L2 flushed between steps."""
    import torch

    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.runner import torch_dtype
    case = C.CASES[args.config]
    B, S, H, D = case.batch, case.seq_len, case.n_heads, case.head_dim
    dim = H * D
    dt = torch_dtype(case.dtype)
    if dt == torch.float32:
        raise SystemExit("--proj needs a 16-bit configuration")
    split = min(case.split_row, S) if case.split_row else 0
    g = torch.Generator(device="cuda").manual_seed(9)
    o = torch.randn((B * S, dim), device="cuda", generator=g).to(dt)
    w = [(torch.randn((dim, dim), device="cuda", generator=g) * dim ** -0.5).to(dt)
         for _ in range(2)]
    bias = [torch.randn(dim, device="cuda", generator=g) for _ in range(2)]
    gate = [torch.rand(dim, device="cuda", generator=g) for _ in range(2)]
    hidden = torch.randn((B * S, dim), device="cuda", generator=g)
    ctx = L.Context(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    o3, h3 = o.view(B, S, dim), hidden.view(B, S, dim)
    segs = [(0, split, 0), (split, S, 1)] if split else [(0, S, 0)]

    def fused():
        L.out_project(ctx, o, hidden, w[0], w[1] if split else None, batch=B, seq_len=S,
                      split_row=split, bias0=bias[0], bias1=bias[1], gate0=gate[0],
                      gate1=gate[1])

    def unfused():
        for s0, s1, k in segs:
            y = torch.matmul(o3[:, s0:s1], w[k].t()).float()
            h3[:, s0:s1] += gate[k] * (y + bias[k])

    res = {}
    for name, fn in (("fused", fused), ("cublas_plus_torch", unfused)):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        res[name] = sum(ts) / len(ts)
    flops = 2.0 * B * S * dim * dim
    print(json.dumps({
        "out_projection": case.name, "M": B * S, "N": dim, "K": dim, "split_row": split,
        "dtype": case.dtype, "fused_ms": res["fused"],
        "fused_tflops": flops / (res["fused"] / 1e3) / 1e12,
        "cublas_plus_torch_ms": res["cublas_plus_torch"],
        "speedup": res["cublas_plus_torch"] / res["fused"], "steps": args.steps}), flush=True)
    ctx.close()


def varlen_bench(args):
    """Packed cond/uncond sequences (4352 and 4096 tokens) in one launch pair
    (prologue + attention) against one fused call per sequence."""
    import numpy as np
    import torch

    import llmr_attn as L
    H, D = 30, 128
    lens = (4352, 4096)
    T = sum(lens)
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn((1, T, H, D), device="cuda", generator=g).bfloat16()
               for _ in range(3))
    gain = torch.ones(D, device="cuda")
    tabs = []
    for i, n in enumerate(lens):
        pos = np.stack([np.full(n, i), np.arange(n) // 64, np.arange(n) % 64], 1).astype(np.int32)
        tabs.append(L.rope_tables(pos, (32, 48, 48), 256.0))
    cos = torch.from_numpy(np.concatenate([c for c, _ in tabs])).cuda()
    sin = torch.from_numpy(np.concatenate([s_ for _, s_ in tabs])).cuda()
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, norm_q=True, norm_k=True,
                       rope=True, eps=1e-5)
    o = torch.empty((1, T, H * D), device="cuda", dtype=torch.bfloat16)
    ctx = L.Context(0)
    ctx.reserve(3 * T * H * D * 2)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def packed():
        L.attention_varlen(ctx, q, k, v, o, cfg, lens, q_gain=gain, k_gain=gain, cos=cos,
                           sin=sin)

    def separate():
        off = 0
        for n in lens:
            sl = slice(off, off + n)
            L.attention_fused(ctx, q[:, sl], k[:, sl], v[:, sl], o[:, sl], cfg, batch=1,
                              seq_len=n, q_gain=gain, k_gain=gain, cos=cos[sl], sin=sin[sl])
            off += n

    res = {}
    for name, fn in (("packed", packed), ("separate", separate)):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        res[name] = sum(ts) / len(ts)
    flops = sum(4.0 * H * n * n * D for n in lens)
    print(json.dumps({"varlen": "zimage_cfg_pair", "seq_lens": lens, "n_heads": H,
                      "packed_ms": res["packed"], "separate_ms": res["separate"],
                      "packed_tflops": flops / (res["packed"] / 1e3) / 1e12,
                      "speedup": res["separate"] / res["packed"], "steps": args.steps}),
          flush=True)
    ctx.close()


def vae_bench(args):
    """vae_attention at a 1024x1024 image's latent (128 x 128 = 16384 tokens),
    one head of 512 (Flux / Z-Image VAE) and of 384 (Qwen VAE), fp32 [S, C]
    in and out as the reference binds them. Device-resident inputs with the
    L2 flushed per step (kernel and cast times from the op's own events), the
    whole mirror call from pinned host buffers (e2e), and the oracle
    restatement of the shader on all host cores over a row sample."""
    import numpy as np
    import torch

    import llmr_attn as L
    peak, _, kind = peaks()
    if not args.profile_run:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        cores = host_cores()
        O.set_threads(cores)
    S = 16384
    ctx = L.Context(0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for D in ((512,) if args.profile_run else (512, 384)):
        g = torch.Generator(device="cuda").manual_seed(D)
        q, k, v = (torch.randn((S, D), device="cuda", generator=g) for _ in range(3))
        o = torch.empty((S, D), device="cuda")
        ctx.reserve(3 * S * D * 2)
        scale = D ** -0.5

        def call():
            L.vae_attention(ctx, q, k, v, o, D, 1, S, scale)

        if args.profile_run:
            # W + K calls (cast + wide kernel each) and nothing else, for ncu.
            for _ in range(args.warmup + args.steps):
                call()
            torch.cuda.synchronize()
            break

        for _ in range(max(args.warmup, 3)):
            call()
        torch.cuda.synchronize()
        ctx.profile(True)
        tot, cast, attn = [], [], []
        l0 = ctx.launches
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            call()
            b.record()
            c_ms, k_ms = ctx.profile_read()
            torch.cuda.synchronize()
            tot.append(a.elapsed_time(b))
            cast.append(c_ms)
            attn.append(k_ms)
        launches = (ctx.launches - l0) / args.steps
        ctx.profile(False)
        # End to end: pinned host Q, K, V -> device, the call, O -> pinned host.
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        ho = torch.empty((S, D)).pin_memory()
        e2e = []
        for _ in range(min(args.steps, 10)):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            q.copy_(hq, non_blocking=True)
            k.copy_(hk, non_blocking=True)
            v.copy_(hv, non_blocking=True)
            call()
            ho.copy_(o, non_blocking=True)
            b.record()
            torch.cuda.synchronize()
            e2e.append(a.elapsed_time(b))
        flops = 4.0 * S * S * D
        ms, cast_ms, attn_ms = (sum(x) / len(x) for x in (tot, cast, attn))
        e2e_ms = sum(e2e) / len(e2e)
        # The oracle (the shader's fp32 restatement) over a row sample.
        nq, nk, nv = (x.numpy() for x in (hq, hk, hv))
        rows = 32
        t0 = time.perf_counter()
        O.vae_attention(nq, nk, nv, D, 1, S, scale, rows=(0, rows))
        cpu_s = time.perf_counter() - t0
        cpu_tf = flops * rows / S / cpu_s / 1e12
        print(json.dumps({
            "vae": f"vae_attention S{S} D{D} fp32 [S,C]", "steps": args.steps,
            "ms_per_call": ms, "cast_ms": cast_ms, "kernel_ms": attn_ms,
            "tflops_call": flops / ms / 1e9, "tflops_kernel": flops / attn_ms / 1e9,
            "kernel_mma_tflops": 1.5 * flops / attn_ms / 1e9,
            "kernel_frac_of_peak": flops / attn_ms / 1e9 / peak, "peak_tflops": peak,
            "peak_source": kind, "gpu_launches_per_call": launches,
            "e2e": {"ms": e2e_ms, "tflops": flops / e2e_ms / 1e9,
                    "h2d_bytes": 3 * S * D * 4, "d2h_bytes": S * D * 4},
            "cpu_baseline": {"tflops": cpu_tf, "cores": cores, "kind": "port",
                             "sample": f"{rows} of {S} query rows",
                             "full_op_ms_extrapolated": flops / (cpu_tf * 1e12) * 1e3}}),
            flush=True)
    ctx.close()


def cpu_table(args):
    """The oracle per configuration on all host cores and on one core, each
    over a row sample of about 8 s, extrapolated to the whole op."""
    import llmr_attn as L
    from llmr_attn import configs as C
    cores = host_cores()
    for name, case in C.CASES.items():
        prep = C.prepare(case, L.rope_tables)
        for threads in (0, 1):
            tf, rows, dt = cpu_sample(case, prep, budget_s=8.0, threads=threads)
            print(json.dumps({"cpu_table": name, "cores": cores if threads == 0 else 1,
                              "rows_sampled": rows, "of_rows": case.seq_len, "seconds": dt,
                              "tflops": tf, "full_op_ms_extrapolated": case.flops / (tf * 1e12) * 1e3,
                              "kind": "port (oracle restatement of the reference shaders)"}),
                  flush=True)


def configs_module():
    """llmr_attn/configs.py loaded as a standalone module (numpy only)."""
    import importlib.util
    path = os.path.join(ROOT, "llm-runner_b200", "llmr_attn", "configs.py")
    spec = importlib.util.spec_from_file_location("llmr_bench_configs", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # dataclasses resolve the module by name
    spec.loader.exec_module(mod)
    return mod


def run_reference(args):
    """CPU reference arm: rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    # The configurations' input recipe is pure numpy; it is loaded by path so
    # that this arm never imports the product package (which maps the CUDA
    # library), and the RoPE tables come from the oracle's own builder.
    C = configs_module()
    cores = host_cores()
    O.set_threads(cores)     # torchrun sets OMP_NUM_THREADS=1 per process
    case = C.CASES[args.config]
    prep = C.prepare(case, O.rope_tables)
    S, H, D = case.seq_len, case.n_heads, case.head_dim
    split = min(case.split_row, S)
    qb, kb, vb = (np.ascontiguousarray(a[0].reshape(S, H * D)) for a in (prep.q, prep.k, prep.v))

    def prologue():
        """The reference block's ops before the attention, over all tokens
        (the sequence orc_attention_block restates): per-head RMSNorm of Q and
        K with the txt / img gain sets, Q / K / V to [H, S, D], RoPE."""
        qn, kn = qb.copy(), kb.copy()
        for x, g in ((qn, prep.q_gain), (kn, prep.k_gain)):
            if g is None:
                continue
            g = np.asarray(g, np.float32).reshape(-1, D)
            if split > 0:
                O.batch_head_norm(x[:split], g[0], H, D, split, case.eps)
            O.batch_head_norm(x[split:], g[1] if g.shape[0] > 1 else g[0], H, D, S - split,
                              case.eps)
        qt, kt, vt = (O.transpose_heads(x, S, H, D, 0) for x in (qn, kn, vb))
        if prep.cos is not None:
            O.mrope(qt, prep.cos, prep.sin, S, H, head_dim=D)
            O.mrope(kt, prep.cos, prep.sin, S, H, head_dim=D)
        return qt, kt, vt

    # The prologue is done once per whole op; a step of `rows` query rows is
    # charged its share of it, so the sampled rate is the whole op's rate.
    pro = []
    for _ in range(3):
        t0 = time.perf_counter()
        qt, kt, vt = prologue()
        pro.append(time.perf_counter() - t0)
    t_pro = sorted(pro)[1]
    rows = min(384, S)   # a window large enough to amortise the per-call output buffer
    times, r0 = [], 0
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        if case.exact:
            O.spatial_attention(qt, kt, vt, D, H, S, case.scale, rows=(r0, min(r0 + rows, S)))
        else:
            O.flash_attention_v2(qt, kt, vt, D, H, S, case.scale,
                                 qb_range=(r0 // 16, (min(r0 + rows, S) + 15) // 16))
        dt = time.perf_counter() - t0 + t_pro * rows / S
        if i >= args.warmup:
            times.append(dt)
        r0 = (r0 + rows) % S
    ms = 1e3 * sum(times) / len(times)
    tflops = 4.0 * H * rows * S * D / (ms / 1e3) / 1e12
    kernel = "spatial_attention" if case.exact else "flash_attention_v2"
    sample = (f"per step: {kernel} on {rows} query rows x {H} heads over all S={S} keys, "
              f"plus {rows}/{S} of the norm + transpose + RoPE prologue over all tokens "
              f"(timed once: {t_pro * 1e3:.1f} ms)")
    line = {"metric": METRIC, "value": tflops, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (fp16 operands)", "data": "synthetic",
            "config": config_block(case, args.gpus),
            "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": cores,
                             "kind": "port", "sample": sample},
            "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference (C3 + Slang + Vulkan) cannot be built or run here; this is "
                    "the oracle's line-by-line C++ restatement of its shaders"}
    print(json.dumps(line), flush=True)


def f64_rows(q, k, v, qg, kg, cos, sin, case, rows, heads):
    """fp64 restatement of the fused op for query rows `rows` (a slice) and
    heads `heads` (a range), on the GPU: per-head RMSNorm with the txt/img
    gain set of each row, the interleaved RoPE rotation, Q / K / V rounded to
    fp16 (the reference's load rounding), exact softmax. q/k/v: [1, S, H, D]
    device tensors; returns [len(rows), len(heads) * D] float64."""
    import torch
    S, D = q.shape[1], q.shape[3]
    split = min(case.split_row, S)

    def prep(x, g, r0, r1, h, rope):
        x = x[0, r0:r1, h].double()
        if g is not None:
            gs = g.double().reshape(-1, D)
            sel = torch.zeros(r1 - r0, dtype=torch.long, device=x.device)
            if gs.shape[0] > 1 and split > 0:
                sel[torch.arange(r0, r1, device=x.device) >= split] = 1
            x = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + case.eps) * gs[sel]
        if rope:
            c, s_ = cos[r0:r1].double(), sin[r0:r1].double()
            y = torch.empty_like(x)
            y[:, 0::2] = x[:, 0::2] * c - x[:, 1::2] * s_
            y[:, 1::2] = x[:, 0::2] * s_ + x[:, 1::2] * c
            x = y
        return x.half().double()

    out = []
    for h in heads:
        qn = prep(q, qg, rows.start, rows.stop, h, cos is not None)
        kn = prep(k, kg, 0, S, h, cos is not None)
        vn = prep(v, None, 0, S, h, False)
        out.append(torch.softmax((qn @ kn.T) * case.scale, dim=-1) @ vn)
    return torch.cat(out, dim=1)


def roofline_block(case, achieved, peak, peak_kind, traffic):
    """Roofline of the dominant kernel. The fp16/bf16 configs run on
    kind::f16 (bound: the measured dense BF16 peak). The fp32 exact config
    runs three TF32 products per fp32 product on kind::tf32, whose rate is
    half the BF16 rate: its tensor-pipe bound for algorithmic flops is a
    sixth of the BF16 peak."""
    if case.exact and case.head_dim == 64:
        bound = peak / 6.0
        return {"bound": "tensor", "achieved": achieved, "peak": bound, "unit": "TFLOP/s",
                "frac": achieved / bound, "traffic": None,
                "kernel": "attn_exact_tc_kernel (3xTF32, kind::tf32)",
                "peak_source": f"{peak_kind} bf16_tflops / 2 (TF32 rate) / 3 (passes)",
                "note": "achieved includes the TF32 split kernel (the op's second phase)"}
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": traffic,
            "kernel": f"fa_fwd_tc_kernel<{case.head_dim}, {case.dtype}>",
            "peak_source": f"{peak_kind} bf16_tflops (burst)"}


def exact_depth_block(args, local, peak, peak_kind):
    """The exact fp32 path on a Depth-Anything-shaped case (B1 H16 S1370 D64,
    0.5 * N(0, 1), scale 1/8) through the spatial_attention mirror: the
    tensor-core kernel (context workspace reserved) against the fp32 FMA
    kernel (no workspace), CUDA events, L2 flushed between steps."""
    import numpy as np
    import torch

    import llmr_attn as L
    H, S, D = 16, 1370, 64
    rng = np.random.default_rng(1)
    q, k, v = (torch.from_numpy(rng.standard_normal((H, S, D), dtype=np.float32) * 0.5)
               .to(f"cuda:{local}") for _ in range(3))
    o = torch.empty((H, S, D), device=f"cuda:{local}")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")
    flops = 4.0 * H * S * S * D
    res = {"workload": f"spatial_attention mirror, H{H} S{S} D{D} fp32 [H, S, D]"}
    for name, ws in (("tensor_cores", 4 * H * D * (4 * S + 2 * ((S + 3) // 4 * 4))),
                     ("fma", 0)):
        ctx = L.Context(local, workspace_bytes=ws)
        call = lambda: L.spatial_attention(ctx, q, k, v, None, o, D, H, S, 0.125)
        for _ in range(3):
            call()
        ctx.sync()
        ts = []
        for _ in range(max(5, min(args.steps, 20))):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            call()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        ms = sum(ts) / len(ts)
        res[name] = {"ms": ms, "tflops": flops / (ms / 1e3) / 1e12}
        ctx.close()
    res["tensor_core_frac_of_bound"] = res["tensor_cores"]["tflops"] / (peak / 6.0)
    res["speedup_over_fma"] = res["fma"]["ms"] / res["tensor_cores"]["ms"]
    return res


def strong_scaling_block(args, world, rank, local):
    """The north star's multi-GPU target, measured inside the same torchrun
    launch as the weak-scaling line: Qwen-Image-Edit 2048^2 (B1 H24 S33792
    D128 bf16, QK-RMSNorm + 3-axis RoPE) as ONE attention spread over all
    ranks (strong scaling), as (a) a head split (H/N heads per GPU, no
    collective) and (b) the sequence-sharded ring with both K/V transports
    (copy-engine pulls; NCCL P2P with 0 / 8 / 16 SMs left free for NCCL's
    kernels). T1 is the whole call on one GPU: every rank runs it on its own
    GPU at the same time (no communication) and rank 0's time is T1, so T1
    and T_N are taken with every GPU busy, in the same power and clock state.
    Each mode is timed in three trials (T1 and the head split alternate;
    each ring mode follows with its own three): one trial = `steps` calls
    after a barrier, its time the max over ranks of CUDA-event time; the line
    carries each mode's best trial and all three (clocks drift by several per
    cent over a run on these GPUs). Each mode's assembled output is checked
    on row windows against an fp64 restatement (max / mean error over all
    ranks)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.dist import RingAttention, RingOps, head_split_attention, partition_units
    from llmr_attn.runner import attn_config

    case = C.CASES["qwen_edit_2048"]
    S, H, D = case.seq_len, case.n_heads, case.head_dim
    dev = torch.device(f"cuda:{local}")
    g = torch.Generator(device=dev).manual_seed(1000 + case.seed)  # identical on every rank
    q, k, v = (torch.randn((1, S, H, D), device=dev, generator=g).to(torch.bfloat16)
               for _ in range(3))
    rng = np.random.default_rng(case.seed)
    qg = torch.from_numpy(rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)).to(dev)
    kg = torch.from_numpy(rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)).to(dev)
    cos, sin = (torch.from_numpy(t).to(dev) for t in
                L.rope_tables(C.case_ids(case), case.rope[0], case.rope[1]))
    cfg = attn_config(case, S)
    steps = max(3, min(args.steps, 10))
    warm = 2
    trials = 3
    stream = torch.cuda.Stream(device=dev)
    trial_ms = {}

    def trial(step_fn, ctx, rank0_only=False):
        """One trial: `steps` calls after a barrier; the max over ranks (rank
        0's time when rank0_only), in ms per call."""
        with torch.cuda.stream(stream):
            dist.barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(steps):
                step_fn()
            b.record(stream)
            torch.cuda.synchronize()
            ctx.sync()
        ms = a.elapsed_time(b) / steps
        t = torch.tensor([ms if (rank == 0 or not rank0_only) else 0.0], dtype=torch.float64,
                         device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def warm_up(step_fn, ctx):
        with torch.cuda.stream(stream):
            for _ in range(warm):
                step_fn()
            ctx.sync()

    def check(err_max, err_sum, n):
        t = torch.tensor([err_max], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        u = torch.tensor([err_sum, float(n)], dtype=torch.float64, device=dev)
        dist.all_reduce(u)
        return {"max_abs_err": float(t.item()), "mean_abs_err": float(u[0] / max(u[1], 1.0))}

    res = {"workload": f"{case.name}: B1 H{H} S{S} D{D} bf16, QK-RMSNorm + RoPE, one "
                       f"attention over {world} GPUs", "steps": steps, "warmup": warm,
           "trials": trials,
           "timing": "best of the trials; each trial the max over ranks (T1: rank 0, with "
                     "every rank running the whole call on its own GPU at the same time)",
           "flop_per_call": case.flops}
    with torch.cuda.stream(stream):
        ctx = L.Context(local, stream=stream)
    ctx.reserve(3 * S * H * D * 2)
    o_t1 = torch.empty((1, S, H * D), dtype=torch.bfloat16, device=dev)
    o_hs = torch.empty((1, S, H * D), dtype=torch.bfloat16, device=dev)
    run_t1 = lambda: L.attention_fused(ctx, q, k, v, o_t1, cfg, batch=1, seq_len=S,
                                       q_gain=qg, k_gain=kg, cos=cos, sin=sin)
    run_hs = lambda: head_split_attention(ctx, q, k, v, o_hs, cfg, batch=1, seq_len=S,
                                          rank=rank, world=world, q_gain=qg, k_gain=kg,
                                          cos=cos, sin=sin)
    # T1 and (a) the head split, alternating.
    warm_up(run_t1, ctx)
    warm_up(run_hs, ctx)
    trial_ms["t1"], trial_ms["headsplit"] = [], []
    for _ in range(trials):
        trial_ms["t1"].append(trial(run_t1, ctx, rank0_only=True))
        trial_ms["headsplit"].append(trial(run_hs, ctx))
    t1 = min(trial_ms["t1"])
    hs_ms = min(trial_ms["headsplit"])
    res["t1_ms"] = t1
    windows = [(1008, 1072), (S - 32, S)]
    emax, esum, n = 0.0, 0.0, 0
    for _, h0, h1 in partition_units(1, H, world, rank):
        for r0, r1 in windows:
            want = f64_rows(q, k, v, qg, kg, cos, sin, case, range(r0, r1), range(h0, h1))
            err = (o_hs[0, r0:r1, h0 * D:h1 * D].double() - want).abs()
            emax, esum, n = max(emax, err.max().item()), esum + err.sum().item(), n + err.numel()
    res["headsplit"] = {"ms": hs_ms, "efficiency": t1 / (world * hs_ms),
                        "heads_per_gpu": f"{H // world}" if H % world == 0 else "uneven",
                        **check(emax, esum, n)}

    # (b) sequence ring: rank r holds tokens [r*S/N, (r+1)*S/N).
    s_loc = S // world
    sl = slice(rank * s_loc, (rank + 1) * s_loc)
    qs, ks, vs = (x[:, sl].contiguous() for x in (q, k, v))
    o_loc = torch.empty((1, s_loc, H * D), dtype=torch.bfloat16, device=dev)
    for transport, reserve in (("copy", 0), ("nccl", 0), ("nccl", 8), ("nccl", 16)):
        with torch.cuda.stream(stream):
            rctx = L.Context(local, stream=stream)
            if reserve:
                rctx.set_sm_budget(torch.cuda.get_device_properties(dev).multi_processor_count
                                   - reserve)
            ring = RingAttention(RingOps(rctx, cfg, s_loc, rank * s_loc), H, D, S, rank, world,
                                 dev, transport=transport)
        key = "ring_copy" if transport == "copy" else f"ring_nccl_free_sms_{reserve}"
        run_ring = lambda: ring.forward(qs, ks, vs, o_loc, qg, kg, cos, sin)
        warm_up(run_ring, rctx)
        trial_ms[key] = [trial(run_ring, rctx) for _ in range(trials)]
        ms = min(trial_ms[key])
        w0 = rank * s_loc
        want = f64_rows(q, k, v, qg, kg, cos, sin, case, range(w0, w0 + 64), range(H))
        err = (o_loc[0, :64].double() - want).abs()
        res[key] = {"ms": ms, "efficiency": t1 / (world * ms),
                    **check(err.max().item(), err.sum().item(), err.numel())}
        torch.cuda.synchronize()
        dist.barrier()
        ring.close()
        rctx.close()
    ctx.close()
    tflops = {k_: case.flops / (v_["ms"] / 1e3) / 1e12 for k_, v_ in res.items()
              if isinstance(v_, dict) and "ms" in v_}
    res["tflops_whole_job"] = tflops
    res["trial_ms"] = trial_ms
    return res


def run_strong(args):
    """One attention of the configuration spread over all ranks (strong
    scaling): `headsplit` gives each rank a contiguous share of the (b, h)
    units with no communication; `ring` shards the sequence and moves the
    fp16 K/V blocks between ranks (copy engines or NCCL P2P, --transport)
    while each rank computes. With --matrix, every listed (config, mode,
    transport) in turn, in one process group.
    Time per step = max over ranks of the CUDA-event time of the call."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    if args.matrix:
        runs = []
        for ent in args.matrix.split(","):
            parts = ent.split(":")
            runs.append((parts[0], parts[1], parts[2] if len(parts) > 2 else args.transport,
                         int(parts[3]) if len(parts) > 3 else args.copy_streams))
    else:
        runs = [(args.config, args.mode, args.transport, args.copy_streams)]
    for config, mode, transport, copy_streams in runs:
        strong_case(args, config, mode, transport, copy_streams)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def strong_case(args, config, mode, transport, copy_streams=1):
    import numpy as np
    import torch
    import torch.distributed as dist

    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.dist import RingAttention, RingOps, head_split_attention
    from llmr_attn.runner import attn_config, torch_dtype

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    case = C.CASES[config]
    prep = C.prepare(case, L.rope_tables)
    B, S, H, D = prep.q.shape
    dt = torch_dtype(case.dtype)
    dev = f"cuda:{local}"
    stream = torch.cuda.Stream(device=dev)
    g32 = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    cfg = attn_config(case, S)
    with torch.cuda.stream(stream):
        ctx = L.Context(local, stream=stream)
        qg, kg, cos, sin = g32(prep.q_gain), g32(prep.k_gain), g32(prep.cos), g32(prep.sin)
        if mode == "headsplit":
            q, k, v = (torch.from_numpy(a).to(dev).to(dt) for a in (prep.q, prep.k, prep.v))
            o = torch.empty((B, S, H * D), dtype=dt, device=dev)
            from llmr_attn.dist import partition_units
            runs = partition_units(B, H, world, rank)
            need = max(L.workspace_bytes(L.make_desc(L.AttnConfig(**{**cfg.__dict__,
                                                                     "n_heads": h1 - h0}),
                                                     1, S, L._dtype_code(q), L._dtype_code(o)))
                       for _, h0, h1 in runs)
            ctx.reserve(need)
            def step():
                head_split_attention(ctx, q, k, v, o, cfg, batch=B, seq_len=S, rank=rank,
                                     world=world, q_gain=qg, k_gain=kg, cos=cos, sin=sin)
            units = sum(h1 - h0 for _, h0, h1 in runs)
        else:
            if S % world:
                raise SystemExit("ring needs seq_len divisible by the number of GPUs")
            s_loc = S // world
            sl = slice(rank * s_loc, (rank + 1) * s_loc)
            q, k, v = (torch.from_numpy(np.ascontiguousarray(a[:, sl])).to(dev).to(dt)
                       for a in (prep.q, prep.k, prep.v))
            o = torch.empty((1, s_loc, H * D), dtype=dt, device=dev)
            ring = RingAttention(RingOps(ctx, cfg, s_loc, rank * s_loc,
                                         copy_streams=copy_streams), H, D, S, rank, world,
                                 dev, transport=transport)
            def step():
                ring.forward(q, k, v, o, qg, kg, cos, sin)
            units = H
        for _ in range(max(args.warmup, 3)):
            step()
        ctx.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        l0 = ctx.launches
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for s_, e_ in ev:
            s_.record(stream)
            step()
            e_.record(stream)
        torch.cuda.synchronize()
        ctx.sync()
        launches = ctx.launches - l0
    total = torch.tensor([sum(s_.elapsed_time(e_) for s_, e_ in ev)], dtype=torch.float64,
                         device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    ms = float(total.item()) / args.steps
    value = case.flops / (ms / 1e3) / 1e12
    peak, _, kind = peaks()
    if rank == 0:
        print(json.dumps({
            "metric": f"{case.name} attention TFLOP/s (whole job, strong scaling)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": case.dtype,
            "data": "synthetic", "mode": mode,
            "transport": transport if mode == "ring" else None,
            "copy_streams": copy_streams if mode == "ring" and transport == "copy" else None,
            "config": {"workload": case.name, "batch": B, "n_heads": H, "seq_len": S,
                       "head_dim": D, "units_rank0": units},
            "pct_of_peak_per_gpu": 100.0 * value / world / peak, "peak_source": kind,
            "gpu_launches_rank0": launches}), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if mode == "ring":
        ring.close()
    ctx.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.cpu_table:
        cpu_table(args)
        return
    if args.qkv:
        qkv_bench(args)
        return
    if args.proj:
        proj_bench(args)
        return
    if args.varlen:
        varlen_bench(args)
        return

    if args.vae:
        vae_bench(args)
        return
    if args.profile_run:
        profile_run(args)
        return
    if args.mode != "batch" or args.matrix:
        run_strong(args)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.runner import to_device

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    case = C.CASES[args.config]
    prep = C.prepare(case, L.rope_tables)
    # Each rank owns one batch element; make its inputs distinct.
    if rank:
        rng = np.random.default_rng(case.seed * 1000 + rank)
        for a in (prep.q, prep.k, prep.v):
            a[...] = C.round_to(rng.standard_normal(a.shape, dtype=np.float32), case.dtype)
    dc = to_device(prep, device=local)
    ctx = L.Context(local)
    ctx.reserve(L.workspace_bytes(dc.desc()))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")
    flops = case.flops  # per rank (one batch element)

    sampler = ClockSampler(local)
    t_warm = time.perf_counter()
    i = 0
    while i < max(args.warmup, 3) or time.perf_counter() - t_warm < 1.5:
        flush.zero_()
        dc.run(ctx)
        torch.cuda.synchronize()
        i += 1
    ctx.sync()

    # Timed region: the fused call as a user makes it (prologue, then the
    # attention kernel launched behind it with programmatic dependent launch).
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = ctx.launches
    for k in range(args.steps):
        flush.zero_()
        ev[k][0].record()
        dc.run(ctx)
        ev[k][1].record()
    torch.cuda.synchronize()
    launches = ctx.launches - l0
    if world > 1:
        dist.barrier()
    ctx.sync()

    # Per-kernel times for the roofline: the same steps with the library's
    # own events around each kernel (an event between the two launches
    # serialises them, so each kernel is timed alone).
    ctx.profile(True)
    attn_ms, pro_ms = [], []
    for k in range(args.steps):
        flush.zero_()
        dc.run(ctx)
        p, a = ctx.profile_read()  # waits for this step
        pro_ms.append(p)
        attn_ms.append(a)
    ctx.profile(False)
    ctx.sync()
    total_ms = sum(s.elapsed_time(e) for s, e in ev)
    t = torch.tensor([total_ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_step = total_ms / args.steps
    value = world * flops / (ms_step / 1e3) / 1e12

    # End to end through the public API: pinned host inputs -> device, the
    # fused op, result -> pinned host, every step.
    hq, hk, hv = (x.cpu().pin_memory() for x in (dc.q, dc.k, dc.v))
    ho = torch.empty(dc.o.shape, dtype=dc.o.dtype).pin_memory()
    e2e_steps = min(args.steps, 20)
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(e2e_steps)]
    torch.cuda.synchronize()
    for k in range(e2e_steps):
        flush.zero_()
        e2e_ev[k][0].record()
        dc.q.copy_(hq, non_blocking=True)
        dc.k.copy_(hk, non_blocking=True)
        dc.v.copy_(hv, non_blocking=True)
        dc.run(ctx)
        ho.copy_(dc.o, non_blocking=True)
        e2e_ev[k][1].record()
    torch.cuda.synchronize()
    ctx.sync()
    e2e_serial_ms = sum(s.elapsed_time(e) for s, e in e2e_ev) / e2e_steps

    # The same steps pipelined as a serving loop runs them: step i's inputs are
    # copied in (pinned host -> device) on one stream while step i-1 computes
    # on another and step i-2's result is copied out on a third (PCIe is full
    # duplex). Two device buffer sets; every step still moves its own inputs
    # and result across PCIe inside the timed region. 50 steps (a denoising
    # run's worth), so the pipeline's fill and drain weigh little.
    pipe_steps = 50
    dc2 = to_device(prep, device=local)
    bufs = [dc, dc2]
    s_h2d, s_cmp, s_d2h = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ctx_p = L.Context(local, stream=s_cmp)
    ctx_p.reserve(L.workspace_bytes(dc.desc()))
    ho2 = [ho, torch.empty(dc.o.shape, dtype=dc.o.dtype).pin_memory()]
    mk = lambda: torch.cuda.Event(enable_timing=False)
    h2d_done = [mk() for _ in range(pipe_steps)]
    cmp_done = [mk() for _ in range(pipe_steps)]
    d2h_done = [mk() for _ in range(pipe_steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_start.record(s_h2d)
    for i in range(pipe_steps):
        b = bufs[i % 2]
        if i >= 2:
            s_h2d.wait_event(cmp_done[i - 2])     # step i-2 finished reading b's inputs
        with torch.cuda.stream(s_h2d):
            b.q.copy_(hq, non_blocking=True)
            b.k.copy_(hk, non_blocking=True)
            b.v.copy_(hv, non_blocking=True)
        h2d_done[i].record(s_h2d)
        s_cmp.wait_event(h2d_done[i])
        if i >= 2:
            s_cmp.wait_event(d2h_done[i - 2])     # step i-2's result has left b.o
        b.run(ctx_p)
        cmp_done[i].record(s_cmp)
        s_d2h.wait_event(cmp_done[i])
        with torch.cuda.stream(s_d2h):
            ho2[i % 2].copy_(b.o, non_blocking=True)
        d2h_done[i].record(s_d2h)
    s_d2h.wait_stream(s_h2d)
    s_d2h.wait_stream(s_cmp)
    t_end.record(s_d2h)
    torch.cuda.synchronize()
    ctx_p.sync()
    e2e_ms = t_start.elapsed_time(t_end) / pipe_steps
    ctx_p.close()
    te = torch.tensor([e2e_ms], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())
    clocks = sampler.stop()

    peak, hbm, peak_kind = peaks()
    a_ms = statistics.mean(attn_ms)
    achieved = flops / (a_ms / 1e3) / 1e12
    traffic = None
    tp = os.path.join(ROOT, "profiles", "fa_fwd_tc_flux_traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get("dram_bytes_per_launch")

    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": case.dtype,
        "data": f"synthetic (seeded N(0,1) {case.dtype} Q/K/V"
                + (f", {case.gain} gains)" if case.norm else ")"),
        "config": config_block(case, world),
        "value_per_gpu": value / world,
        "pct_of_peak": 100.0 * (value / world) / peak,
        "phases_ms": {"prologue": statistics.mean(pro_ms), "attention": a_ms,
                      "note": "each kernel timed alone (library events between the launches); "
                              "ms_per_step overlaps the attention kernel's set-up with the "
                              "prologue's tail (programmatic dependent launch)"},
        "roofline": roofline_block(case, achieved, peak, peak_kind, traffic),
        "e2e": {"value": world * flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": 3 * dc.q.numel() * dc.q.element_size(),
                "d2h_bytes_per_step": dc.o.numel() * dc.o.element_size(),
                "ms_per_step": e2e_ms, "steps": pipe_steps,
                "schedule": "pipelined: H2D of step i, compute of step i-1, D2H of step i-2 "
                            "on three streams, two device buffer sets",
                "serial_ms_per_step": e2e_serial_ms},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if case.exact:
        line["exact_depth_shaped"] = exact_depth_block(args, local, peak, peak_kind)
    if world > 1 and not args.no_strong:
        line["strong_scaling"] = strong_scaling_block(args, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, rows, dt = cpu_sample(case, prep)
        line["cpu_baseline"] = {
            "value": tf, "unit": "TFLOP/s", "cores": host_cores(), "kind": "port",
            "sample": f"{rows} of {case.seq_len} query rows x {case.n_heads} heads, "
                      f"{dt:.1f} s, oracle restatement of the reference shaders"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
