"""Benchmark of the routed-expert hot path on B200 (one JSON line on rank 0).

Workload (BASELINE.json metric "MoE-layer tokens/s at 1/2/4/8 B200; MX matvec HBM GB/s"):
config 2, the DeepSeek-V4-like MXFP4 MoE layer: hidden 7168, 256 routed experts + 1 shared,
intermediate 2048, bf16 router with sigmoid + bias noaux_tc top-8 (x2.5), a 128-token prefill
chunk per GPU (x ~ N(0,1) bf16).  Random-init, seeded synthetic weights (no checkpoints).
On N GPUs (torchrun) the layer runs expert parallel: rank r holds 256/N routed experts plus
the replicated router and shared expert, and routes its own 128 tokens (weak scaling: 128*N
tokens per step); token rows and expert outputs cross NVLink inside the kernels.

  value     tokens/s, inputs already in HBM (urb_moe_forward_device), device-timed
  e2e       tokens/s through the host-pointer C ABI (urb_moe_forward), H2D of x and D2H of the
            output + routes inside the timed region
  roofline  the dominant kernel (block-scaled grouped gate/up pass, k_bs_grouped): algorithmic
            bytes per launch (touched experts' packed MXFP4 gate+up tiles + the f32 gate|up
            outputs) / its mean CUDA-event duration, against the measured HBM copy bandwidth;
            `traffic` is the DRAM bytes per launch from the committed ncu capture
            (profiles/k_bs_grouped_c2_traffic.md)
  cpu_baseline / --impl reference: the CPU restatement of the reference path (oracle/) on the
            host cores, on a bounded token sample
  per_rank  (N > 1) every rank's gate/up fraction of HBM on its held experts and the
            exchange kernels' share of its step, with the minimum / maximum over ranks

Every step streams all touched experts' weights (~5.9 GB > 126 MB L2), so no L2 flush is
needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, TOP_K, TOKENS, SCALE = 7168, 2048, 8, 128, 2.5
EXPERTS = 256
SEED = 20261201


def profiled_traffic():
    """DRAM bytes per gate/up launch recorded by the committed ncu capture, or None."""
    p = os.path.join(ROOT, "profiles", "k_bs_grouped_c2_traffic.md")
    try:
        for line in open(p):
            if line.startswith("roofline-traffic gate_up_dram_bytes_per_launch"):
                return int(line.split()[-1])
    except OSError:
        pass
    return None


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML during the timed region (read-only)."""

    def __init__(self, device: int, period_s: float = 0.01):
        self.device, self.period, self.rows = device, period_s, []
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.device)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # no NVML: report no samples
            self.nv, self.err = None, str(e)
        return self

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.rows.append((mhz, reasons))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self.nv:
            self.t.join(timeout=2)

    def summary(self):
        if not self.nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        nv = self.nv
        names = {"hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
                 "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                 "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                 "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4)}
        seen = set()
        for _, r in self.rows:
            for n, bit in names.items():
                if r & bit:
                    seen.add(n)
        mhz = [m for m, _ in self.rows]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(mhz)}


def make_weights(seed: int, experts: int, held=None):
    """Seeded C2 weights: per expert (gate, up, down) MXFP4, then the shared expert (last), bf16
    router and bias.  Every expert has its own stream (seed + 1000 + e; shared: seed + 999), so
    a rank of an expert-parallel group draws only the experts it holds (``held``: range of
    expert ids, default all) and they equal the single-GPU weights."""
    from urbilateria_b200 import synthetic as syn

    def expert(s):
        g = syn.rng(s)
        return [syn.mxfp4_matrix(g, INTER, HIDDEN), syn.mxfp4_matrix(g, INTER, HIDDEN),
                syn.mxfp4_matrix(g, HIDDEN, INTER)]

    held = range(experts) if held is None else held
    mats = [expert(seed + 1000 + e) for e in held] + [expert(seed + 999)]
    g = syn.rng(seed)
    router = syn.bf16_normal(g, (experts, HIDDEN), 0.02)
    bias = syn.normal_f32(g, experts, 0.01)
    return mats, router, bias


def make_input(seed: int, rank: int):
    from urbilateria_b200 import synthetic as syn
    return syn.normal_bf16_as_f32(syn.rng(seed + 1 + rank), (TOKENS, HIDDEN))


def oracle_layer(mats, router, bias):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import urb_oracle as oracle
    oracle.build()
    om = [[oracle.Matrix(oracle.MXFP4, r, c, p, s, group_size=32, validate=False)
           for (p, s), (r, c) in zip(m, [(INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)])]
          for m in mats]
    ro = oracle.Matrix(oracle.BF16, EXPERTS, HIDDEN, router, validate=False)
    layer = oracle.MoeLayer(ro, bias, [m[0] for m in om[:EXPERTS]], [m[1] for m in om[:EXPERTS]],
                            [m[2] for m in om[:EXPERTS]], tuple(om[EXPERTS]), TOP_K, 1, 1, True,
                            SCALE)
    return oracle, layer, om


def cpu_tokens_per_s(layer, x, budget_s: float, threads: int):
    """Times the oracle layer token by token until the budget is spent (at least 1 token)."""
    done, t0 = 0, time.perf_counter()
    while True:
        layer.forward(x[done % x.shape[0]][None, :], threads=threads)
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s or done >= x.shape[0]:
            return done / el, done, el


def cpu_model() -> str:
    """The host CPU's model name (first /proc/cpuinfo entry), or the platform's processor."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_baseline_figures(layer, x, budget_s: float, budget_1t_s: float):
    """The oracle layer timed on all host cores and on one core (bounded token samples)."""
    threads = os.cpu_count() or 1
    layer.forward(x[:1], threads=threads)
    tps, n, el = cpu_tokens_per_s(layer, x, budget_s, threads)
    tps1, n1, el1 = cpu_tokens_per_s(layer, x, budget_1t_s, 1)
    return {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(), "value_1_thread": tps1,
            "sample": "%d tokens of the same 128-token chunk, token by token through the GLM "
                      "composition oracle on %d threads (%.1f s); 1 thread: %d tokens (%.1f s)"
                      % (n, threads, el, n1, el1)}, n


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path (restated in oracle/) on the host cores."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    mats, router, bias = make_weights(SEED, EXPERTS)
    _, layer, _ = oracle_layer(mats, router, bias)
    x = make_input(SEED, 0)
    for _ in range(max(0, min(args.warmup, 1))):
        layer.forward(x[:1], threads=threads)
    # Each step is a bounded sample; the whole run stays within about two minutes whatever
    # --steps is (at least 0.5 s of work per step).
    step_s = max(0.5, min(args.ref_step_s, 120.0 / max(1, args.steps)))
    vals = []
    t_all = time.perf_counter()
    for s in range(args.steps):
        tps, n, el = cpu_tokens_per_s(layer, x[s % TOKENS:], step_s, threads)
        vals.append(tps)
    total = time.perf_counter() - t_all
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": "moe_layer_tokens_per_s", "value": v,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * TOKENS / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": workload_config(world),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "cpu_model": cpu_model(),
                             "sample": "token-by-token GLM composition until %.1fs per step "
                                       "(oracle/urb_oracle.cpp, ordered-F64 Rayon-style row "
                                       "parallelism)" % step_s},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "wall_s": total}
    print(json.dumps(line), flush=True)


def bench_matvec(urb, ctx, stream, local, pk_hbm, copies=20, reps=10):
    """Config 0 (MXFP4 matvec 4096x7168, E8M0 119..127, x ~ N(0,1)): 20 distinct weight copies
    (312 MB > 2x L2) are used round-robin so every launch streams from HBM.  The launches are
    captured once in a CUDA graph and replayed, so the CUDA-event time is device time, not the
    host's per-call launch cost."""
    import torch
    from urbilateria_b200 import synthetic as syn
    g = syn.rng(SEED + 7)
    rows, cols = 4096, 7168
    mats = [urb.MxFp4Matrix.from_packed(rows, cols, 32, *syn.mxfp4_matrix(g, rows, cols), ctx=ctx)
            for _ in range(copies)]
    x = torch.from_numpy(syn.normal_f32(g, cols)).to(f"cuda:{local}")
    y = torch.empty(rows, device=f"cuda:{local}")
    for m in mats[:3]:
        m.matmul_rows_device(x.data_ptr(), 1, y.data_ptr())
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for m in mats:
            m.matmul_rows_device(x.data_ptr(), 1, y.data_ptr())
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        stream.synchronize()
    ms = e0.elapsed_time(e1) / (reps * copies)
    nbytes = rows * cols // 2 + rows * cols // 32 + cols * 4 + rows * 4
    gbs = nbytes / (ms / 1e3) / 1e9
    del graph
    for m in mats:
        m.free()
    kernel = ("k_matvec1<MXFP4> (CUDA cores, 16-row blocks)" if os.environ.get("URB_MATVEC") == "cuda_cores"
              else "k_mv_tc<MXFP4> (tcgen05 kind::mxf4, x as 12 E2M1 digit terms, split-K clusters)")
    return {"kernel": kernel, "us_per_launch": ms * 1e3,
            "bytes_per_launch": nbytes, "achieved_gbs": gbs, "frac_of_measured_hbm": gbs / pk_hbm,
            "launches": reps * copies,
            "l2": "20 distinct 15.6 MB weight copies round-robin; CUDA-graph replay"}


def kernel_ms(ctx, native, fn, reps):
    """Runs fn() reps times with the library profiler on: device ms per call summed over the
    library's kernels (launch gaps excluded), and the stream's ms per call (events)."""
    import ctypes
    import torch
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    ctx.lib.urb_profile_reset(ctx.h)
    ctx.lib.urb_profile_enable(ctx.h, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ctx.lib.urb_profile_enable(ctx.h, 0)
    total, launches, per_kind = 0.0, 0, {}
    for k, name in enumerate(native.KERNEL_NAMES):
        t, n = ctypes.c_double(), ctypes.c_int64()
        ctx.lib.urb_profile_read(ctx.h, k, ctypes.byref(t), ctypes.byref(n))
        total += t.value
        launches += n.value
        if n.value:
            per_kind[name] = t.value / reps * 1e3
    kernel_ms.per_kind = per_kind  # microseconds per call, by kernel kind, of the last run
    return total / reps, e0.elapsed_time(e1) / reps, launches // reps


def bench_c1(urb, native, ctx, dev, pk_hbm, g):
    """Config 1: BF16 SwiGLU FFN (urb_gated_mlp_forward_device) at T = 1 and 32."""
    import torch
    from urbilateria_b200 import synthetic as syn
    # Config 1: BF16 SwiGLU FFN, gate/up [768 x 2048], down [2048 x 768] ~ N(0, 0.02); T = 1
    # and 32.  9.4 MB of weights fit L2, so 27 distinct copies (254 MB) are used in turn.
    H1, I1, copies = 2048, 768, 27
    gb, ub, db = (syn.bf16_normal(g, (I1, H1), 0.02), syn.bf16_normal(g, (I1, H1), 0.02),
                  syn.bf16_normal(g, (H1, I1), 0.02))
    mlps = [(urb.Bf16Matrix.from_bits(I1, H1, gb, ctx=ctx), urb.Bf16Matrix.from_bits(I1, H1, ub, ctx=ctx),
             urb.Bf16Matrix.from_bits(H1, I1, db, ctx=ctx)) for _ in range(copies)]
    c1 = {"workload": "C1 BF16 SwiGLU FFN, hidden 2048, intermediate 768", "weights_copies": copies}
    for T in (1, 32):
        d_x = torch.from_numpy(syn.normal_bf16_as_f32(g, (T, H1))).to(dev)
        d_y = torch.empty_like(d_x)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        it = [0]

        def fn():
            m = mlps[it[0] % copies]
            it[0] += 1
            ctx.check(ctx.lib.urb_gated_mlp_forward_device(ctx.h, m[0].h, m[1].h, m[2].h,
                                                           d_x.data_ptr(), T, d_y.data_ptr(),
                                                           st.data_ptr()))
        for _ in range(copies):
            fn()
        k_ms, s_ms, n = kernel_ms(ctx, native, fn, 4 * copies)
        # The products are a few microseconds, less than the host needs to issue them, so the
        # device time is taken from a CUDA graph of one call per weight copy.
        stream = torch.cuda.current_stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(copies):
                fn()
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(10):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        g_ms = e0.elapsed_time(e1) / (10 * copies)
        del graph
        if int(st.item()) != 0:
            raise RuntimeError("config 1 forward reported status %d" % int(st.item()))
        nbytes = 3 * I1 * H1 * 2 + T * (H1 * 4 + H1 * 4)
        c1["T%d" % T] = {"us": g_ms * 1e3, "timing": "CUDA-graph replay, device time per call",
                         "eager_stream_us": s_ms * 1e3, "launches": n,
                         "tokens_per_s": T / (g_ms / 1e3), "bytes": nbytes,
                         "achieved_gbs": nbytes / (g_ms / 1e3) / 1e9,
                         "frac_of_measured_hbm": nbytes / (g_ms / 1e3) / 1e9 / pk_hbm}
    for m in mlps:
        for x in m:
            x.free()
    return c1


def bench_configs(urb, native, ctx, local, pk_hbm):
    """Configs 1, 3 and 4 of the benchmark set, each timed on this GPU with the library's own
    device API (inputs resident), reported beside its algorithmic bytes and the measured HBM
    peak.  Device time is the sum of the library's kernels per call (the profiler's events),
    which for the small C1 product excludes the host's launch cadence."""
    import torch
    from urbilateria_b200 import synthetic as syn
    dev = f"cuda:{local}"
    out = {}
    g = syn.rng(SEED + 11)

    out["c1"] = bench_c1(urb, native, ctx, dev, pk_hbm, g)

    out["c3"] = bench_c3(urb, native, ctx, dev, pk_hbm, g)
    out["c4"] = bench_c4(urb, native, ctx, local, pk_hbm, 1, 0)
    out["int_glm"] = bench_int(urb, ctx, g, dev, pk_hbm)
    return out


def bench_c3(urb, native, ctx, dev, pk_hbm, g, E3=128):
    """Config 3: MXFP8 experts (hidden 4096, intermediate 1536; E4M3 fp8-cast N(0,1), E8M0
    117..123 per 32), 512 tokens with Zipf(1.1) top-8 routes: the experts half of the layer with
    the caller's routes.  Every expert is its own HBM copy of one generated matrix set.  E3 = 128
    is config 3; fewer experts only for profiling captures."""
    import torch
    from urbilateria_b200 import synthetic as syn
    out = {}
    H3, I3, T3, K3 = 4096, 1536, 512, 8
    gv, gs = syn.mxfp8_matrix(g, I3, H3)
    uv, us_ = syn.mxfp8_matrix(g, I3, H3)
    dv, ds = syn.mxfp8_matrix(g, H3, I3)
    experts = [urb.GatedMlp(urb.MxFp8Matrix.from_packed(I3, H3, 1, 32, gv, gs, ctx=ctx),
                            urb.MxFp8Matrix.from_packed(I3, H3, 1, 32, uv, us_, ctx=ctx),
                            urb.MxFp8Matrix.from_packed(H3, I3, 1, 32, dv, ds, ctx=ctx))
               for _ in range(E3)]
    r3 = urb.Bf16Matrix.from_bits(E3, H3, syn.bf16_normal(g, (E3, H3), 0.02), ctx=ctx)
    layer3 = urb.RuntimeMoeLayer(r3, np.zeros(E3, np.float32), experts, None,
                                 urb.MoeGeometry(K3, 1, 1, True, 1.0))
    ids = syn.zipf_routes(g, T3, E3, K3).astype(np.int32)
    w = g.random((T3, K3)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    d_x = torch.from_numpy(syn.normal_bf16_as_f32(g, (T3, H3))).to(dev)
    d_ids, d_w = torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev)
    d_y = torch.empty_like(d_x)
    st = torch.zeros(1, dtype=torch.int32, device=dev)

    def fn3():
        ctx.check(ctx.lib.urb_moe_forward_routed_device(ctx.h, layer3.h, d_x.data_ptr(), T3,
                                                        d_ids.data_ptr(), d_w.data_ptr(),
                                                        d_y.data_ptr(), st.data_ptr()))
    for _ in range(3):
        fn3()
    k_ms, s_ms, n = kernel_ms(ctx, native, fn3, 10)
    if int(st.item()) != 0:
        raise RuntimeError("config 3 forward reported status %d" % int(st.item()))
    counts = np.bincount(ids.ravel(), minlength=E3)
    per_expert = 3 * (I3 * H3 + I3 * H3 // 32)
    nbytes = int((counts > 0).sum()) * per_expert
    flops = 2.0 * T3 * K3 * 3 * I3 * H3
    out["c3"] = {"workload": "C3 MXFP8 grouped experts: %d x (4096 x 1536 SwiGLU), 512 tokens, " % E3 +
                             "Zipf(1.1) top-8 (caller routes)",
                 "kernel_us": k_ms * 1e3, "stream_us": s_ms * 1e3, "launches": n,
                 "tokens_per_s": T3 / (k_ms / 1e3), "touched_experts": int((counts > 0).sum()),
                 "max_expert_tokens": int(counts.max()), "bytes": nbytes,
                 "kernels_us": kernel_ms.per_kind,
                 "achieved_gbs": nbytes / (k_ms / 1e3) / 1e9,
                 "frac_of_measured_hbm": nbytes / (k_ms / 1e3) / 1e9 / pk_hbm,
                 "tflops": flops / (k_ms / 1e3) / 1e12}
    layer3.free()
    for e in experts:
        for mtx in (e.gate, e.up, e.down):
            mtx.free()
    r3.free()
    return out["c3"]


def c4_weights(urb, ctx, dev, layer, held, experts=384):
    """Config 4 layer `layer`: MXFP4 gate/up [2048 x 7168] and down [7168 x 2048] for the routed
    experts in `held` plus the shared expert (nibbles uniform 0..15, E8M0 uniform 119..127,
    drawn on the GPU from one generator per expert, so every rank draws the same weights for
    the experts it holds), a bf16 router [384 x 7168] ~ N(0, 0.02) and a bias ~ N(0, 0.01)."""
    import torch
    from urbilateria_b200 import synthetic as syn

    def mlp(seed):
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        mats = []
        for r, c in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)):
            p = torch.randint(0, 256, (r * c // 2,), dtype=torch.uint8, device=dev, generator=gen)
            sc = torch.randint(119, 128, (r * c // 32,), dtype=torch.uint8, device=dev, generator=gen)
            mats.append(urb.MxFp4Matrix.from_device(r, c, 32, p.data_ptr(), p.numel(), sc.data_ptr(),
                                                    sc.numel(), ctx=ctx))
        return urb.GatedMlp(*mats)
    base = SEED + 40000 * (layer + 1)
    routed = [mlp(base + e) for e in held]
    shared = mlp(base + experts)
    g = syn.rng(base)
    router = urb.Bf16Matrix.from_bits(experts, HIDDEN, syn.bf16_normal(g, (experts, HIDDEN), 0.02), ctx=ctx)
    return routed, shared, router, syn.normal_f32(g, experts, 0.01)


def bench_bf16_layer(urb, native, ctx, local, pk_hbm, tokens=128):
    """A Qwen3.6-A3B-shaped BF16 MoE layer (hidden 2048, 128 BF16 experts of intermediate 768,
    top-8 + a shared expert, bf16 router ~ N(0, 0.02), weights ~ N(0, 0.02)): the layer forward
    on the tcgen05 kind::f16 grouped passes, tokens/s and the per-kernel device times."""
    import torch
    from urbilateria_b200 import synthetic as syn
    dev = f"cuda:{local}"
    H, I, E, K = 2048, 768, 128, 8
    g = syn.rng(SEED + 19)

    def mlp():
        return urb.GatedMlp(urb.Bf16Matrix.from_bits(I, H, syn.bf16_normal(g, (I, H), 0.02), ctx=ctx),
                            urb.Bf16Matrix.from_bits(I, H, syn.bf16_normal(g, (I, H), 0.02), ctx=ctx),
                            urb.Bf16Matrix.from_bits(H, I, syn.bf16_normal(g, (H, I), 0.02), ctx=ctx))
    experts = [mlp() for _ in range(E)]
    shared = mlp()
    router = urb.Bf16Matrix.from_bits(E, H, syn.bf16_normal(g, (E, H), 0.02), ctx=ctx)
    layer = urb.RuntimeMoeLayer(router, syn.normal_f32(g, E, 0.01), experts, shared,
                                urb.MoeGeometry(K, 1, 1, True, 1.0))
    d_x = torch.from_numpy(syn.normal_bf16_as_f32(g, (tokens, H))).to(dev)
    d_y = torch.empty_like(d_x)
    st = torch.zeros(1, dtype=torch.int32, device=dev)

    def fn():
        layer.forward_device(d_x.data_ptr(), tokens, d_y.data_ptr(), 0, 0, st.data_ptr())
    for _ in range(5):
        fn()
    k_ms, s_ms, n = kernel_ms(ctx, native, fn, 20)
    if int(st.item()) != 0:
        raise RuntimeError("BF16 layer forward reported status %d" % int(st.item()))
    per_expert = 3 * H * I * 2
    out = {"workload": "Qwen3.6-A3B-shaped BF16 MoE layer: hidden 2048, 128 experts inter 768 top-8 + "
                       "shared, %d tokens" % tokens,
           "stream_us": s_ms * 1e3, "kernel_us": k_ms * 1e3, "launches": n,
           "tokens_per_s": tokens / (s_ms / 1e3), "kernels_us": kernel_ms.per_kind,
           "weight_bytes": (E + 1) * per_expert}
    layer.free()
    for e in experts + [shared]:
        for m in (e.gate, e.up, e.down):
            m.free()
    router.free()
    return out


def bench_c4_layer(urb, native, ctx, local, pk_hbm):
    """One config-4 layer (384 MXFP4 experts + shared, hidden 7168) at B = 1 and 8: the graph
    time of one forward and the library's per-kernel device times (for profiling the decode
    path's kernel chain)."""
    import torch
    from urbilateria_b200 import synthetic as syn
    dev = f"cuda:{local}"
    stream = torch.cuda.current_stream()
    routed, shared, router, bias = c4_weights(urb, ctx, dev, 0, range(384))
    layer = urb.RuntimeMoeLayer(router, bias, routed, shared, urb.MoeGeometry(TOP_K, 1, 1, True, SCALE))
    g = syn.rng(SEED + 17)
    out = {"workload": "one C4 layer: 7168, 384 MXFP4 experts top-8 + 1 shared, inter 2048"}
    for B in (1, 8):
        d_x = torch.from_numpy(syn.normal_bf16_as_f32(g, (B, HIDDEN))).to(dev)
        d_y = torch.empty_like(d_x)
        st = torch.zeros(1, dtype=torch.int32, device=dev)

        def fn():
            layer.forward_device(d_x.data_ptr(), B, d_y.data_ptr(), 0, 0, st.data_ptr())
        for _ in range(5):
            fn()
        k_ms, s_ms, n = kernel_ms(ctx, native, fn, 20)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(20):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        if int(st.item()) != 0:
            raise RuntimeError("config 4 layer forward reported status %d" % int(st.item()))
        out["B%d" % B] = {"graph_us": e0.elapsed_time(e1) / 20 * 1e3, "stream_us": s_ms * 1e3,
                          "launches": n, "kernels_us": kernel_ms.per_kind}
    layer.free()
    for e in routed + [shared]:
        for m in (e.gate, e.up, e.down):
            m.free()
    router.free()
    return out


def bench_c4(urb, native, ctx, local, pk_hbm, world, rank, dist=None):
    """Config 4: 4 stacked MoE layers, each with its own 384 MXFP4 routed experts (top-8, the
    config-2 routing) + 1 shared expert (4 x 385 x 23.4 MB = 36 GB of distinct weights on one
    GPU), h <- h + MoE_l(h) then rescaled to unit RMS (the synthetic weights grow h ~10^5 per
    layer and would overflow f32 within a step; the rescale stands in for the norm a real model
    has between layers), decode batches of B = 1 / 8 / 64 one-token sequences.  One GPU: the
    layers run whole and the step is also timed as one CUDA graph.  N GPUs: rank r holds
    experts shard_range(384, N, r) of every layer plus the replicated router and shared expert
    and owns token_range(B, N, r) of the batch (expert parallel, tokens and outputs over
    NVLink); the step time is the max over ranks."""
    import torch
    from urbilateria_b200 import synthetic as syn
    from urbilateria_b200.expert_parallel import ExpertParallelMoeLayer, shard_range, token_range
    dev = f"cuda:{local}"
    E4, L4 = 384, 4
    eb, ec = shard_range(E4, world, rank) if world > 1 else (0, E4)
    geo = urb.MoeGeometry(TOP_K, 1, 1, True, SCALE)
    layers, eps, owned = [], [], []
    t0 = time.perf_counter()
    for l in range(L4):
        routed, shared, router, bias = c4_weights(urb, ctx, dev, l, range(eb, eb + ec), E4)
        owned.append((routed, shared, router))
        if world == 1:
            layers.append(urb.RuntimeMoeLayer(router, bias, routed, shared, geo))
        else:
            lay = urb.RuntimeMoeLayer(router, bias, routed, shared, geo, expert_range=(eb, ec))
            layers.append(lay)
            eps.append(ExpertParallelMoeLayer(lay, world, rank, 64, timeout_ms=20000))
    torch.cuda.synchronize()
    per_expert = 3 * (INTER * HIDDEN // 2 + INTER * HIDDEN // 32)
    c4 = {"workload": "C4 stacked MoE decode: 4 distinct layers x (7168, 384 MXFP4 experts top-8 "
                      "+ 1 shared, inter 2048), h <- h + MoE(h) rescaled to unit RMS",
          "layers": L4, "resident_weight_bytes_per_gpu": L4 * (ec + 1) * per_expert,
          "upload_s": time.perf_counter() - t0,
          "parallelism": "ep%d" % world if world > 1 else "single"}
    g = syn.rng(SEED + 13)
    for B in (1, 8, 64):
        h_all = syn.normal_bf16_as_f32(g, (B, HIDDEN))
        tb, tc_ = token_range(B, world, rank) if world > 1 else (0, B)
        d_h = torch.from_numpy(h_all[tb:tb + tc_].copy()).to(dev) if tc_ else torch.empty((0, HIDDEN), device=dev)
        d_o = torch.empty_like(d_h)
        d_ids = torch.empty((max(tc_, 1), TOP_K), dtype=torch.int32, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)

        def step(record=None):
            for li, lay in enumerate(layers):
                if world == 1:
                    lay.forward_device(d_h.data_ptr(), B, d_o.data_ptr(), d_ids.data_ptr() if record is not None else 0,
                                       0, st.data_ptr())
                else:
                    eps[li].forward_device(d_h.data_ptr() if tc_ else 0, tc_, d_o.data_ptr() if tc_ else 0,
                                           st.data_ptr(), d_ids.data_ptr() if (tc_ and record is not None) else 0)
                if record is not None and tc_:
                    record.append(d_ids[:tc_].cpu().numpy().copy())
                if tc_:
                    d_h.add_(d_o)
                    d_h.mul_(torch.rsqrt(d_h.square().mean(dim=1, keepdim=True)))
        # Experts each layer touches (bytes the step must stream), from one recorded step.
        rec = []
        step(rec)
        torch.cuda.synchronize()
        if int(st.item()) != 0:
            c4["B%d" % B] = {"error": "status %d" % int(st.item())}
            continue
        touched = 0
        for li in range(L4):
            ids = rec[li] if rec and tc_ else np.zeros((0, TOP_K), np.int32)
            if world > 1:
                every = [None] * world
                dist.all_gather_object(every, ids)
                ids = np.concatenate([e for e in every if e is not None and len(e)]) if any(
                    e is not None and len(e) for e in every) else ids
            mine = np.unique(ids[(ids >= eb) & (ids < eb + ec)]) if ids.size else []
            touched += len(mine) + 1
        for _ in range(3):
            step()
        stream = torch.cuda.current_stream()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        step_us = e0.elapsed_time(e1) / reps * 1e3
        graph_us = None
        if world == 1:
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    step()
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize()
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                graph_us = e0.elapsed_time(e1) / reps * 1e3
                del graph
            except Exception as exc:  # capture refused: report the eager figures only
                graph_us = "not captured: %s" % str(exc).splitlines()[0][:120]
        if dist:
            t = torch.tensor([step_us], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            step_us = float(t.item())
        if int(st.item()) != 0:
            c4["B%d" % B] = {"error": "status %d" % int(st.item())}
            continue
        nbytes = touched * per_expert + L4 * E4 * HIDDEN * 2
        best = graph_us if isinstance(graph_us, float) else step_us
        c4["B%d" % B] = {"step_us": step_us, "graph_us": graph_us,
                         "tokens_per_s": B / (best / 1e6),
                         "touched_experts_per_step_this_gpu": touched,
                         "bytes_per_step_this_gpu": nbytes,
                         "achieved_gbs_this_gpu": nbytes / (best / 1e6) / 1e9,
                         "frac_of_measured_hbm": nbytes / (best / 1e6) / 1e9 / pk_hbm,
                         "timing": ("CUDA-graph replay of the 4-layer step" if isinstance(graph_us, float)
                                    else "eager stream, max over ranks")}
    for ep in eps:
        ep.free()
    for lay in layers:
        lay.free()
    for routed, shared, router in owned:
        for e in routed + [shared]:
            for mtx in (e.gate, e.up, e.down):
                mtx.free()
        router.free()
    return c4


def bench_int(urb, ctx, g, dev, pk_hbm, reps=5):
    """GLM converted-checkpoint formats (Int4Matrix with 64-column groups, Int8Matrix per row),
    2048 x 7168, at 1 and 8 tokens: device time of one product as CUDA-graph replays over
    distinct copies (>= 260 MB, so weights stream from HBM), beside the payload + scale bytes."""
    import math
    import numpy as np
    import torch
    stream = torch.cuda.ExternalStream(ctx.stream)
    rows, cols, grp = 2048, 7168, 64
    res = {}
    for fmt in ("int4", "int8"):
        if fmt == "int4":
            packed = g.integers(0, 256, size=rows * cols // 2, dtype=np.uint8)
            scales = (np.abs(g.standard_normal(rows * cols // grp)) * 0.02 + 1e-3).astype(np.float32)
            nbytes = packed.size + scales.size * 4
            make = lambda: urb.Int4Matrix.from_packed(rows, cols, grp, packed, scales, ctx=ctx)
        else:
            data = g.integers(-128, 128, size=(rows, cols)).astype(np.int8)
            scales = (np.abs(g.standard_normal(rows)) * 0.01 + 1e-4).astype(np.float32)
            nbytes = data.size + rows * 4
            make = lambda: urb.Int8Matrix.from_packed(rows, cols, data, scales, ctx=ctx)
        mats = [make() for _ in range(math.ceil(260e6 / nbytes))]
        for T in (1, 8):
            x = torch.randn(T, cols, device=dev)
            y = torch.empty(T, rows, device=dev)
            for m in mats[:3]:
                m.matmul_rows_device(x.data_ptr(), T, y.data_ptr())
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for m in mats:
                    m.matmul_rows_device(x.data_ptr(), T, y.data_ptr())
            with torch.cuda.stream(stream):
                for _ in range(3):
                    graph.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                stream.synchronize()
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
                stream.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(mats))
            gbs = nbytes / (us / 1e6) / 1e9
            res[f"{fmt}_T{T}"] = {"us": us, "bytes": nbytes, "achieved_gbs": gbs,
                                  "frac_of_measured_hbm": gbs / pk_hbm}
            del graph
        for m in mats:
            m.free()
    return {"workload": "GLM INT4 (group 64) / INT8 (per-row) matrix 2048 x 7168, 1 and 8 tokens",
            "copies": "distinct weight copies >= 260 MB, CUDA-graph replay", **res}


def workload_config(world):
    return {"workload": "C2 MXFP4 MoE layer: hidden 7168, 256+1 experts, inter 2048, top-8 "
                        "noaux_tc x2.5, 128-token chunk per GPU",
            "hidden": HIDDEN, "experts": EXPERTS, "shared_experts": 1, "intermediate": INTER,
            "top_k": TOP_K, "tokens_per_gpu": TOKENS, "weights": "MXFP4 E2M1+E8M0/32",
            "parallelism": "ep%d" % world if world > 1 else "single",
            "l2": "working set 5.9 GB/step > 126 MB L2 (no flush needed)", "seed": SEED}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-step-s", type=float, default=4.0)
    ap.add_argument("--cpu-sample-s", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-matvec", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the config 1 / 3 / 4 measurements")
    ap.add_argument("--experts", type=int, default=256,
                    help="routed experts (256 = config 2; smaller only for profiling captures)")
    ap.add_argument("--tokens", type=int, default=128,
                    help="tokens per GPU (128 = config 2; other values only for profiling)")
    ap.add_argument("--int-only", action="store_true",
                    help="profiling: time only the INT4 / INT8 products and print their figures")
    ap.add_argument("--only", choices=["matvec", "c1", "c3", "c4layer", "bf16layer"],
                    help="profiling: time only the config-0 matvec, config 1, config 3, one config-4 "
                         "layer or a BF16 (Qwen3.6-shaped) layer and print its figures")
    ap.add_argument("--c3-experts", type=int, default=128,
                    help="experts of --only c3 (128 = config 3; fewer only for profiling captures)")
    args = ap.parse_args()
    global EXPERTS, TOKENS
    EXPERTS = args.experts
    TOKENS = args.tokens

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import urbilateria_b200 as urb
    from urbilateria_b200 import native

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))

    ctx = urb.Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    if args.only:
        from urbilateria_b200 import synthetic as syn
        with torch.cuda.stream(stream):
            if args.only == "matvec":
                res = bench_matvec(urb, ctx, stream, local, peaks()[0])
            elif args.only == "c1":
                res = bench_c1(urb, native, ctx, f"cuda:{local}", peaks()[0], syn.rng(SEED + 11))
            elif args.only == "c4layer":
                res = bench_c4_layer(urb, native, ctx, local, peaks()[0])
            elif args.only == "bf16layer":
                res = bench_bf16_layer(urb, native, ctx, local, peaks()[0])
            else:
                res = bench_c3(urb, native, ctx, f"cuda:{local}", peaks()[0], syn.rng(SEED + 11),
                               args.c3_experts)
        print(json.dumps(res))
        return
    if args.int_only:
        from urbilateria_b200 import synthetic as syn
        print(json.dumps(bench_int(urb, ctx, syn.rng(SEED + 11), f"cuda:{local}",
                                   peaks()[0])))
        return

    keep_host = (rank == 0 and world == 1 and not args.no_cpu)
    # One GPU: the whole layer.  N GPUs: expert parallel, rank r holding experts
    # shard_range(256, N, r) (plus the replicated router and shared expert) and its own
    # 128-token chunk; token rows and expert outputs cross NVLink inside the kernels.
    from urbilateria_b200.expert_parallel import ExpertParallelMoeLayer, shard_range
    eb, ec = shard_range(EXPERTS, world, rank) if world > 1 else (0, EXPERTS)
    mats, router, bias = make_weights(SEED, EXPERTS, range(eb, eb + ec))
    dev = []
    for m in mats:
        gm = [urb.MxFp4Matrix.from_packed(r, c, 32, p, s, ctx=ctx)
              for (p, s), (r, c) in zip(m, [(INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER)])]
        dev.append(urb.GatedMlp(*gm))
    rd = urb.Bf16Matrix.from_bits(EXPERTS, HIDDEN, router, ctx=ctx)
    geo = urb.MoeGeometry(TOP_K, 1, 1, True, SCALE)
    if world == 1:
        layer = urb.RuntimeMoeLayer(rd, bias, dev[:ec], dev[ec], geo)
        ep = None
    else:
        layer = urb.RuntimeMoeLayer(rd, bias, dev[:ec], dev[ec], geo, expert_range=(eb, ec))
        ep = ExpertParallelMoeLayer(layer, world, rank, TOKENS, timeout_ms=20000)
    if not keep_host:
        del mats

    x = make_input(SEED, rank)
    d_x = torch.from_numpy(x).to(f"cuda:{local}")
    d_out = torch.empty_like(d_x)
    d_status = torch.zeros(1, dtype=torch.int32, device=f"cuda:{local}")
    # Routing of this input (identical every step): touched experts for the roofline bytes.
    if ep is None:
        out0, ids0, w0, extra = layer.forward_batch(x, TOKENS, details=True)
        touched = int((extra["counts"] > 0).sum())
    else:
        dist.barrier()
        out0, ids0, w0 = ep.forward_batch(x, TOKENS)
        every = [None] * world
        dist.all_gather_object(every, ids0)
        ids_all = np.concatenate(every).ravel()
        touched = int(np.unique(ids_all[(ids_all >= eb) & (ids_all < eb + ec)]).size)
    pk_hbm, pk_tf, pk_kind = peaks()

    if ep is None:
        def step():
            layer.forward_device(d_x.data_ptr(), TOKENS, d_out.data_ptr(), 0, 0,
                                 d_status.data_ptr())
    else:
        def step():
            ep.forward_device(d_x.data_ptr(), TOKENS, d_out.data_ptr(), d_status.data_ptr())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        if dist:
            dist.barrier()
        ctx.lib.urb_profile_reset(ctx.h)
        ctx.lib.urb_profile_enable(ctx.h, 1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                step()
            e1.record(stream)
            torch.cuda.synchronize()
        ctx.lib.urb_profile_enable(ctx.h, 0)
        ms = e0.elapsed_time(e1)
        # Per-kernel device time of the timed region.
        import ctypes
        kern = {}
        for k, name in enumerate(native.KERNEL_NAMES):
            t, n = ctypes.c_double(), ctypes.c_int64()
            ctx.lib.urb_profile_read(ctx.h, k, ctypes.byref(t), ctypes.byref(n))
            if n.value:
                kern[name] = {"ms_per_launch": t.value / n.value, "launches": n.value}
        # The profiler's events add a little overhead; time the same steps without it too.
        stream.synchronize()
        if dist:
            dist.barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = min(ms, e0.elapsed_time(e1))

    matvec = None if (args.no_matvec or world > 1) else bench_matvec(urb, ctx, stream, local, pk_hbm)
    configs = None
    if not args.no_configs and world == 1:
        with torch.cuda.stream(stream):
            configs = bench_configs(urb, native, ctx, local, pk_hbm)

    # End to end through the host-pointer ABI (pinned host input/output).
    hx = torch.from_numpy(x).pin_memory()
    hout = torch.empty_like(hx).pin_memory()
    hid = torch.empty((TOKENS, TOP_K), dtype=torch.int32).pin_memory()
    hw = torch.empty((TOKENS, TOP_K), dtype=torch.float32).pin_memory()

    def e2e_step():
        if ep is None:
            ctx.check(ctx.lib.urb_moe_forward(ctx.h, layer.h, hx.data_ptr(), TOKENS,
                                              hout.data_ptr(), hid.data_ptr(), hw.data_ptr(),
                                              None, None, None, None, None))
        else:
            ctx.check(ctx.lib.urb_ep_forward(ctx.h, ep.h, hx.data_ptr(), TOKENS, hout.data_ptr(),
                                             hid.data_ptr(), hw.data_ptr()))

    ms_e2e = float("nan")
    if not args.no_e2e:
        for _ in range(2):
            e2e_step()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1)

    if dist:
        t = torch.tensor([ms, ms_e2e], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = t.tolist()

    tokens_total = TOKENS * world * args.steps
    value = tokens_total / (ms / 1e3)
    e2e = tokens_total / (ms_e2e / 1e3)

    # Roofline of the dominant kernel: the grouped gate/up pass streams gate+up of every
    # touched expert (held by this rank) and of the shared expert once, 2 * (7,340,032 packed +
    # 458,752 scale) bytes per expert, and writes the f32 h = silu(gate) * up row of every
    # activation column (routes to the held experts + own tokens).
    gu_bytes_per_expert = 2 * (INTER * HIDDEN // 2 + INTER * HIDDEN // 32)
    n_cols = (TOKENS * TOP_K + TOKENS) if ep is None else \
        int(((ids_all >= eb) & (ids_all < eb + ec)).sum()) + TOKENS
    gu_bytes = (touched + 1) * gu_bytes_per_expert + n_cols * INTER * 4
    gu = kern.get("gate_up", {})
    achieved = gu_bytes / (gu.get("ms_per_launch", float("nan")) / 1e3) / 1e9
    roofline = {"kernel": "k_bs_grouped<MXFP4> gate/up (tcgen05.mma kind::mxf4 block_scale)",
                "bound": "hbm", "achieved": achieved, "peak": pk_hbm, "unit": "GB/s",
                "frac": achieved / pk_hbm, "peak_kind": pk_kind, "bytes_per_launch": gu_bytes,
                "traffic": profiled_traffic()}
    dn_bytes = (touched + 1) * (HIDDEN * INTER // 2 + HIDDEN * INTER // 32)
    dn = kern.get("down", {})
    layer_bytes = (touched + 1) * 3 * (INTER * HIDDEN // 2 + INTER * HIDDEN // 32) + \
        EXPERTS * HIDDEN * 2
    if ep is not None:
        roofline["note"] = "rank 0 of %d: %d held experts touched, %d activation columns" % (
            world, touched, n_cols)

    per_rank = None
    if dist:
        # Every rank's own figures (the layer's load differs by rank with the routes): gate/up
        # fraction of HBM on its held experts, and the exchange kernels' share of the step.
        ex = kern.get("exchange", {})
        ex_us = ex.get("ms_per_launch", 0.0) * ex.get("launches", 0) / args.steps * 1e3
        mine = {"rank": rank, "touched_experts": touched, "activation_columns": n_cols,
                "gate_up_us": gu.get("ms_per_launch", float("nan")) * 1e3,
                "gate_up_frac_of_hbm": achieved / pk_hbm,
                "down_us": dn.get("ms_per_launch", float("nan")) * 1e3,
                "exchange_us_per_step": ex_us,
                "exchange_share_of_step": ex_us / (ms / args.steps * 1e3)}
        every = [None] * world
        dist.all_gather_object(every, mine)
        per_rank = {"ranks": every,
                    "min_gate_up_frac_of_hbm": min(r["gate_up_frac_of_hbm"] for r in every),
                    "max_exchange_share_of_step": max(r["exchange_share_of_step"] for r in every)}

    line = {"metric": "moe_layer_tokens_per_s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "mxf4: E2M1 weights x E2M1 activation residual terms (6 per token), E8M0 "
                     "scales, f32 accumulate",
            "data": "synthetic", "config": workload_config(world),
            "e2e": {"value": e2e, "unit": "tokens/s",
                    "h2d_bytes_per_step": TOKENS * HIDDEN * 4,
                    "d2h_bytes_per_step": TOKENS * HIDDEN * 4 + TOKENS * TOP_K * 8},
            "roofline": roofline,
            "layer_hbm_gbs": layer_bytes / (ms / args.steps / 1e3) / 1e9,
            "down_gbs": dn_bytes / (dn.get("ms_per_launch", float("nan")) / 1e3) / 1e9,
            "touched_experts": touched, "held_experts": [eb, ec], "kernels": kern,
            "per_rank": per_rank, "matvec_c0": matvec, "configs": configs,
            # Kernels per profiled region: the router-logits region launches two (the x
            # widening and the f64 chain kernel), every other region one.
            "gpu_launches": sum(v["launches"] * (2 if k == "router_logits" else 1) for k, v in kern.items()),
            "clocks": clk.summary()}

    if rank == 0 and world == 1 and not args.no_cpu:
        oracle, olayer, _ = oracle_layer(mats, router, bias)
        threads = os.cpu_count() or 1
        line["cpu_baseline"], n = cpu_baseline_figures(olayer, x, args.cpu_sample_s,
                                                       args.cpu_sample_s / 2)
        # Parity of the benchmarked forward on the sampled tokens (routes must match).
        o_out, o_ids, _, _, _ = olayer.forward(x[:n], threads=threads)
        line["parity_sample"] = {
            "tokens": n, "routes_equal": bool(np.array_equal(o_ids, ids0[:n])),
            "rel_l2": float(np.linalg.norm(out0[:n] - o_out) / np.linalg.norm(o_out))}
    if world > 1 and not args.no_configs:
        # Config 4 expert parallel across the group (stacked decode, B = 1 / 8 / 64 in all).
        with torch.cuda.stream(stream):
            line["configs"] = {"c4": bench_c4(urb, native, ctx, local, pk_hbm, world, rank, dist)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
