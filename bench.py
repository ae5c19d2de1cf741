#!/usr/bin/env python
"""Benchmark of the fused int4 GEMV hot path on B200.

Metric: q4 GEMV achieved HBM GB/s on the int4 projections of one
Qwen2-7B-shape decoder layer at batch 1 (the benchmark's second config: q
3584->3584, k/v 3584->512, o 3584->3584, gate/up 3584->18944, down
18944->3584, group size 64).  A step is one pass of the layer's projections
as the device stage launches them: q|k|v (one launch, rows concatenated), o,
gate|up (one launch), down -- four launches of the GEMV kernel, each from its
own fp32 activation row.  Weights are random (synthetic, seeded) in the
reference's packed layout; four copies of the layer (526 MB, larger than the
126 MB L2) rotate between steps so every step streams from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun, one rank per GPU; every rank runs its own
copy of the layer workload (weak scaling) and the time is the max over ranks;
beside it every N > 1 run measures config 5, the planner's pipeline of the
7B-shape model over the N GPUs (NCCL hand-off, row-sharded lm_head), as
`pipeline` with its tok/s, roofline and a token-parity check on every rank.
`--impl reference` times the reference's own CPU kernel (kernel/q4gemv.c,
built from source into oracle/_ref/) on the host cores for the same metric.
Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GS = 64
HIDDEN, INTER, KV = 3584, 18944, 512
# (name, n_out, n_in) as the stage launches them
LAUNCHES = [("qkv", HIDDEN + 2 * KV, HIDDEN), ("o", HIDDEN, HIDDEN),
            ("gate_up", 2 * INTER, HIDDEN), ("down", HIDDEN, INTER)]
# the seven projections of the layer, each as its own GEMV
PROJECTIONS = [("q", HIDDEN, HIDDEN), ("k", KV, HIDDEN), ("v", KV, HIDDEN), ("o", HIDDEN, HIDDEN),
               ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]
COPIES = 4
METRIC = "q4 GEMV achieved HBM GB/s (Qwen2-7B-shape layer int4 projections, batch 1)"
WORKLOAD = "qwen2-7b-layer-int4-projections-m1"
FALLBACK_HBM_GBS = 6650.0


def alg_bytes(n_out: int, n_in: int, gs: int = GS, m: int = 1) -> int:
    """Algorithmic bytes of one GEMV: packed weights + fp16 scales and biases +
    fp32 x + fp32 out."""
    return n_out * n_in // 2 + n_out * (n_in // gs) * 4 + m * n_in * 4 + m * n_out * 4


STEP_BYTES = sum(alg_bytes(n, k) for _, n, k in LAUNCHES)
LAYER_BYTES = sum(alg_bytes(n, k) for _, n, k in PROJECTIONS)


def config_dict():
    return {"workload": WORKLOAD, "hidden": HIDDEN, "intermediate": INTER, "kv_rows": KV,
            "group_size": GS, "batch_tokens": 1,
            "launches": [f"{n}:{r}x{k}" for n, r, k in LAUNCHES],
            "l2": f"{COPIES} rotating weight copies ({COPIES * LAYER_BYTES / 1e6:.0f} MB) > 126 MB L2"}


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak() -> float:
    """Dense bf16 tensor-core peak in TFLOP/s: the burst cuBLAS figure from
    MEASURED_PEAKS.json, else the fallback measurement on this pool."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        return 1590.0


TRAFFIC_FILE = os.path.join("profiles", "gemv_stream_traffic.txt")


def profiled_traffic():
    """DRAM bytes (read + write) per GEMV launch of the layer step as one ncu
    capture measured them, with where and when that capture was taken:
    (bytes or None, source string)."""
    path = os.path.join(ROOT, TRAFFIC_FILE)
    info = {}
    try:
        for line in open(path):
            if ":" in line:
                k, v = line.split(":", 1)
                info[k.strip()] = v.strip()
    except OSError:
        return None, "no capture"
    try:
        nbytes = float(info["traffic_bytes_per_launch"].split()[0])
    except (KeyError, ValueError):
        return None, "no capture"
    return nbytes, f"ncu capture {TRAFFIC_FILE} ({info.get('captured', 'undated')})"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.02):
        self.samples = []
        self.period = period_s
        self.stop_ev = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self.stop_ev.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.thread.start()
        return self

    def __exit__(self, *a):
        self.stop_ev.set()
        if self.ok:
            self.thread.join(timeout=1.0)

    def summary(self, t0: float, t1: float):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        used = inside or [min(self.samples, key=lambda s: abs(s[0] - (t0 + t1) / 2))] if self.samples else []
        reasons = set()
        for _, _, rs in used:
            for bit, name in self.REASONS.items():
                if rs & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median([s[1] for s in used]) if used else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples_in_timed_region": len(inside)}


# ---------------------------------------------------------------- ours
def run_ours(args, rank: int, world: int, local_rank: int):
    import numpy as np
    import torch
    import torch.distributed as dist

    from hetero_infer_b200 import _lib, cuda_model, synth

    lib = _lib.load()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def q4_on_device(n_out, n_in):
        w = torch.randint(-2 ** 31, 2 ** 31 - 1, (n_out, n_in // 8), dtype=torch.int32, device=dev,
                          generator=gen)
        s = (torch.randn(n_out, n_in // GS, device=dev, generator=gen).abs() * 0.01).half()
        b = (s.float() * -8.0).half()
        return w, s, b

    copies = [{name: q4_on_device(n, k) for name, n, k in LAUNCHES} for _ in range(COPIES)]
    xs = {name: torch.randn(1, k, device=dev, generator=gen) for name, n, k in LAUNCHES}
    outs = {name: torch.empty(1, n, device=dev) for name, n, k in LAUNCHES}
    stream = torch.cuda.Stream(dev)

    def launch(name, n, k, wsb, x, out):
        w, s, b = wsb
        rc = lib.hq4_gemv(w.data_ptr(), s.data_ptr(), b.data_ptr(), x.data_ptr(), out.data_ptr(),
                          n, k, GS, 1, stream.cuda_stream)
        _lib.check(rc, "hq4_gemv")

    def step(c):
        for name, n, k in LAUNCHES:
            launch(name, n, k, copies[c][name], xs[name], outs[name])

    # one graph per weight copy (one step each) and one covering all copies
    graphs = []
    with torch.cuda.stream(stream):
        for c in range(COPIES):
            step(c)
        torch.cuda.synchronize(dev)
        for c in range(COPIES):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(c)
            graphs.append(g)
        g_all = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_all, stream=stream):
            for c in range(COPIES):
                step(c)

    def run_steps(k):
        full, rem = divmod(k, COPIES)
        for _ in range(full):
            g_all.replay()
        for c in range(rem):
            graphs[c].replay()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    with torch.cuda.stream(stream):
        run_steps(args.warmup)
    torch.cuda.synchronize(dev)

    sampler = ClockSampler(local_rank)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with sampler:
        time.sleep(0.05)
        barrier()
        torch.cuda.synchronize(dev)
        t_wall0 = time.perf_counter()
        with torch.cuda.stream(stream):
            e0.record(stream)
            run_steps(args.steps)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        t_wall1 = time.perf_counter()
        barrier()
        time.sleep(0.05)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * args.steps * STEP_BYTES / (ms_max * 1e-3) / 1e9

    pipe = None
    if world > 1:
        pipe = pipeline_suite(rank, world, dev)
    result = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        traffic, traffic_src = profiled_traffic()
        result = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights x fp32 activations (u8*s8->s32 tensor-core dot, fp32 scale/accumulate)",
            "data": "synthetic (seeded random int4 weights, fp32 N(0,1) activations)",
            "config": config_dict(),
            "roofline": {"bound": "hbm", "achieved": round(value / world, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(value / world / peak, 4),
                         "frac_of_8000": round(value / world / 8000.0, 4),
                         "traffic": traffic, "traffic_source": traffic_src,
                         "algorithmic_bytes_per_launch": STEP_BYTES / len(LAUNCHES),
                         "kernel": "gemv_stream_kernel (avg over the step's 4 launches)"},
            "clocks": sampler.summary(t_wall0, t_wall1),
            "gpu_launches": len(LAUNCHES) * args.steps,
        }
        if pipe is not None:
            # config 5 beside the headline: the pipelined decode over the N GPUs
            result["pipeline"] = pipe
            result["pipeline_tok_s"] = pipe["micro8"]["tok_s"]
            result["pipeline_parity"] = pipe["parity"]
        if not args.no_extras:
            result["per_projection"] = per_projection(lib, dev, gen, stream, q4_on_device)
            result["gemv_3584x18944"] = result["per_projection"]["gate"]
            result["gemm_w4a16"] = gemm_bench(lib, dev, gen, stream, q4_on_device)
            result["e2e"] = e2e_qlinear(args, dev, cuda_model, synth, np)
            if world == 1:
                result["decode"] = decode_bench(dev, cpu_seconds=args.cpu_seconds)
            if world == 1:
                result["cpu_baseline"] = cpu_baseline(args, budget_s=args.cpu_seconds)
    if world > 1:
        barrier()
    return result


def per_projection(lib, dev, gen, stream, q4_on_device, launches_per=200):
    """Each of the seven projections alone, back to back, rotating weight
    copies that together exceed L2 (CUDA events around a graph)."""
    import torch
    from hetero_infer_b200 import _lib
    out = {}
    peak, _ = measured_peak()
    for name, n, k in PROJECTIONS:
        nbytes = alg_bytes(n, k)
        reps = max(2, -(-400_000_000 // nbytes))
        ws = [q4_on_device(n, k) for _ in range(reps)]
        x = torch.randn(1, k, device=dev, generator=gen)
        y = torch.empty(1, n, device=dev)
        torch.cuda.synchronize(dev)  # generated on the default stream, timed on `stream`

        def one(i):
            w, s, b = ws[i % reps]
            _lib.check(lib.hq4_gemv(w.data_ptr(), s.data_ptr(), b.data_ptr(), x.data_ptr(),
                                    y.data_ptr(), n, k, GS, 1, stream.cuda_stream), "hq4_gemv")

        with torch.cuda.stream(stream):
            for i in range(reps):
                one(i)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(reps * 2):
                    one(i)
            g.replay()
            torch.cuda.synchronize(dev)
            n_rep = max(1, launches_per // (reps * 2))
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n_rep):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / (n_rep * reps * 2)
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"shape": f"{n}x{k}", "us": round(us, 3), "GB/s": round(gbs, 1),
                     "frac": round(gbs / peak, 4), "frac_of_8000": round(gbs / 8000.0, 4),
                     "bytes": nbytes}
        del ws
    return out


def gemm_bench(lib, dev, gen, stream, q4_on_device, launches=60):
    """Benchmark config 3: gate/up (18944x3584) and down (3584x18944) at
    M = 1, 4, 16, 64, 256 tokens of bf16 activations through hq4_gemm_w4a16
    (the register-path kernel up to 16 tokens, tcgen05/TMEM above), fp32
    out; M = 1 also through the decode GEMV (x as fp32, exact).  Rotating
    weight copies > L2; CUDA events around graph replays.  Roofline: HBM for
    every M (algorithmic bytes = packed weights + scales/biases + x + out),
    and the tensor peak (2 M N K flops) beside it."""
    import torch
    from hetero_infer_b200 import _lib, ops
    hbm_peak, _ = measured_peak()
    tc_peak = measured_tensor_peak()
    out = {}
    for name, n, k in (("gate_up", 18944, 3584), ("down", 3584, 18944)):
        nbytes_w = n * k // 2 + n * (k // 64) * 4
        reps = max(2, -(-400_000_000 // nbytes_w))
        ws = [q4_on_device(n, k) for _ in range(reps)]
        torch.cuda.synchronize(dev)
        for m in (1, 4, 16, 64, 256):
            x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
            xf = x.float()
            y = torch.empty(m, n, device=dev)
            work = ops.gemm_workspace(n, k, m, dev)
            torch.cuda.synchronize(dev)
            plan = ops.gemm_plan(n, k, m)
            variants = [("gemm", plan["kernel"])] + ([("gemv", "gemv_stream")] if m == 1 else [])
            row = {}
            for label, kern in variants:
                def one(i):
                    w, s_, b_ = ws[i % reps]
                    if label == "gemm":
                        _lib.check(lib.hq4_gemm_w4a16(w.data_ptr(), s_.data_ptr(), b_.data_ptr(), x.data_ptr(), 0,
                                                      y.data_ptr(), n, k, GS, m, None, None, work.data_ptr(),
                                                      work.numel(), stream.cuda_stream), "hq4_gemm_w4a16")
                    else:
                        _lib.check(lib.hq4_gemv(w.data_ptr(), s_.data_ptr(), b_.data_ptr(), xf.data_ptr(),
                                                y.data_ptr(), n, k, GS, 1, stream.cuda_stream), "hq4_gemv")
                with torch.cuda.stream(stream):
                    for i in range(reps):
                        one(i)
                    torch.cuda.synchronize(dev)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        for i in range(reps * 2):
                            one(i)
                    g.replay()
                    torch.cuda.synchronize(dev)
                    n_rep = max(1, launches // (reps * 2))
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(n_rep):
                        g.replay()
                    e1.record(stream)
                torch.cuda.synchronize(dev)
                us = e0.elapsed_time(e1) * 1e3 / (n_rep * reps * 2)
                xb = m * k * (2 if label == "gemm" else 4)
                nbytes = nbytes_w + xb + m * n * 4
                gbs = nbytes / (us * 1e-6) / 1e9
                tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
                row[label] = {"kernel": kern, "us": round(us, 3), "GB/s": round(gbs, 1),
                              "hbm_frac": round(gbs / hbm_peak, 4), "TFLOP/s": round(tf, 1),
                              "tensor_frac": round(tf / tc_peak, 4)}
                del g
            out[f"{name}_m{m}"] = row
        del ws
    return out


def decode_bench(dev, n_tokens: int = 128, prompt_len: int = 32, cpu_seconds: float = 0.0):
    """Benchmark config 4: greedy decode of the random-init Qwen2-7B-shape model
    on one device -- 32-token prompt, then one CUDA-graph replay per generated
    token (embedding, 28 layers, head, argmax, position advance).  Decode tok/s
    over the graph-replayed steps (CUDA events); TTFT is the prefill plus first
    token, after one untimed prefill.  With cpu_seconds > 0 the same model's greedy decode on the host
    cores (the reference's NumPy stage procedure over the reference's own
    kernel) is timed beside it as s/token."""
    import numpy as np
    import torch
    from hetero_infer_b200 import cuda_model, synth

    class Spec:
        start, end, embed, head = 0, 28, True, True

    cfg = dict(synth.QWEN2_7B)
    t0 = time.perf_counter()
    w = synth.model_weights(cfg, 0)
    stage = cuda_model.Stage(cfg, Spec, w, device=dev, max_ctx=512)
    t_load = time.perf_counter() - t0
    prompt = synth.prompt_ids(0, prompt_len, cfg["vocab_size"])
    per_token_bytes = 28 * sum(alg_bytes(n, k) for _, n, k in PROJECTIONS) + alg_bytes(cfg["vocab_size"], HIDDEN)

    def run(persistent):
        dec = cuda_model.GreedyDecoder(stage, persistent=persistent)
        torch.cuda.synchronize(dev)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(dec.stream)
        dec.prefill(prompt)
        e1.record(dec.stream)
        dec.capture()
        torch.cuda.synchronize(dev)
        n_steps = n_tokens - 2
        e1b = torch.cuda.Event(enable_timing=True)
        e1b.record(dec.stream)
        dec.steps(n_steps)
        e2.record(dec.stream)
        torch.cuda.synchronize(dev)
        toks = dec.tokens()
        ms = e1b.elapsed_time(e2)
        tok_s = n_steps / (ms * 1e-3)
        out = {"tok_s": round(tok_s, 1), "ms_per_token": round(ms / n_steps, 4),
               "ttft_ms": round(e0.elapsed_time(e1), 2), "generated": len(toks),
               "prompt_tokens": prompt_len, "timed_steps": n_steps,
               "weight_GB_per_s": round(per_token_bytes * tok_s / 1e9, 1),
               "launches_per_token": 5 if dec.plan is not None else 28 * 5 + 4,
               "persistent_layers": dec.plan is not None, "first_tokens": toks[:8]}
        if dec.plan is not None:
            out["plan"] = dec.plan.info()
        dec.graph = None  # the graph holds the plan's launch: release it first
        torch.cuda.synchronize(dev)
        if dec.plan is not None:
            dec.plan.close()
        del dec
        return out, toks

    # one untimed prefill first: the first launches of each kernel and the
    # first tensor maps of each weight are one-time set-up, not time to first token
    warm = cuda_model.GreedyDecoder(stage)
    warm.prefill(prompt)
    torch.cuda.synchronize(dev)
    del warm
    res, toks = run(False)
    res_pers, toks_pers = run(True)
    # the host-core baseline runs after the device timings: the reference
    # kernel's worker threads must not compete with the host thread that
    # issues the prefill's launches
    cpu = cpu_decode_baseline(cfg, w, cpu_seconds) if cpu_seconds > 0 else None
    del w
    peak, peak_kind = measured_peak()
    achieved = per_token_bytes * res["tok_s"] / 1e9
    res.update({"hbm_ceiling_tok_s": round(peak * 1e9 / per_token_bytes, 1),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                             "unit": "GB/s", "frac": round(achieved / peak, 4),
                             "bytes_per_token": per_token_bytes,
                             "what": "weight bytes streamed per token (28 layers' projections + lm_head, "
                                     "algorithmic) x tok/s"},
                "persistent_plan": res_pers, "tokens_equal_persistent_path": toks == toks_pers,
                "model": "qwen2-7b-shape random int4 (28 layers, h3584, 28q/4kv, i18944, v152064)",
                "setup_s": round(t_load, 1)})
    if cpu is not None:
        res["cpu_baseline"] = cpu
    return res


def cpu_decode_baseline(cfg, w, budget_s: float, prompt_len: int = 4):
    """Config 4 on the host cores: greedy decode of the same 7B-shape model
    through the reference's NumPy stage procedure (oracle/stage.py, pinned bit
    for bit to hetero/cpu_model.py:309-368) whose GEMVs call the reference's
    own kernel built from source (kernel/q4gemv.c, AVX2 build, all cores),
    as QLinear._gemv calls it (cpu_model.py:109-117).  A short prompt (rows
    <= 16 take the GEMV path) then decode steps until the budget runs out;
    s/token over the decode steps."""
    import numpy as np
    from hetero_infer_b200 import synth
    from oracle import stage as ost
    cores = cpu_cores()
    os.environ["HETERO_KERNEL_THREADS"] = str(min(cores, 16))
    kern, kind, what = cpu_kernel()
    if kern is None:
        from oracle.q4 import Oracle
        orc = Oracle()
    else:
        class _RefOrc:  # the reference kernel behind the oracle stage's product calls
            def gemv_f32(self, w_, s_, b_, x, gs):
                return kern.gemv(w_, s_, b_, x, gs, nthreads=cores)

            def dequant(self, w_, s_, b_, r0, r1, gs):
                return kern.dequant(w_, s_, b_, r0, r1, gs, nthreads=cores)
        orc = _RefOrc()
    L, H = cfg["num_hidden_layers"], cfg["hidden_size"]
    st = ost.OracleStage(cfg, w, 0, L, True, True, embed_rows=lambda ids: synth.embed_rows(0, ids, H), orc=orc)
    caches = st.new_caches()
    prompt = synth.prompt_ids(0, prompt_len, cfg["vocab_size"])
    z = st(prompt, caches, apply_head=True, last_only=True)
    tok = int(z[0, -1].argmax())
    steps = 0
    t0 = time.perf_counter()
    while True:
        z = st(np.array([[tok]]), caches, apply_head=True, last_only=True)
        tok = int(z[0, -1].argmax())
        steps += 1
        if time.perf_counter() - t0 > budget_s or steps >= 64:
            break
    dt = time.perf_counter() - t0
    return {"value": round(dt / steps, 4), "unit": "s/token", "tok_s": round(steps / dt, 2), "cores": cores,
            "kind": "port" if kern is None else "reference",
            "sample": f"{steps} greedy decode steps of the 7B-shape model after a {prompt_len}-token prompt "
                      f"({dt:.1f} s); NumPy stage procedure of hetero/cpu_model.py (oracle/stage.py) with "
                      f"HETERO_KERNEL_THREADS={min(cores, 16)}; GEMV: {what}"}


def pipeline_suite(rank: int, world: int, dev, n_tokens: int = 256, prompt_len: int = 32):
    """Benchmark config 5: the 7B-shape random model split by the planner over
    the `world` GPUs, hidden states handed on by NCCL send/recv, the lm_head
    row-sharded over all ranks (on a side stream), 4 and 8 independent
    streams in flight, `n_tokens` per stream; the reference's fp16 wire (4 and
    8 streams) and its int8 codec (8 streams).  Every decode tick is a CUDA-
    graph replay per rank (send/recv and the stage's layers) plus one per
    finished stream's head.  Aggregate decode tok/s: wall clock between two
    device synchronisations around the decode, max over ranks.

    Roofline: every generated token streams the whole model's weights once
    (split over the stages), so achieved = tok/s x weight bytes per token,
    against world x the measured HBM peak.

    Parity (checked on every rank, all-reduced): the fp32 wire carries the
    hidden state unchanged, so the pipelined model computes the unsplit one;
    stream 0 is fed the prompt of the reference's own 7B decode and its 128
    tokens must equal the ones the reference's NumPy backend generated
    (tests/golden/golden_7b.json).  The fp16 wire's tokens follow the
    reference's pipeline, which overflows fp16 on this model."""
    import json as _json
    import torch
    import torch.distributed as dist
    from hetero_infer_b200 import pipeline, planner, synth
    cfg = dict(synth.QWEN2_7B)
    plan = planner.plan_gpu_pipeline(cfg, world, layer_s=60e-6, head_s=52e-6)
    spec = plan.specs[rank]
    w = synth.model_weights(cfg, 0, layers=range(spec.start, spec.end), embed=spec.embed, head=True)
    per_token_bytes = 28 * sum(alg_bytes(n, k) for _, n, k in PROJECTIONS) + alg_bytes(cfg["vocab_size"], HIDDEN)
    peak, peak_kind = measured_peak()
    rows = pipeline.head_rows(cfg["vocab_size"], world, rank)

    def run(comp, prompts, n_tok):
        comp.release_graphs()
        pr = pipeline.PipelineRank(pipeline.Comm(rank, world, dev), comp, len(prompts))
        pr.prefill(prompts)
        dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        pr.decode(n_tok - 1)
        torch.cuda.synchronize(dev)
        dt = time.perf_counter() - t0
        pr.close()  # its graphs hold NCCL calls: released before the process group goes
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return pr, float(t.item())

    out = {"cuts": plan.cuts, "head": "row-sharded over all ranks", "tokens_per_stream": n_tokens,
           "timing": "host wall clock around the decode loop, device synchronised on both sides (sampled "
                     "tokens stay on the device), max over ranks"}
    for wire, micros in (("float16", (4, 8)), ("int8", (8,))):
        comp = pipeline.DeviceCompute(cfg, spec, w, rows, dev, max_ctx=512, wire=wire)
        for m in micros:
            prompts = [synth.prompt_ids(1000 + i, prompt_len, cfg["vocab_size"]) for i in range(m)]
            pr, dt = run(comp, prompts, n_tokens)
            gen = m * (n_tokens - 1)
            tok_s = gen / dt
            achieved = tok_s * per_token_bytes / 1e9
            key = f"micro{m}" + ("" if wire == "float16" else "_int8_wire")
            out[key] = {"streams": m, "decode_tokens": gen, "tok_s": round(tok_s, 1), "seconds": round(dt, 3),
                        "ticks": pr.ticks, "ms_per_tick": round(dt * 1e3 / pr.ticks, 4),
                        "wire": "fp16 (reference format)" if wire == "float16" else
                                "int8 codec (reference transport codec, on device)",
                        "first_tokens": pr.tokens[0][:6],
                        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(world * peak, 1),
                                     "peak_kind": f"{world} x {peak_kind}", "unit": "GB/s",
                                     "frac": round(achieved / (world * peak), 4)}}
        del comp
        torch.cuda.empty_cache()
    gold = _json.load(open(os.path.join(ROOT, "tests", "golden", "golden_7b.json")))
    comp = pipeline.DeviceCompute(cfg, spec, w, rows, dev, max_ctx=512, wire="float32")
    del w
    gp = synth.prompt_ids(gold["seed"], gold["prompt_tokens"], cfg["vocab_size"])
    others = [synth.prompt_ids(2000 + i, prompt_len, cfg["vocab_size"]) for i in range(3)]
    pr, dt = run(comp, [gp] + others, gold["generated"])
    ref = [st["token"] for st in gold["variants"]["float"]["steps"]]
    ok = torch.tensor([1 if pr.tokens[0] == ref else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    out["parity"] = bool(ok.item())
    out["parity_check"] = (f"fp32-wire pipeline, stream 0 of 4: {gold['generated']} greedy tokens vs the reference "
                           f"NumPy backend's unsplit decode (tests/golden/golden_7b.json), every rank")
    del comp
    torch.cuda.empty_cache()
    return out


def e2e_qlinear(args, dev, cuda_model, synth, np):
    """The same metric through the reference-facing API: the reference's
    QLinear calling convention (hetero/cpu_model.py:145-158) with NumPy
    activations on the host -- every call copies x host->device, runs the
    GEMV, and copies the result back."""
    import torch
    layers = []
    for c in range(2):
        layers.append([cuda_model.QLinear(*synth.q4_linear(c, f"e2e.{name}", n, k, GS), None, GS, 4,
                                          device=dev) for name, n, k in PROJECTIONS])
    xs = [synth.activation(7, f"e2e.x.{name}", (1, k)) for name, n, k in PROJECTIONS]
    h2d = sum(x.nbytes for x in xs)
    d2h = sum(4 * n for _, n, _ in PROJECTIONS)
    steps = max(20, min(args.steps, 300))
    for i in range(5):
        for q, x in zip(layers[i % 2], xs):
            q(x)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(steps):
        for q, x in zip(layers[i % 2], xs):
            q(x)
    torch.cuda.synchronize(dev)
    dt = time.perf_counter() - t0
    return {"value": round(steps * LAYER_BYTES / dt / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "hetero_infer_b200.cuda_model.QLinear.__call__(numpy) x 7 projections",
            "steps": steps, "ms_per_step": dt * 1e3 / steps}


# ---------------------------------------------------------------- CPU arms
def _cpu_layer(seed_base: int, copies: int):
    from hetero_infer_b200 import synth
    return [[synth.q4_linear(seed_base + c, f"cpu.{name}", n, k, GS) for name, n, k in PROJECTIONS]
            for c in range(copies)]


def cpu_kernel():
    """The reference's kernel built from source (oracle/_ref), else our port."""
    from oracle import q4
    if "avx2" in q4.available_ref_variants():
        return q4.RefKernel("avx2"), "reference", "kernel/q4gemv.c -O3 -mavx2 -mfma -mf16c (oracle/_ref)"
    return None, "port", "oracle/q4_oracle.c float path (reference build unavailable)"


def time_cpu_layer(steps: int, threads: int, copies: int = 4, budget_s: float = None):
    """Time `steps` layer steps (7 projections each, as the reference QLinear
    calls q4_gemv) on `threads` host threads; returns (seconds, steps done)."""
    import numpy as np
    os.environ["HETERO_KERNEL_THREADS"] = str(min(threads, 16))
    kern, kind, what = cpu_kernel()
    layers = _cpu_layer(99, copies)
    xs = [np.random.default_rng(5).standard_normal(k).astype(np.float32) for _, n, k in PROJECTIONS]
    if kern is None:
        from oracle.q4 import Oracle
        orc = Oracle()
        call = lambda wsb, x: orc.gemv_f32(*wsb, x, GS)
    else:
        call = lambda wsb, x: kern.gemv(*wsb, x, GS, nthreads=threads)
    for wsb, x in zip(layers[0], xs):
        call(wsb, x)
    done = 0
    t0 = time.perf_counter()
    while done < steps:
        for wsb, x in zip(layers[done % copies], xs):
            call(wsb, x)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    return time.perf_counter() - t0, done, kind, what


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(args, budget_s: float = 10.0):
    cores = cpu_cores()
    dt, done, kind, what = time_cpu_layer(10 ** 9, cores, budget_s=budget_s)
    value = done * LAYER_BYTES / dt / 1e9
    return {"value": round(value, 2), "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{done} layer steps (7 q4_gemv calls each, 4 rotating weight copies, "
                      f"{dt:.1f} s) with HETERO_KERNEL_THREADS={min(cores, 16)}; {what}"}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return None
    cores = cpu_cores()
    # warm-up steps, then at most ~60 s of timed steps
    time_cpu_layer(args.warmup, cores, budget_s=15.0)
    dt, done, kind, what = time_cpu_layer(args.steps, cores, budget_s=60.0)
    value = done * LAYER_BYTES / dt / 1e9
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": done, "warmup": args.warmup, "ms_per_step": dt * 1e3 / max(done, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4 weights x fp32 activations (reference AVX2 path: int16 x, int32 dot)",
        "data": "synthetic (seeded random int4 weights, fp32 N(0,1) activations)",
        "config": config_dict(),
        "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": f"{done} of {args.steps} requested layer steps in {dt:.1f} s "
                                   f"(7 q4_gemv calls each, capped at 60 s); {what}"},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def profile_case(which: str) -> None:
    """A short, fixed run of one kernel family for an ncu capture (a profiler
    replays each captured launch many times, so these cases hold a few GB at
    most and launch little before the captured kernels):

      layer   the four GEMV launches of a Qwen2-7B-shape layer at batch 1
              (q|k|v 4608x3584, o 3584x3584, gate|up 37888x3584, down
              3584x18944), three rounds over two weight copies;
      gemm    hq4_gemm_w4a16 on 18944x3584 at 4 tokens (multi-token
              streaming kernel), 16 tokens (register-path kernel) and 256
              tokens (tcgen05 kernel), bf16 activations, three calls each;
      gemm_down  the same on the down shape, 3584x18944;
      decode  the 7B-shape stage's decode step, per-layer launches, 4 steps
              after a 4-token prompt.

    Weights are seeded random int4 with the benchmark's scale/bias law."""
    import torch
    from hetero_infer_b200 import _lib, ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream

    def q4(n, k):
        w = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=g)
        s_ = (torch.randn(n, k // GS, device=dev, generator=g).abs() * 0.01).half()
        return w, s_, (s_.float() * -8).half()

    if which == "layer":
        mats = [[(q4(n, k), torch.randn(1, k, device=dev, generator=g), torch.empty(1, n, device=dev), n, k)
                 for _, n, k in LAUNCHES] for _ in range(2)]
        for r in range(3):
            for (w, s_, b), x, y, n, k in mats[r % 2]:
                _lib.check(lib.hq4_gemv(w.data_ptr(), s_.data_ptr(), b.data_ptr(), x.data_ptr(), y.data_ptr(),
                                        n, k, GS, 1, st), "hq4_gemv")
    elif which in ("gemm", "gemm_down"):
        n, k = (18944, 3584) if which == "gemm" else (3584, 18944)
        w, s_, b = q4(n, k)
        for m in (4, 16, 256):
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            for _ in range(3):
                ops.q4_gemm(w, s_, b, x, GS)
    elif which == "decode":
        from hetero_infer_b200 import cuda_model, synth

        class Spec:
            start, end, embed, head = 0, 28, True, True
        cfg = dict(synth.QWEN2_7B)
        stage = cuda_model.Stage(cfg, Spec, synth.model_weights(cfg, 0), device=dev, max_ctx=64)
        dec = cuda_model.GreedyDecoder(stage)
        dec.generate(synth.prompt_ids(0, 4, cfg["vocab_size"]), 6)
    else:
        raise SystemExit(f"unknown case {which}")
    torch.cuda.synchronize()
    print(json.dumps({"case": which, "status": lib.hq4_device_status(0)}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip per-projection, e2e and CPU-baseline legs")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--pipeline-only", type=int, default=0, metavar="TOKENS",
                    help="N>1: only run the config-5 pipeline (TOKENS per stream, 4 and 8 streams)")
    ap.add_argument("--decode-only", type=int, default=0, metavar="TOKENS",
                    help="only run the config-4 decode (TOKENS generated) and print its JSON")
    ap.add_argument("--case", choices=["layer", "gemm", "gemm_down", "decode"], default=None,
                    help="run one short fixed case for a profiler capture and exit")
    args = ap.parse_args()
    if args.case:
        profile_case(args.case)
        return
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)

    if args.decode_only:
        import torch
        torch.cuda.set_device(local_rank)
        print(json.dumps(decode_bench(torch.device("cuda", local_rank), n_tokens=max(3, args.decode_only))),
              flush=True)
        return
    if args.pipeline_only and world > 1 and args.impl == "ours":
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dev = torch.device("cuda", local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        out = pipeline_suite(rank, world, dev, n_tokens=max(3, args.pipeline_only))
        if rank == 0:
            print(json.dumps({"pipeline": out, "n_gpus": world}), flush=True)
        dist.destroy_process_group()
        return
    if args.impl == "reference":
        res = run_reference(args, rank, world)
    else:
        if world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        res = run_ours(args, rank, world, local_rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if res is not None and rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
