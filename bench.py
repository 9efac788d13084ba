"""Benchmark of the B200 MoE expert hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Default workload (the configuration its
"MoE-layer tokens/s at 1/2/4/8 B200" metric is quoted on): a GPT-OSS-120B-
shaped MoE decode stack — 36 layers, 128 experts, top-4, H = F = 2880 —
on a batch of 64 tokens with bf16 hidden states ~N(0, 1) and the full
~57 GiB random-init MXFP4 bank resident in HBM.  One step = the 64 tokens
through all 36 MoE layers with residual chaining (identity norm):
router + top-k -> gate_up GEMV + clamped SwiGLU -> down GEMV -> weighted
combine -> residual.  At N > 1 the experts are sharded by index
(e % N) and the per-layer partial sums meet in one NCCL all-reduce
(strong scaling: the 64-token batch is fixed).

Other workloads (parity/inspection, not the headline): gemv (config 0,
batched over copies > 4x L2), oss20-decode1 (config 1), oss120-decode1
(config 2, batch 1), qwen3-decode1 / qwen3-decode32 (config 3),
oss120-prefill (config 4: one GPT-OSS-120B layer, 2048 tokens, 4x skew on 8
hot experts; its experts run on the tensor cores, so its roofline line is
the grouped GEMM's TFLOP/s, with its HBM figures beside it).

`value` is device-timed with inputs resident in HBM; `e2e` times the same
step through the public C-ABI with the hidden states copied from pinned host
memory and the output stream copied back inside the timed region.
`--impl reference` times the reference's CPU path (the oracle port of the
Swift code: the Swift/Metal reference cannot run here) on all host cores.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (preset, T, description)
    "oss120-decode64": ("gpt-oss-120b", 64, "GPT-OSS-120B-shaped MoE decode, 36 layers, batch 64"),
    "oss120-decode1": ("gpt-oss-120b", 1, "GPT-OSS-120B-shaped MoE decode, 36 layers, batch 1"),
    "oss20-decode1": ("gpt-oss-20b", 1, "GPT-OSS-20B-shaped MoE decode, 24 layers, batch 1"),
    "qwen3-decode1": ("qwen3-30b-a3b", 1, "Qwen3-30B-A3B-shaped MoE decode, 48 layers, batch 1"),
    "qwen3-decode32": ("qwen3-30b-a3b", 32, "Qwen3-30B-A3B-shaped MoE decode, 48 layers, batch 32"),
    "oss120-prefill": ("gpt-oss-120b", 2048, "GPT-OSS-120B-shaped MoE prefill layer, 2048 tokens, 4x hot-expert skew on 8 experts"),
    "gemv": (None, 1, "MXFP4 GEMV 2880x2880 (GPT-OSS down_proj shape), batched over copies"),
    "int8-head": (None, 1, "int8 affine GEMV 201088x2880 (GPT-OSS output head), one token"),
}
DEFAULT_WORKLOAD = "oss120-decode64"
# timed steps when --steps is not given: about a second of work each
DEFAULT_STEPS = {"oss120-decode64": 60, "oss120-decode1": 600, "oss20-decode1": 1000,
                 "qwen3-decode1": 600, "qwen3-decode32": 200, "oss120-prefill": 150, "gemv": 2000,
                 "int8-head": 400}
SEED = 0


def peaks(kind: str = "hbm"):
    """Roofline denominator: measured HBM copy GB/s, or dense bf16 TFLOP/s
    (burst: the kernels are timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    key, fallback = ("hbm_gbs", 6650.0) if kind == "hbm" else ("bf16_tflops", 1590.0)
    if os.path.exists(p):
        d = json.load(open(p))
        if key in d:
            return d[key], "measured"
    return fallback, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()  # the first sample, so the timed region is covered from its start
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 10.0:
                time.sleep(0.01)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU reference leg (the oracle port of the reference's Swift CPU path)

class CpuReference:
    """The oracle MoE layer (C restatement of the reference's CPU path) on the
    host cores, for a bounded token sample of layer 0.  The weights are made
    on the host by the same counter hash as the device bank's, so the sample
    computes the workload's own layer."""

    def __init__(self, spec, threads: int, max_tokens: int = 2048, router_bias=None):
        import numpy as np

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        from godwit_b200 import synth

        self.O, self.spec, self.threads = O, spec, threads
        rng = np.random.default_rng(SEED)
        self.x = synth.as_f32(synth.make_hidden(rng, max_tokens, spec.hidden, "bf16"), "bf16")
        self.rw, rb = synth.hash_router(spec, SEED, 0)
        if router_bias is not None:  # the prefill workload's skewed router
            rb = router_bias
        self.rb = rb if (spec.router_bias or router_bias is not None) else None
        self.strides = np.zeros((spec.experts, spec.layout().stride), np.uint8)
        self.ready = set()
        self.n = max(1, min(threads, max_tokens))

    def _need(self, n):
        from godwit_b200 import synth
        for t in range(n):
            e, _ = self.O.router_select(self.O.router_logits(self.rw, self.rb, self.x[t]),
                                        self.spec.top_k)
            for v in e:
                if int(v) not in self.ready:
                    self.strides[int(v)] = synth.hash_expert_stride(self.spec, SEED, 0, int(v))
                    self.ready.add(int(v))

    def calibrate(self, budget_s: float):
        """Grows the token count until one run takes about budget_s."""
        while True:
            self._need(self.n)
            dt = self.run()
            if dt * 2.0 > budget_s or self.n >= self.x.shape[0]:
                return
            self.n = min(self.x.shape[0], int(self.n * max(2.0, min(8.0, budget_s / max(dt, 1e-3) / 2))))

    def run(self) -> float:
        t0 = time.perf_counter()
        self.O.moe_layer(self.spec, self.strides, self.rw, self.rb, self.x[:self.n],
                         threads=self.threads)
        return time.perf_counter() - t0

    def value(self, dt: float) -> float:
        """Tokens/s through the whole stack (layer-tokens/s divided by the depth)."""
        return self.n / dt / self.spec.layers

    def sample(self, dt: float) -> str:
        return (f"{self.n} tokens x layer 0 (of {self.spec.layers}) of the workload's bank, "
                f"scaled to the stack; {dt:.2f} s on {self.threads} threads")


def profiled_traffic(workload: str):
    """`profiles/traffic.json`'s entry for the workload (DRAM bytes per launch
    of its dominant kernel, read off an ncu capture), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f).get(workload)
    except (OSError, ValueError):
        return None


def cpu_reference_sample(spec, threads: int, budget_s: float = 12.0):
    ref = CpuReference(spec, threads)
    ref.calibrate(budget_s)
    dt = ref.run()
    return ref.value(dt), ref.sample(dt)


def cpu_gemv_sample(threads: int, budget_s: float = 10.0):
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from godwit_b200 import synth

    rng = np.random.default_rng(SEED)
    p, s = synth.random_mxfp4(rng, 2880, 2880)
    x = synth.as_f32(synth.make_hidden(rng, 1, 2880, "bf16")[0], "bf16")
    b = synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(rng.normal(0, 0.02, 2880)))
    reps, dt = 1, 0.0
    while True:
        t0 = time.perf_counter()
        for _ in range(reps):
            O.gemv(p, s, x, b, threads=threads)
        dt = time.perf_counter() - t0
        if dt * 2.5 > budget_s or reps > 4096:
            break
        reps *= 2
    gbs = reps * 4_429_440 / dt / 1e9
    return gbs, f"{reps} GEMVs of 2880x2880, {dt:.2f} s on {threads} threads"


# ---------------------------------------------------------------------------

def run_reference(args, workload):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    preset, T, desc = WORKLOADS[workload]
    from godwit_b200.layout import PRESETS
    vals = []
    skew = None
    if preset is None:
        ref = None
    elif workload == "oss120-prefill":
        # the same skewed router as the GPU arm's prefill layer (config 4)
        import numpy as np
        from godwit_b200 import synth
        spec = PRESETS[preset].with_(layers=1)
        x0 = synth.make_hidden(np.random.default_rng(SEED), T, spec.hidden, "bf16")
        rb, delta, h = skewed_router_bias(spec, synth.as_f32(x0, "bf16"))
        skew = skew_record(delta, h)
        ref = CpuReference(spec, threads, router_bias=rb)
    else:
        ref = CpuReference(PRESETS[preset], threads)
    if ref is not None:
        ref.calibrate(4.0)
    for i in range(args.warmup + args.steps):
        if workload == "int8-head":
            v, sample = cpu_int8_sample(threads, budget_s=4.0)
        elif ref is None:
            v, sample = cpu_gemv_sample(threads, budget_s=4.0)
        else:
            dt = ref.run()
            v, sample = ref.value(dt), ref.sample(dt)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    metric, unit = metric_unit(workload)
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": workload_config(workload, args.gpus, args.ep, None, skew),
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "Swift/Metal reference cannot run off Apple hardware; this is the C "
                    "restatement of its CPU path (oracle/mxfp4_oracle.c) on all host cores"}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(workload, world: int = 1, ep: str = "alltoall", layers: int | None = None,
                    skew: dict | None = None) -> dict:
    """The `config` object of a workload: the same in both arms of the
    benchmark (facts of one run, such as fill times, go under "run")."""
    preset, T, desc = WORKLOADS[workload]
    if workload == "gemv":
        return {"workload": "gemv", "rows": 2880, "cols": 2880, "copies": GEMV_COPIES,
                "l2": f"{GEMV_COPIES} distinct copies = {GEMV_COPIES * GEMV_ALG / 1e9:.2f} GB > 4x L2 per launch"}
    if workload == "int8-head":
        alg = HEAD_ROWS * HEAD_COLS + HEAD_ROWS * (HEAD_COLS // 64) * 4 + HEAD_COLS * 2 + HEAD_ROWS * 4
        return {"workload": "int8-head", "rows": HEAD_ROWS, "cols": HEAD_COLS, "tokens": 1,
                "l2": f"{alg / 1e9:.2f} GB of weights per launch > L2"}
    from godwit_b200.layout import PRESETS
    spec = PRESETS[preset]
    if workload == "oss120-prefill":
        spec = spec.with_(layers=1)
    if layers:
        spec = spec.with_(layers=layers)
    per = -(-T // world)
    sliced = world > 1 and ep == "alltoall"
    cfg = {"workload": workload,
           "description": desc if not layers else f"{desc} (profiling run: {spec.layers} layers)",
           "model_shape": spec.name, "layers": spec.layers, "experts": spec.experts, "top_k": spec.top_k,
           "hidden": spec.hidden, "intermediate": spec.intermediate, "tokens": T,
           "parallelism": (f"ep{world} ({'all-to-all, tokens sliced ' + str(per) + ' per rank' if sliced else 'replicated tokens, all-reduce per layer'})"
                           if world > 1 else "single"),
           "l2": "weights streamed per step >> 126 MB L2 (no flush needed)"}
    if skew:
        cfg["skew"] = skew
    return cfg


def metric_unit(workload):
    if workload == "gemv":
        return "MXFP4 expert GEMV HBM GB/s", "GB/s"
    if workload == "int8-head":
        return "int8 affine head GEMV HBM GB/s", "GB/s"
    kind = "prefill" if "prefill" in workload else "decode"
    return f"MoE {kind} tokens/s (" + WORKLOADS[workload][2] + ")", "tokens/s"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: about a second of work — 60 for decode, 150 for "
                         "the prefill layer, 200 for the GEMV, 3 for --impl reference)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-f16", action="store_true",
                    help="oss120-prefill: exact f16 activations instead of config 4's MXFP8 block-scaled MMAs")
    ap.add_argument("--ep", default="alltoall", choices=["alltoall", "replicated"],
                    help="expert parallelism at N > 1: token-sliced all-to-all (default) or replicated tokens")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: hold and run this many layers instead of the model's")
    args = ap.parse_args()
    if args.steps is None:  # about a second of timed work, so the clock sampler sees it
        args.steps = 3 if args.impl == "reference" else DEFAULT_STEPS.get(args.workload, 60)
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args, args.workload)
    if args.workload == "int8-head":
        return run_int8_head(args)
    if args.workload == "gemv":
        return run_gemv(args)
    return run_decode(args)


def _dist_setup(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# Config 4's hot experts: a contiguous block of ids, which the expert
# parallelism's round-robin placement (rank e % N) spreads over the ranks at
# N = 2, 4 and 8.
HOT_EXPERTS = (8, 9, 10, 11, 12, 13, 14, 15)


def skew_record(delta, h) -> dict:
    import numpy as np
    return {"hot_experts": list(HOT_EXPERTS), "delta": round(float(delta), 5),
            "hot_mean_tokens": float(h[list(HOT_EXPERTS)].mean()),
            "other_mean_tokens": float(np.delete(h, list(HOT_EXPERTS)).mean())}


def skewed_router_bias(spec, x_f32, seed=SEED, target=4.0):
    """Config 4's deliberate skew: the router of layer 0 gets a bias offset
    delta on 8 fixed experts, found by bisection on these tokens so that the
    hot experts receive on average `target` x the mean tokens per expert.
    Returns (bias bf16 [E], delta, histogram)."""
    import numpy as np
    from godwit_b200 import synth
    w, b = synth.hash_router(spec, seed, 0)
    logits0 = x_f32 @ synth.bf16_bits_to_f32(w).reshape(spec.experts, spec.hidden).T
    base = synth.bf16_bits_to_f32(b)
    mean = x_f32.shape[0] * spec.top_k / spec.experts

    def hist(delta):
        bb = base.copy()
        bb[list(HOT_EXPERTS)] += delta
        bb = synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(bb))
        top = np.argsort(-(logits0 + bb), axis=1)[:, :spec.top_k]
        return np.bincount(top.ravel(), minlength=spec.experts), bb

    lo, hi = 0.0, 1.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        h, _ = hist(mid)
        if h[list(HOT_EXPERTS)].mean() < target * mean:
            lo = mid
        else:
            hi = mid
    h, bb = hist(hi)
    return synth.f32_to_bf16_bits(bb), hi, h


def run_decode(args):
    import torch

    from godwit_b200 import device as D
    from godwit_b200.ep import AllToAllEP, CudaOps, ReplicatedTokensEP
    from godwit_b200.layout import PRESETS
    from godwit_b200.runtime import Context, ExpertBank
    from godwit_b200 import synth
    import numpy as np

    world, rank, local = _dist_setup(args)
    preset, T, desc = WORKLOADS[args.workload]
    spec = PRESETS[preset]
    prefill = args.workload == "oss120-prefill"
    if prefill:
        spec = spec.with_(layers=1)
    if args.layers:
        spec = spec.with_(layers=args.layers)
    ctx = Context(local)
    block_scaled = prefill and not getattr(args, "prefill_f16", False)
    if block_scaled:
        ctx.set_block_scaled(True)  # config 4: MXFP4 x MXFP8 tcgen05 block-scaled MMAs
    cur = D.bind_stream(ctx)
    bank = ExpertBank(ctx, spec, shard_rank=rank, shard_count=world)
    t0 = time.time()
    bank.fill_synthetic(SEED)
    fill_s = time.time() - t0
    H = spec.hidden
    rng = np.random.default_rng(SEED)
    xb = synth.make_hidden(rng, T, H, "bf16")
    skew = None
    if args.workload == "oss120-prefill":
        rb, delta, h = skewed_router_bias(spec, synth.as_f32(xb, "bf16"))
        rw, _ = synth.hash_router(spec, SEED, 0)
        bank.upload_router(0, rw, rb)
        skew = skew_record(delta, h)
    # At N > 1 each rank holds a slice of the batch (token-sliced expert
    # parallelism, AllToAllEP: the experts of slot rows are applied by their
    # owner after an all-to-all, outputs return by a second one); with
    # --ep replicated every rank holds all T tokens and the partial sums meet
    # in an all-reduce per layer.
    sliced = world > 1 and args.ep == "alltoall"
    per = -(-T // world)
    t0, t1 = (min(T, rank * per), min(T, (rank + 1) * per)) if sliced else (0, T)
    Tr = t1 - t0
    x_host = torch.from_numpy(np.ascontiguousarray(xb[t0:t1]).view(np.int16)).view(torch.bfloat16).pin_memory()
    out_host = torch.empty(Tr, H, dtype=torch.float32).pin_memory()
    x = x_host.to("cuda")
    stream_buf = torch.empty(Tr, H, dtype=torch.float32, device="cuda")
    partial = torch.empty_like(stream_buf)
    x_work = torch.empty_like(x)
    if sliced:
        ep = AllToAllEP(CudaOps(ctx, bank), spec.layers, spec.top_k,
                        capacity_factor=2.0 if prefill else None)
    else:
        ep = ReplicatedTokensEP(CudaOps(ctx, bank), spec.layers)

    def step_eager():
        if world == 1:
            D.moe_stack(ctx, bank, x, stream_buf)
        else:
            if sliced:
                ep.forward(x, stream_buf, x_work, check=False)
            else:
                ep.forward(x, stream_buf, partial, x_work)

    for _ in range(args.warmup):
        step_eager()
    torch.cuda.synchronize()
    # library kernels one step launches (counted on an eager step: a replayed
    # graph does not pass through the library's launch counter)
    l0 = ctx.launch_count()
    step_eager()
    torch.cuda.synchronize()
    launches_per_step = ctx.launch_count() - l0
    # At N > 1 one step (the library's kernels, the exchange's torch ops and
    # the NCCL collectives of all layers) is captured once as a CUDA graph and
    # replayed; one GPU's stack forward already replays its own graph.
    graph, graph_note = None, None
    if world > 1:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cur):
                step_eager()
            graph = g
            graph.replay()
            torch.cuda.synchronize()
        except Exception as e:  # keep measuring, eagerly, and say why
            graph, graph_note = None, f"graph capture failed, eager steps: {type(e).__name__}: {e}"[:300]
            torch.cuda.synchronize()

    def step():
        if graph is not None:
            graph.replay()
        else:
            step_eager()

    def step_e2e():
        x.copy_(x_host, non_blocking=True)
        step()
        out_host.copy_(stream_buf, non_blocking=True)

    for _ in range(2):
        step()
    torch.cuda.synchronize()

    # ---- timed region (device) ----
    sampler = ClockSampler(local)
    sampler.start()
    _barrier(world)
    torch.cuda.synchronize()
    launches0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(cur)
    for _ in range(args.steps):
        step()
    ev1.record(cur)
    torch.cuda.synchronize()
    _barrier(world)
    launches = ctx.launch_count() - launches0 if graph is None else launches_per_step * args.steps
    ms = _max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)

    # ---- e2e through the public API with host buffers ----
    for _ in range(2):
        step_e2e()
    torch.cuda.synchronize()
    _barrier(world)
    ev0.record(cur)
    for _ in range(args.steps):
        step_e2e()
    ev1.record(cur)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    e2e_ms = _max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)

    # ---- kernel timing of the dominant kernels (expert GEMVs) ----
    if sliced:
        ep.raise_if_overflowed()
    ctx.profile_enable(True)
    prof_steps = min(args.steps, 3)
    for _ in range(prof_steps):
        step_eager()
    prof = ctx.profile_read()
    ctx.profile_enable(False)
    expert_ms = prof["gateup_ms"] + prof["down_ms"]
    launches_prof = prof["gateup_launches"] + prof["down_launches"]
    per_pass = spec.expert_weight_bytes + spec.expert_bias_bytes
    alg_bytes = prof["expert_passes"] * per_pass  # + activations (small)
    achieved = alg_bytes / (expert_ms / 1e3) / 1e9 if expert_ms > 0 else None
    peak, peak_kind = peaks()
    step_bytes_total = _max_over_ranks(alg_bytes / prof_steps, 1)
    # prefill runs its experts on the tensor cores (k_grouped): FLOPs of the
    # slots this rank computed, 2 * (2F*H + H*F) each
    slots = T * spec.top_k / world
    flops = 2.0 * slots * (2 * spec.intermediate * spec.hidden + spec.hidden * spec.intermediate)
    tpeak, tpeak_kind = peaks("tensor")
    if block_scaled:  # no measured MXF8F6F4 peak: NVIDIA's dense FP8 figure
        tpeak, tpeak_kind = 4500.0, "nominal dense fp8/mxf8f6f4 (no measured figure)"
    if prefill:
        roofline = {"bound": "tensor", "kernel": "k_grouped (tcgen05 " +
                    ("kind::mxf8f6f4.block_scale" if block_scaled else "kind::f16") +
                    " grouped expert GEMM, gate_up + down)", "achieved": flops / (expert_ms / prof_steps / 1e3) / 1e12,
                    "peak": tpeak, "unit": "TFLOP/s", "peak_kind": tpeak_kind, "traffic": None,
                    "flops_per_step": flops,
                    "hbm_achieved_gbs": achieved, "hbm_peak_gbs": peak,
                    "hbm_frac": (achieved / peak) if achieved else None}
        roofline["frac"] = roofline["achieved"] / tpeak
    else:
        roofline = {"bound": "hbm", "kernel": "k_expert_gemv gate_up + down (expert MXFP4 GEMVs)",
                    "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": (achieved / peak) if achieved else None,
                    "peak_kind": peak_kind, "traffic": None}

    tr = profiled_traffic(args.workload) if not args.layers else None
    if tr and not (prefill and not block_scaled):  # captured on the default mode's dominant kernel
        roofline.update({"traffic": tr["dram_bytes_per_launch"], "traffic_kernel": tr["kernel"],
                         "traffic_alg_bytes": tr["alg_bytes_per_launch_approx"],
                         "traffic_source": tr["source"],
                         "traffic_measured_in_this_run": False})
    roofline.update({"alg_bytes_per_step": step_bytes_total,
                     "expert_passes_per_step": prof["expert_passes"] / prof_steps,
                     "expert_ms_per_step": expert_ms / prof_steps,
                     "launches_timed": launches_prof,
                     "kernel_ms_per_step": {k: round(prof[k + "_ms"] / prof_steps, 4)
                                            for k in ("router", "gateup", "down", "combine")}})

    if rank == 0:
        value = T / (ms / 1e3)
        metric, unit = metric_unit(args.workload)
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("mxfp4 weights x mxfp8 (e4m3 + e8m0 per 32) activations, fp32 accumulate"
                      if block_scaled else "mxfp4 weights x bf16 activations, fp32 accumulate"),
            "data": "synthetic (seeded random-init bank, hidden ~N(0,1))",
            "config": workload_config(args.workload, world, args.ep, args.layers, skew),
            "run": {"bank_fill_s": round(fill_s, 2), "bank_bytes": bank.nbytes(),
                    **({"cuda_graph": graph is not None} if world > 1 else {}),
                    **({"graph_note": graph_note} if graph_note else {})},
            "e2e": {"value": T / (e2e_ms / 1e3), "unit": unit, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": Tr * H * 2, "d2h_bytes_per_step": Tr * H * 4},
            "gpu_launches": launches,
            "roofline": roofline,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline and world == 1:
            threads = os.cpu_count() or 1
            v, sample = cpu_reference_sample(spec, threads)
            v1, sample1 = cpu_reference_sample(spec, 1, budget_s=6.0)
            line["cpu_baseline"] = {"value": v, "unit": unit, "cores": threads, "kind": "port",
                                    "sample": sample,
                                    "single_thread": {"value": v1, "cores": 1, "sample": sample1}}
        if world == 1 and args.workload == DEFAULT_WORKLOAD and not args.layers:
            # config 0 (the metric's GEMV half), measured in the same run
            line["gemv_config0"] = measure_gemv(ctx, cur, local, 1500, 3, 1,
                                                cpu_baseline=not args.no_cpu_baseline)
            line["int8_head"] = measure_int8_head(ctx, cur, local, 200, 3,
                                                  cpu_baseline=not args.no_cpu_baseline)
        print(json.dumps(line), flush=True)
    if world > 1:
        # The teardown of a process group whose collectives a CUDA graph
        # captured has hung here: meet once more and leave without the graph,
        # library or NCCL teardown (process exit releases the GPU).
        torch.cuda.synchronize()
        _barrier(world)
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)
    bank.close()
    ctx.close()
    return 0


GEMV_ROUNDS = 7  # DequantGEMVBenchmark.swift:290-336: one warm-up, then the median of 7 rounds
GEMV_ALG = 4_429_440  # config 0 bytes per GEMV: packed + scales + x + bias + y
GEMV_COPIES = 128     # distinct matrices per batched launch (> 4x the 126 MB L2)


def measure_gemv(ctx, cur, local: int, steps: int, warmup: int, world: int = 1,
                 cpu_baseline: bool = True) -> dict:
    """Config 0 (2880x2880 MXFP4 GEMV, GPT-OSS down_proj shape) batched over
    R distinct copies (> 4x L2), timed the reference's way: warm-up, then
    GEMV_ROUNDS rounds of `steps` batched launches each, median round.
    Returns the JSON fields of its line."""
    import numpy as np
    import torch

    from godwit_b200 import device as D
    from godwit_b200 import synth

    rows = cols = 2880
    alg = GEMV_ALG
    l2 = torch.cuda.get_device_properties(local).L2_cache_size
    R = max(GEMV_COPIES, (4 * l2) // alg + 1)
    rng = np.random.default_rng(SEED)
    p0, s0 = synth.random_mxfp4(rng, rows, cols)
    x0 = synth.make_hidden(rng, 1, cols, "bf16")
    b0 = synth.f32_to_bf16_bits(rng.normal(0, 0.02, rows))
    # copy 0 is config 0's seeded matrix; the rest are independent random copies
    packed = torch.randint(0, 256, (R, rows, cols // 2), dtype=torch.uint8, device="cuda")
    scales = torch.randint(118, 125, (R, rows, cols // 32), dtype=torch.uint8, device="cuda")
    packed[0].copy_(torch.from_numpy(p0))
    scales[0].copy_(torch.from_numpy(s0))
    bias = torch.from_numpy(np.tile(b0.view(np.int16), (R, 1))).cuda()
    x_host = torch.from_numpy(np.tile(x0.view(np.int16), (R, 1))).view(torch.bfloat16).pin_memory()
    x = x_host.to("cuda")
    y = torch.empty(R, rows, dtype=torch.float32, device="cuda")
    y_host = torch.empty(R, rows, dtype=torch.float32).pin_memory()

    def step():
        D.gemv_batched(ctx, packed, scales, bias, x, y)

    for _ in range(max(warmup, 1)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    launches0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rounds = []
    for _ in range(GEMV_ROUNDS):
        ev0.record(cur)
        for _ in range(steps):
            step()
        ev1.record(cur)
        torch.cuda.synchronize()
        rounds.append(ev0.elapsed_time(ev1) / steps)
    launches = ctx.launch_count() - launches0
    ms = _max_over_ranks(statistics.median(rounds), world)
    ev0.record(cur)
    for _ in range(steps):
        x.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y, non_blocking=True)
    ev1.record(cur)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    e2e_ms = _max_over_ranks(ev0.elapsed_time(ev1) / steps, world)
    ctx.profile_enable(True)
    for _ in range(3):
        step()
    prof = ctx.profile_read()
    ctx.profile_enable(False)
    k_ms = prof["gemv_ms"] / max(prof["gemv_launches"], 1)
    achieved = R * alg / (k_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    gbs = R * alg * world / (ms / 1e3) / 1e9
    out = {
        "metric": "MXFP4 expert GEMV HBM GB/s", "value": gbs, "unit": "GB/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms,
        "rounds": GEMV_ROUNDS, "round_ms": [round(r, 4) for r in rounds],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "mxfp4 weights x bf16 x, fp32 accumulate", "data": "synthetic",
        "config": workload_config("gemv") if R == GEMV_COPIES else
                  {"workload": "gemv", "rows": rows, "cols": cols, "copies": R,
                   "l2": f"{R} distinct copies = {R * alg / 1e9:.2f} GB > 4x L2 per launch"},
        "run": {"protocol": f"warm-up, then median of {GEMV_ROUNDS} rounds of {steps} launches"},
        "e2e": {"value": R * alg * world / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": R * cols * 2, "d2h_bytes_per_step": R * rows * 4},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "k_gemv", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                     "alg_bytes_per_launch": R * alg, "traffic": None},
        "clocks": clocks,
    }
    if cpu_baseline and world == 1:
        threads = os.cpu_count() or 1
        v, sample = cpu_gemv_sample(threads)
        v1, sample1 = cpu_gemv_sample(1, budget_s=5.0)
        out["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                               "sample": sample,
                               "single_thread": {"value": v1, "cores": 1, "sample": sample1}}
    del packed, scales, bias, x, y
    torch.cuda.empty_cache()
    return out


HEAD_ROWS, HEAD_COLS = 201088, 2880  # GPT-OSS output head (vocabulary x hidden)


def cpu_int8_sample(threads: int, budget_s: float = 8.0):
    """The oracle port of int8_affine_gemv on a bounded slice of the head's
    rows, grown until it takes about `budget_s`; GB/s of weights streamed."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    rng = np.random.default_rng(SEED)
    rows = 2048
    while True:
        codes = rng.integers(0, 256, (rows, HEAD_COLS), dtype=np.uint8)
        meta = rng.integers(0x3800, 0x3900, (rows, HEAD_COLS // 64, 2), dtype=np.uint16)
        x = rng.standard_normal((1, HEAD_COLS)).astype(np.float16).astype(np.float32)
        t0 = time.perf_counter()
        O.int8_gemv(codes, meta, x, threads=threads)
        dt = time.perf_counter() - t0
        if dt * 4 > budget_s or rows >= HEAD_ROWS:
            break
        rows = min(HEAD_ROWS, rows * 4)
    nbytes = rows * HEAD_COLS + rows * (HEAD_COLS // 64) * 4
    return nbytes / dt / 1e9, f"{rows} of the head's {HEAD_ROWS} rows, one token, {dt:.2f} s on {threads} threads"


def measure_int8_head(ctx, cur, local: int, steps: int, warmup: int, cpu_baseline: bool = True) -> dict:
    """The trunk's largest int8 projection: the GPT-OSS output head (201088 x
    2880 int8 codes + bf16 scale/zero per 64, 0.62 GB > L2) for one token,
    int8_affine_gemv (router.metal:65-98).  Timed like config 0: warm-up, then
    the median of GEMV_ROUNDS rounds of `steps` launches."""
    import numpy as np
    import torch

    from godwit_b200 import device as D

    rows, cols = HEAD_ROWS, HEAD_COLS
    g = torch.Generator(device="cuda").manual_seed(SEED)
    codes = torch.randint(0, 256, (rows, cols), dtype=torch.uint8, device="cuda", generator=g)
    # bf16 scales ~1.5e-4 and zero points ~ -0.02 (a +-0.02 weight range)
    sc = torch.empty(rows, cols // 64, device="cuda").uniform_(1e-4, 2e-4, generator=g)
    zr = -sc * 127.5
    meta = torch.stack([sc.to(torch.bfloat16), zr.to(torch.bfloat16)], -1).contiguous().view(torch.int16)
    x_host = torch.randn(1, cols, generator=torch.Generator().manual_seed(SEED)).half().pin_memory()
    x = x_host.to("cuda")
    y = torch.empty(1, rows, dtype=torch.float32, device="cuda")
    y_host = torch.empty(1, rows, dtype=torch.float32).pin_memory()
    alg = rows * cols + rows * (cols // 64) * 4 + cols * 2 + rows * 4

    def step():
        D.int8_affine_gemv(ctx, codes, meta, None, x, y)

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    launches0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rounds = []
    for _ in range(GEMV_ROUNDS):
        ev0.record(cur)
        for _ in range(steps):
            step()
        ev1.record(cur)
        torch.cuda.synchronize()
        rounds.append(ev0.elapsed_time(ev1) / steps)
    launches = ctx.launch_count() - launches0
    ms = statistics.median(rounds)
    ev0.record(cur)
    for _ in range(steps):
        x.copy_(x_host, non_blocking=True)
        step()
        y_host.copy_(y, non_blocking=True)
    ev1.record(cur)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    e2e_ms = ev0.elapsed_time(ev1) / steps
    peak, peak_kind = peaks()
    gbs = alg / (ms / 1e3) / 1e9
    out = {
        "metric": "int8 affine head GEMV HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
        "steps": steps, "warmup": warmup, "ms_per_step": ms, "rounds": GEMV_ROUNDS,
        "round_ms": [round(r, 4) for r in rounds], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 affine (bf16 scale/zero per 64) x f16, fp32 accumulate",
        "data": "synthetic",
        "config": workload_config("int8-head"),
        "run": {"protocol": f"warm-up, then median of {GEMV_ROUNDS} rounds of {steps} launches"},
        "e2e": {"value": alg / (e2e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": cols * 2,
                "d2h_bytes_per_step": rows * 4},
        "gpu_launches": launches,
        # one kernel per step: the round timing is the kernel's own duration
        "roofline": {"bound": "hbm", "kernel": "k_int8_gemv", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "peak_kind": peak_kind, "alg_bytes_per_launch": alg, "traffic": None},
        "clocks": clocks,
    }
    if cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample = cpu_int8_sample(threads)
        out["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}
    del codes, meta, sc, zr, x, y
    torch.cuda.empty_cache()
    return out


def run_int8_head(args):
    from godwit_b200 import device as D
    from godwit_b200.runtime import Context

    world, rank, local = _dist_setup(args)
    ctx = Context(local)
    cur = D.bind_stream(ctx)
    line = measure_int8_head(ctx, cur, local, args.steps, args.warmup, cpu_baseline=not args.no_cpu_baseline)
    if rank == 0:
        line["n_gpus"] = world
        print(json.dumps(line), flush=True)
    ctx.close()
    return 0


def run_gemv(args):
    from godwit_b200 import device as D
    from godwit_b200.runtime import Context

    world, rank, local = _dist_setup(args)
    ctx = Context(local)
    cur = D.bind_stream(ctx)
    line = measure_gemv(ctx, cur, local, args.steps, args.warmup, world,
                        cpu_baseline=not args.no_cpu_baseline)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
