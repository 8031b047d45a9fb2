"""Benchmark of the Mamba-3 single-token decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {native,reference}]
                    [--workload NAME]

Default workload: the 24-layer MIMO rank-4 stack (residual + RMSNorm between
blocks), d_model=2048, d_inner=4096, headdim=64 (64 heads), d_state=128,
bf16 weights, fp32 state, a global batch of 256 sequences split evenly over
the N GPUs (strong scaling: 256 / N sequences per GPU) -- the largest
configuration of the reference's decode that one GPU holds.  Weights:
torch.manual_seed(0), in_proj / out_proj ~ N(0, 0.02), the other parameters
per the layer's own init; inputs u ~ N(0, 1) from seed 1 + rank; synthetic
data, zero initial state.  Every workload's batch is global and split the
same way.

A step is one decode step of the rank's sequences through all layers,
replayed from one captured CUDA graph.  Between timed steps L2 is flushed
by writing a 256 MiB buffer; each step is timed with its own CUDA event
pair on the launching stream (the flush is outside the pair).  ``value`` =
global batch x K / (max over ranks of the summed step times).

``e2e`` times the public API end to end: per step, the pinned host input
is copied to the device, the decoder's ``step`` replays the graph, the
output is copied back to pinned host memory and the stream synchronised
so the host holds the result; the event pair brackets all of it.  Its mean
and p50 are reported.

``roofline`` is the dominant kernel of one layer (the fused decode kernel,
or the single-launch step where a layer runs as one kernel): algorithmic
HBM bytes per launch over its mean duration in an event-timed loop with
the same L2 flush (replayed from a one-node CUDA graph, so host dispatch
stays out of the timing), against the measured HBM copy bandwidth.  At
N=1 the default run adds ``fused_rooflines``: the same measurement for the
fused kernel of the d512 bf16 SISO layer at batch 512 and of the d1024
fp32 MIMO layers (R = 1, 2, 4, 8) at batch 4096.

``cpu_baseline`` and ``--impl reference`` time the reference's own
PyTorch CPU decode (``Mamba3Decoder(model, use_triton=False).step``,
composed over the stack's ``MambaBlock``s) on the host cores, unmodified,
in a separate interpreter (``oracle/reference_cpu.py``, from the copy that
``oracle/stage_reference.py`` staged under ``baseline/_ref``); without that
copy they fall back to the numpy restatement (``kind: "port"``).

Multi-GPU (torchrun): every rank decodes its share of the global batch with
a full weight replica and its own graph; no collective runs on the decode
path (NCCL is used for the barrier and the max-over-ranks timing only).
"""

from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "mamba3-fused-triton-kernel_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402

# name -> (layer kwargs, global batch, weight dtype)
WORKLOADS = {
    "mimo_r4_d256_b128": (dict(d_model=256, d_state=64, headdim=32, is_mimo=True, mimo_rank=4), 128, "f32"),
    "siso_d256_b1": (dict(d_model=256, d_state=64, headdim=32), 1, "f32"),
    "siso_d256_b1024": (dict(d_model=256, d_state=64, headdim=32), 1024, "f32"),
    "siso_d512_b512_bf16": (dict(d_model=512, d_state=128, headdim=64), 512, "bf16"),
    "mimo_r8_d512_b512_bf16": (dict(d_model=512, d_state=128, headdim=64, is_mimo=True, mimo_rank=8), 512, "bf16"),
    "mimo_r4_d1024_b4096": (dict(d_model=1024, d_state=128, headdim=64, is_mimo=True, mimo_rank=4), 4096, "f32"),
    "mimo_r1_d1024_b4096": (dict(d_model=1024, d_state=128, headdim=64, is_mimo=True, mimo_rank=1), 4096, "f32"),
    "mimo_r8_d1024_b4096": (dict(d_model=1024, d_state=128, headdim=64, is_mimo=True, mimo_rank=8), 4096, "f32"),
}
# residual stacks: workload -> number of layers (the 24-layer bf16 stack of
# the reference's multi-GPU configuration)
STACKS = {"stack24_d2048_b256_bf16": 24, "lm24_d2048_b256_bf16": 24}
WORKLOADS["stack24_d2048_b256_bf16"] = (dict(d_model=2048, d_state=128, headdim=64, is_mimo=True, mimo_rank=4),
                                        256, "bf16")
# the same stack as a language model: token ids in, logits out (embedding,
# 24 blocks, final norm, LM head tied to the embedding; the default vocabulary)
LM_WORKLOADS = {"lm24_d2048_b256_bf16": 50277}
LM_STACK_PROFILE = {"lm24_d2048_b256_bf16": "stack24_d2048_b256_bf16"}  # same fused kernel and shapes
# prompt prefill of one MIMO layer (Mamba3Decoder.prefill): batch sequences x prompt tokens
PREFILLS = {"prefill_d2048_b64_l512_bf16": 512, "prefill_siso_d2048_b64_l512_bf16": 512}
WORKLOADS["prefill_d2048_b64_l512_bf16"] = (dict(d_model=2048, d_state=128, headdim=64, is_mimo=True,
                                                 mimo_rank=4), 64, "bf16")
WORKLOADS["prefill_siso_d2048_b64_l512_bf16"] = (dict(d_model=2048, d_state=128, headdim=64), 64, "bf16")
WORKLOADS["lm24_d2048_b256_bf16"] = WORKLOADS["stack24_d2048_b256_bf16"]
DEFAULT_WORKLOAD = "stack24_d2048_b256_bf16"
# Published reference number for the default workload: MIMO d256 B=128
# full-fused + CUDA graph P50 step latency 0.295 ms on an A100-PCIE-40GB
# (reference README.md:229) -> 128 / 0.295 ms tokens/s.
PUBLISHED = {"mimo_r4_d256_b128": 128 / 0.295e-3}
FLUSH_BYTES = 256 * 1024 * 1024
HBM_FALLBACK_GBS = 6650.0


def fused_bytes_per_launch(m, batch: int, zx_bytes: int, y_bytes: int) -> int:
    """Algorithmic HBM bytes of one fused decode launch: the in_proj output
    row (read), ssm_state and bx_prev (read + write), angle_state (read +
    write), the gated output (write) and the per-head parameters (read once)."""
    H, P, D, R, A = m.nheads, m.headdim, m.d_state, m.mimo_rank, m.num_rope_angles
    S = batch * H * (D if m.is_mimo else P * D)
    params = 4 * (2 * H + 2 * D + 2 * H * R * D + (2 * H * R * P if m.is_mimo else 0))
    return batch * m.d_in_proj * zx_bytes + 16 * S + 8 * batch * H * A + batch * m.d_inner * y_bytes + params


def step_bytes_per_launch(m, batch: int, es: int) -> int:
    """Algorithmic HBM bytes of one single-launch decode step: both projection
    weights, the input and output rows, ssm_state and bx_prev (read + write),
    angle_state (read + write) and the per-head parameters.  The in_proj
    output and the gated output stay in L2 between the kernel's phases."""
    H, P, D, R, A = m.nheads, m.headdim, m.d_state, m.mimo_rank, m.num_rope_angles
    S = batch * H * D
    params = es * (2 * H + 2 * D + 2 * H * R * D + 2 * H * R * P)
    weights = es * (m.d_in_proj * m.d_model + m.d_model * m.d_inner)
    return weights + 2 * batch * m.d_model * es + 16 * S + 8 * batch * H * A + params


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def profile_traffic(workload: str, kernel: str):
    """DRAM bytes per launch of the dominant kernel (``kernel``: "step" for
    the single-launch step, "fused" for the fused decode kernel) recorded by
    an ncu capture summary of this workload under profiles/ (a line
    ``dram_bytes_per_launch[<kernel>]: N``), or None."""
    import glob
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", f"*{workload}*.md"))):
        with open(path) as f:
            mt = re.search(r"dram_bytes_per_launch\[" + kernel + r"\]:\s*([0-9]+)", f.read())
        if mt:
            return int(mt.group(1))
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while running."""

    FIELDS = ("index,timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.proc = None
        self.gpu_ids = gpu_ids
        self.marks = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(map(str, self.gpu_ids)), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def mark(self):
        self.marks.append(time.time())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = time.mktime(time.strptime(f[1].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                ts += float("0." + f[1].split(".")[1]) if "." in f[1] else 0.0
                rows.append((ts, int(f[2]), int(f[3]), f[5:9]))
            except (ValueError, IndexError):
                continue
        if not rows:
            return None
        window = "timed"
        sel = [r for r in rows if len(self.marks) >= 2 and self.marks[0] <= r[0] <= self.marks[-1]]
        if not sel:
            sel, window = rows, "whole run (timed region shorter than the sampling interval)"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in sel for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": int(np.median([r[1] for r in sel])), "sm_max_mhz": max(r[2] for r in sel),
                "reasons": reasons, "samples": len(sel), "window": window}


def cpu_oracle_rate(kw, batch, dtype_name, steps=None, budget_s=10.0, warmup=1):
    """Time the numpy oracle decode step on the host cores; returns
    (tokens/s, steps timed, cores used)."""
    from oracle import mamba3_oracle as orc
    dims = orc.layer_dims(**kw)
    bf16 = dtype_name == "bf16"
    params = orc.synthetic_params(dims, 0, bf16=bf16, randomize_small=False)
    st = orc.init_state(dims, batch)
    us = orc.synthetic_inputs(dims, batch, 16, 1, bf16=bf16)  # cycled, like the GPU side
    for i in range(warmup):
        _, st = orc.decode_step(us[i % 16], params, dims, st, bf16=bf16)
    n, t0 = 0, time.perf_counter()
    while True:
        _, st = orc.decode_step(us[n % 16], params, dims, st, bf16=bf16)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and (el >= budget_s or n >= 10000)):
            break
    return batch * n / el, n, os.cpu_count() or 1


def shard_rows(global_batch: int, world: int) -> int:
    """Sequences each rank decodes: the global batch split evenly (strong
    scaling); every sequence is independent, so no collective is needed."""
    if global_batch % world:
        raise SystemExit(f"the global batch {global_batch} does not split evenly over {world} GPUs")
    return global_batch // world


def reference_cpu_rate(kw, batch, dtype_name, layers=1, steps=0, budget_s=10.0, warmup=1, ssm=False):
    """The reference's own PyTorch CPU decode of `batch` sequences through
    `layers` blocks (with `ssm`: its state-update-only MIMO decode), timed on
    the host cores in its own interpreter (oracle/reference_cpu.py, no GPU
    visible).  Returns (result dict, None) or (None, why it is unavailable)."""
    cmd = [sys.executable, os.path.join(ROOT, "oracle", "reference_cpu.py"), "--layer", json.dumps(kw),
           "--dtype", dtype_name, "--batch", str(batch), "--layers", str(layers), "--warmup", str(warmup),
           "--budget", str(budget_s)]
    if steps:
        cmd += ["--steps", str(steps)]
    if ssm:
        cmd += ["--ssm"]
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1", CUDA_VISIBLE_DEVICES="")
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=1800)
    except subprocess.TimeoutExpired:
        return None, "the reference CPU run timed out"
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return None, f"the reference CPU run failed (rc {r.returncode}): {r.stderr.strip()[-200:]}"
    d = json.loads(lines[-1])
    if "unavailable" in d:
        return None, d["unavailable"]
    return d, None


def cpu_baseline(kw, batch, dtype_name, layers=1, budget_s=10.0, steps=0, warmup=1):
    """(cpu_baseline dict, ms per step, steps timed): the reference's own
    CPU decode when its staged copy is present, else the numpy port."""
    d, why = reference_cpu_rate(kw, batch, dtype_name, layers, steps, budget_s, warmup)
    if d is not None:
        what = f" through {layers} MambaBlocks (x <- x + step(norm(x)))" if layers > 1 else ""
        return ({"value": round(d["tokens_per_s"], 1), "unit": "tokens/s", "cores": d["threads"],
                 "kind": "reference",
                 "sample": f"{d['steps']} steps of the reference's Mamba3Decoder(use_triton=False).step on "
                           f"{batch} sequences{what}, {dtype_name} weights, torch CPU with {d['threads']} "
                           f"threads, p50 {d['p50_ms']:.2f} ms"},
                d["ms_per_step"], d["steps"])
    rate, n, cores = cpu_oracle_rate(kw, batch, dtype_name, steps=steps or None, budget_s=budget_s, warmup=warmup)
    rate /= layers
    return ({"value": round(rate, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
             "sample": f"{n} oracle decode steps of one layer x {batch} sequences (numpy restatement), rate "
                       f"divided by {layers} layers; the reference itself was unavailable: {why}"},
            1000.0 * batch / rate, n)


def config_dict(workload, kw, global_batch, world, dtype_name, reference=False):
    published = PUBLISHED.get(workload)
    if reference:
        par, l2, step = ("rank 0 only (host cores), the whole global batch", "n/a (CPU)",
                         "the reference's PyTorch CPU decode step")
    else:
        par = f"batch-sharded x{world} ({global_batch // world} sequences per GPU), no collective on the decode path"
        l2 = "flushed (256 MiB write) before every timed step; per-step CUDA events"
        step = ("CUDA-graph replay of Mamba3Decoder.step: one single-launch kernel (in_proj, fused update, "
                "out_proj) for MIMO layers it takes, else in_proj GEMM + fused decode kernel + out_proj GEMM")
    return {"workload": workload, "batch_per_gpu": global_batch // world, "global_batch": global_batch,
            **kw, "weights": dtype_name, "state": "f32", "parallelism": par, "l2": l2, "step": step,
            "baseline": ("A100 full-fused+graph P50 0.295 ms at B=128 (reference README.md:229)"
                         if published else None)}


def run_reference(args, kw, global_batch, dtype_name, rank):
    """--impl reference: the reference's own PyTorch CPU decode of the whole
    global batch on rank 0's host cores (stacks: through all their blocks),
    each timed step one decode step; bounded to about a minute of steps."""
    if rank != 0:
        return
    if args.workload in SSM_WORKLOADS:
        d, why = reference_cpu_rate(kw, global_batch, dtype_name, 1, args.steps, 60.0, min(args.warmup, 3), ssm=True)
        if d is None:
            print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
            return
        cpu = {"value": round(d["tokens_per_s"], 1), "unit": "sequences/s", "cores": d["threads"],
               "kind": "reference",
               "sample": f"{d['steps']} calls of the reference's mamba3_mimo_decode_ref on {global_batch} "
                         f"sequences, torch CPU with {d['threads']} threads, p50 {d['p50_ms']:.2f} ms"}
        line = {"metric": "state-update sequences/s", "value": cpu["value"], "unit": "sequences/s",
                "impl": "reference", "n_gpus": args.gpus, "steps": d["steps"], "warmup": args.warmup,
                "ms_per_step": round(d["ms_per_step"], 4), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": config_dict(args.workload, kw, global_batch, 1, dtype_name, reference=True),
                "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": "sequences/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    layers = STACKS.get(args.workload, 1)
    cpu, ms, n = cpu_baseline(kw, global_batch, dtype_name, layers, budget_s=60.0, steps=args.steps,
                              warmup=min(args.warmup, 3))
    cfg = config_dict(args.workload, kw, global_batch, 1, dtype_name, reference=True)
    cfg["layers"] = layers
    metric = "decode tokens/s"
    if args.workload in PREFILLS:
        # a prefill on the host is one decode step per prompt token, so its
        # tokens/s is the decode rate; ms_per_step stays one batch of tokens
        metric = "prefill tokens/s"
        cfg["prompt_tokens"] = PREFILLS[args.workload]
        cpu["sample"] += " (a prefill on the host steps every prompt token)"
    if args.workload in LM_WORKLOADS:
        cpu["sample"] += " (embedding and LM head not included)"
    line = {
        "metric": metric, "value": cpu["value"], "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": n, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype_name,
        "data": "synthetic", "config": cfg, "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Harness:
    """Per-rank plumbing shared by every workload: the device, the process
    group (N > 1), the L2 flush buffer, event-timed loops, max over ranks
    and the clock sampler."""

    def __init__(self, world: int, rank: int, local: int):
        import datetime

        import torch.distributed as dist

        self.dist, self.world, self.rank = dist, world, rank
        torch.cuda.set_device(local)
        self.dev = torch.device("cuda", local)
        if world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
        self.flush = torch.empty(FLUSH_BYTES // 4, device=self.dev, dtype=torch.float32)
        self.stream = torch.cuda.current_stream(self.dev)
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        try:
            gpus = [int(x) for x in vis.split(",")][:world] if vis else list(range(world))
        except ValueError:
            gpus = list(range(world))
        self.sampler = ClockSampler(gpus) if rank == 0 else None

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], device=self.dev, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed_loop(self, fn, n: int, pre_sync: bool = False) -> np.ndarray:
        """n calls of fn(i), each bracketed by its own CUDA event pair on the
        launching stream after an L2 flush; per-call milliseconds.  With
        ``pre_sync`` the host waits for the flush before the pair (end-to-end
        calls that synchronise themselves), else a short device sleep keeps
        the GPU busy while the host enqueues the call."""
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            self.flush.zero_()
            if pre_sync:
                self.stream.synchronize()
            else:
                torch.cuda._sleep(20000)
            ev[i][0].record(self.stream)
            fn(i)
            ev[i][1].record(self.stream)
        torch.cuda.synchronize(self.dev)
        return np.array([a.elapsed_time(b) for a, b in ev])

    def graphed(self, fn, warm: int = 3):
        """fn captured in a CUDA graph (after `warm` calls on a side stream)."""
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            for _ in range(warm):
                fn()
        self.stream.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def clocks_start(self):
        if self.sampler:
            self.sampler.start()
            time.sleep(0.2)

    def clocks_mark(self):
        if self.sampler:
            self.sampler.mark()

    def clocks_stop(self):
        return self.sampler.stop() if self.sampler else None

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def e2e_summary(h: Harness, ms: np.ndarray, tokens_per_step: int, h2d: int, d2h: int, path: str) -> dict:
    total = h.max_over_ranks(float(ms.sum()))
    p50 = h.max_over_ranks(float(np.percentile(ms, 50)))
    return {"value": round(tokens_per_step * len(ms) / (total / 1000.0), 1), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(total / len(ms), 5),
            "p50_ms": round(p50, 5), "steps": len(ms), "path": path}


def fused_kernel_roofline(h: Harness, kw: dict, batch: int, dtype_name: str, n: int, copies: int = 4) -> dict:
    """One layer's fused decode kernel alone: `copies` launches back to back
    in one graph, each on its own carried state (together beyond L2), L2
    flushed before every replay; the mean CUDA-event time per launch over n
    replays and its algorithmic HBM bytes against the measured copy
    bandwidth."""
    from src.kernels.linear import linear
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3

    wdtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    torch.manual_seed(0)
    model = Mamba3(**kw, device=h.dev, dtype=wdtype)
    with torch.no_grad():
        model.in_proj.weight.normal_(0.0, 0.02)
        decs = [Mamba3Decoder(model, use_triton_full_fused=True) for _ in range(copies)]
        launches = [d._fused_launch(d.init_state(batch, device=h.dev)) for d in decs]
        gen = torch.Generator(device=h.dev).manual_seed(1)
        zx = linear(torch.randn(batch, model.d_model, device=h.dev, generator=gen).to(wdtype), model.in_proj.weight)
        y = torch.zeros(batch, model.d_inner, device=h.dev, dtype=wdtype)
        g = h.graphed(lambda: [L.run(zx, y) for L in launches])
        ms = h.timed_loop(lambda i: g.replay(), n) / copies
    del g, launches, decs
    es = 2 if wdtype == torch.bfloat16 else 4
    nbytes = fused_bytes_per_launch(model, batch, es, es)
    mean = h.max_over_ranks(float(ms.mean()))
    peak, peak_kind = hbm_peak()
    achieved = nbytes / (mean * 1e-3) / 1e9
    return {"kernel": "m3_mimo_full_fused" if model.is_mimo else "m3_siso_full_fused", "batch": batch,
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes, "mean_launch_ms": round(mean, 5),
            "method": f"{copies} launches back to back in one graph on distinct states, L2 flushed before each "
                      "replay; mean per launch"}


# the stack's projections alone: 24 layers of in_proj (9440 x 2048) and
# out_proj (2048 x 4096), bf16, batch 256, in one CUDA graph, timed for the
# library's tcgen05 GEMM (m3_linear_bf16) and for cuBLAS
PROJECTIONS = {"proj24_d2048_b256_bf16": 24, "proj24_d2048_b32_bf16": 24, "proj24_d2048_b8_bf16": 24,
               "proj24_d2048_b1_bf16": 24}
WORKLOADS["proj24_d2048_b256_bf16"] = (dict(d_model=2048, d_state=128, headdim=64, is_mimo=True, mimo_rank=4), 256,
                                       "bf16")
# the same projections at one GPU's share of the stack's batch 256 under
# strong scaling over 8 GPUs (32 rows), and at small-batch decodes (8 rows,
# 1 row), where the weight-streaming kernel (m3_linear_bf16_skinny) is timed
# as well
WORKLOADS["proj24_d2048_b32_bf16"] = (dict(d_model=2048, d_state=128, headdim=64, is_mimo=True, mimo_rank=4), 32,
                                      "bf16")
WORKLOADS["proj24_d2048_b8_bf16"] = (dict(d_model=2048, d_state=128, headdim=64, is_mimo=True, mimo_rank=4), 8,
                                     "bf16")
WORKLOADS["proj24_d2048_b1_bf16"] = (dict(d_model=2048, d_state=128, headdim=64, is_mimo=True, mimo_rank=4), 1,
                                     "bf16")


# fused-kernel rooflines added to the default run at N=1: the wide SISO layer
# at its largest batch and the throughput sweep's layer at every rank
EXTRA_ROOFLINES = ["siso_d512_b512_bf16", "mimo_r1_d1024_b4096", "mimo_r2_d1024_b4096", "mimo_r4_d1024_b4096",
                   "mimo_r8_d1024_b4096"]
WORKLOADS["mimo_r2_d1024_b4096"] = (dict(d_model=1024, d_state=128, headdim=64, is_mimo=True, mimo_rank=2), 4096,
                                    "f32")


def run_stack(args, kw, global_batch, dtype_name, layers, world, rank, local):
    """A residual stack of `layers` MIMO blocks decoded token by token through
    Mamba3StackDecoder, the whole stack step in one CUDA graph, each rank
    decoding its share of the global batch.  `roofline` is one layer's fused
    decode kernel; the projections' rate is reported beside it."""
    from src.kernels.linear import linear
    from src.models.lm import Mamba3LMDecoder
    from src.models.mamba3 import MambaBlock, MambaConfig, MambaLMHeadModel
    from src.models.stack import Mamba3StackDecoder

    h = Harness(world, rank, local)
    dev = h.dev
    batch = shard_rows(global_batch, world)
    wdtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    torch.manual_seed(0)
    mkw = {k: v for k, v in kw.items() if k != "d_model"}
    vocab = LM_WORKLOADS.get(args.workload)
    blocks = []
    with torch.no_grad():
        if vocab is not None:
            lm = MambaLMHeadModel(MambaConfig(d_model=kw["d_model"], n_layer=layers, vocab_size=vocab, ssm_cfg=mkw),
                                  device=dev, dtype=wdtype)
            blocks = list(lm.layers)
        else:
            for _ in range(layers):
                blocks.append(MambaBlock(kw["d_model"], mkw, device=dev, dtype=wdtype))
        for blk in blocks:
            blk.mixer.in_proj.weight.normal_(0.0, 0.02)
            blk.mixer.out_proj.weight.normal_(0.0, 0.02)
    model = blocks[0].mixer
    if vocab is not None:
        dec = Mamba3LMDecoder(lm, use_cuda_graph=True, use_triton_full_fused=True)
    else:
        dec = Mamba3StackDecoder(blocks, use_cuda_graph=True, use_triton_full_fused=True)
    states = dec.init_state(batch, device=dev)
    K, W = args.steps, args.warmup
    gen = torch.Generator(device="cpu").manual_seed(1 + rank)
    n_inputs = 16
    if vocab is not None:  # token ids in, logits out
        u_host = torch.randint(0, vocab, (n_inputs, batch), generator=gen).pin_memory()
        out_shape = (batch, lm.vocab_size)
    else:
        u_host = torch.randn(n_inputs, batch, kw["d_model"], generator=gen).to(wdtype).pin_memory()
        out_shape = (batch, kw["d_model"])
    u_dev = u_host.to(dev)
    with torch.no_grad():
        dec.warmup_cuda_graph(states, n_warmup=2)
        for i in range(W):
            dec.step(u_dev[i % n_inputs], states)

    h.clocks_start()
    h.barrier()
    h.clocks_mark()
    with torch.no_grad():
        step_ms = h.timed_loop(lambda i: dec.step(u_dev[i % n_inputs], states), K)
    h.barrier()
    h.clocks_mark()
    total_ms = h.max_over_ranks(float(step_ms.sum()))
    p50_all = h.max_over_ranks(float(np.percentile(step_ms, 50)))
    p99_all = h.max_over_ranks(float(np.percentile(step_ms, 99)))
    value = global_batch * K / (total_ms / 1000.0)

    # the fused kernel (roofline): every layer's launch on its own carried
    # state (the stack's 24 x 37.7 MB, far beyond L2), back to back in one
    # graph as the stack step runs them, so its mean per launch is the
    # kernel's average launch duration; one launch alone and the two
    # projections each from their own graph, L2 flushed before every replay
    es = 2 if wdtype == torch.bfloat16 else 4
    xn = torch.randn(batch, kw["d_model"], device=dev).to(wdtype)
    with torch.no_grad():
        zx = linear(xn, model.in_proj.weight)
        y = torch.zeros(batch, model.d_inner, device=dev, dtype=wdtype)
        launches = [dec.layers[l]._fused_launch(states[l]) for l in range(layers)]
        graphs = [h.graphed(fn, warm=2) for fn in (lambda: [L.run(zx, y) for L in launches],
                                                   lambda: launches[0].run(zx, y),
                                                   lambda: linear(xn, model.in_proj.weight),
                                                   lambda: linear(y, model.out_proj.weight))]
        n_k = min(K, 200)
        fa_ms, f1_ms, gi_ms, go_ms = (h.timed_loop(lambda i, g=g: g.replay(), n_k) for g in graphs)
    del graphs
    k_mean = h.max_over_ranks(float(fa_ms.mean())) / layers
    k_single = h.max_over_ranks(float(f1_ms.mean()))
    gi_mean = h.max_over_ranks(float(gi_ms.mean()))
    go_mean = h.max_over_ranks(float(go_ms.mean()))
    nbytes = fused_bytes_per_launch(model, batch, es, es)
    peak, peak_kind = hbm_peak()
    achieved = nbytes / (k_mean * 1e-3) / 1e9
    gemm_flop = 2.0 * batch * model.d_model * (model.d_in_proj + model.d_inner)

    # end to end through the public API: pinned input in, output back to the host
    out_host = torch.empty(*out_shape, dtype=wdtype).pin_memory()
    u_stage = torch.empty(u_host.shape[1:], device=dev, dtype=u_host.dtype)

    def e2e_step(i):
        u_stage.copy_(u_host[i % n_inputs], non_blocking=True)
        out, _ = dec.step(u_stage, states)
        out_host.copy_(out, non_blocking=True)
        h.stream.synchronize()

    h.barrier()
    with torch.no_grad():
        e2e_ms = h.timed_loop(e2e_step, max(min(K, 500), 1), pre_sync=True)
    h.barrier()
    e2e = e2e_summary(h, e2e_ms, global_batch, u_stage.numel() * u_stage.element_size(),
                      out_host.numel() * out_host.element_size(),
                      "pinned input copied in, graph replay, output copied to pinned host memory, stream sync")
    clocks = h.clocks_stop()

    extra = None
    if world == 1 and args.fused_rooflines and vocab is None:
        extra = {}
        for name in EXTRA_ROOFLINES:
            ekw, eb, edt = WORKLOADS[name]
            extra[name] = fused_kernel_roofline(h, ekw, eb, edt, min(K, 50))
    cpu = None
    if rank == 0 and world == 1:
        cpu, _, _ = cpu_baseline(kw, global_batch, dtype_name, layers, budget_s=args.cpu_budget)
        if vocab is not None:
            cpu["sample"] += " (embedding and LM head not included)"
    h.close()
    if rank == 0:
        cfg = config_dict(args.workload, kw, global_batch, world, dtype_name)
        proj = "cuBLAS bf16" if dtype_name == "bf16" else "cuBLAS / small-batch fp32"
        cfg.update({"layers": layers, "step": "CUDA-graph replay of Mamba3StackDecoder.step: per layer "
                    f"in_proj ({proj}) + fused decode kernel + out_proj ({proj}), residual add + RMSNorm "
                    "kernel between blocks"})
        if vocab is not None:
            cfg.update({"model": "MambaLMHeadModel", "vocab_size": vocab, "padded_vocab": lm.vocab_size,
                        "step": "CUDA-graph replay of Mamba3LMDecoder.step: token ids -> embedding, per layer "
                        f"in_proj ({proj}) + fused decode kernel + out_proj ({proj}) + residual add and RMSNorm "
                        "kernel, final norm, LM head -> logits"})
        line = {
            "metric": "decode tokens/s", "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total_ms / K, 5),
            "p50_step_ms": round(p50_all, 5), "p99_step_ms": round(p99_all, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": dtype_name, "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": "fused decode (m3_mimo_full_fused), one layer",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes,
                         "mean_launch_ms": round(k_mean, 5),
                         "method": f"{layers} launches back to back in one graph, each on its own layer's carried "
                                   "state, L2 flushed before each replay; mean per launch",
                         "single_launch_ms": round(k_single, 5),
                         "traffic": profile_traffic(LM_STACK_PROFILE.get(args.workload, args.workload), "fused")},
            "kernels_ms": {"fused_decode_per_layer": round(k_mean, 5),
                           "in_proj_gemm_per_layer": round(gi_mean, 5),
                           "out_proj_gemm_per_layer": round(go_mean, 5),
                           "projection_tflops": round(gemm_flop / ((gi_mean + go_mean) * 1e-3) / 1e12, 1)},
            "fused_rooflines": extra,
            "e2e": e2e,
            "gpu_launches": K * (2 * layers + 1),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    dec._graph = None


def run_projections(args, kw, global_batch, dtype_name, layers, world, rank, local):
    """The stack's projection GEMMs alone: per layer in_proj (d_in_proj x
    d_model) and out_proj (d_model x d_inner) with their own bf16 weights,
    all layers in one CUDA graph, replayed without an L2 flush (the 1.3 GB
    of weights stream from HBM anyway); timed for the library's tcgen05 GEMM
    (m3_linear_bf16), for the weight-streaming kernel
    (m3_linear_bf16_skinny) when a rank's batch is at most 64 rows, and for
    cuBLAS.  `value` is the rate in tokens/s (batch x steps / time) of the
    faster library kernel; the per-layer times, FLOP rates and weight-stream
    bandwidths of all of them are beside it."""
    import torch.nn.functional as F

    from src.kernels.linear import SKINNY_MAX_M, linear_bf16, linear_bf16_skinny
    from src.models.mamba3 import Mamba3

    h = Harness(world, rank, local)
    dev = h.dev
    batch = shard_rows(global_batch, world)
    m = Mamba3(**kw, device="meta")
    n_in, k_in, n_out, k_out = m.d_in_proj, m.d_model, m.d_model, m.d_inner
    torch.manual_seed(0)
    w_in = [(torch.randn(n_in, k_in, device=dev) * 0.02).bfloat16() for _ in range(layers)]
    w_out = [(torch.randn(n_out, k_out, device=dev) * 0.02).bfloat16() for _ in range(layers)]
    x = torch.randn(batch, k_in, device=dev).bfloat16()
    y = torch.randn(batch, k_out, device=dev).bfloat16()
    ref = (x.double() @ w_in[0].double().T)
    err = float((linear_bf16(x, w_in[0], torch.float32).double() - ref).abs().max())
    impls = [("m3_linear_bf16", lambda a, b: linear_bf16(a, b))]
    if batch <= SKINNY_MAX_M:
        err = max(err, float((linear_bf16_skinny(x, w_in[0], torch.float32).double() - ref).abs().max()))
        impls.append(("m3_linear_bf16_skinny", lambda a, b: linear_bf16_skinny(a, b)))
    impls.append(("cublas", F.linear))

    def chain(lin):
        def f():
            for l in range(layers):
                lin(x, w_in[l])
                lin(y, w_out[l])
        return f

    K, W = args.steps, args.warmup
    results = {}
    h.clocks_start()
    h.barrier()
    h.clocks_mark()
    for name, lin in impls:
        g = h.graphed(chain(lin), warm=max(W, 1))
        ms = h.timed_loop(lambda i: g.replay(), K)
        del g
        results[name] = h.max_over_ranks(float(np.median(ms)))
    h.barrier()
    h.clocks_mark()
    clocks = h.clocks_stop()
    h.close()
    if rank == 0:
        flop = 2.0 * batch * layers * (n_in * k_in + n_out * k_out)
        wbytes = 2.0 * layers * (n_in * k_in + n_out * k_out)
        per = {k: round(v / layers * 1000.0, 2) for k, v in results.items()}
        best = min((k for k in results if k != "cublas"), key=lambda k: results[k])
        line = {
            "metric": "projection tokens/s", "value": round(global_batch / (results[best] * 1e-3), 1),
            "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W, "impl_timed": best,
            "ms_per_step": round(results[best], 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {**config_dict(args.workload, kw, global_batch, world, dtype_name), "layers": layers,
                       "step": "24 x (in_proj, out_proj) GEMMs in one CUDA graph, no L2 flush (weights > L2)"},
            "us_per_layer": per,
            "tflops": {k: round(flop / (v * 1e-3) / 1e12, 1) for k, v in results.items()},
            "weight_gbs": {k: round(wbytes / (v * 1e-3) / 1e9, 1) for k, v in results.items()},
            "max_abs_err_vs_float64": err,
            "gpu_launches": K * 2 * layers * (len(results) - 1),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)


# the kernel-level state-update entry point alone (the reference's
# mamba3_mimo_decode_triton, src/kernels/mimo_decode.py:394-457) on the
# throughput sweep's layer shape, and a d_state-32 layer whose fused step
# runs the row kernel (the streamed kernel takes d_state >= 36)
SSM_WORKLOADS = {"ssm_mimo_r4_d1024_b4096"}
WORKLOADS["ssm_mimo_r4_d1024_b4096"] = (dict(d_model=1024, d_state=128, headdim=64, is_mimo=True, mimo_rank=4),
                                        4096, "f32")
WORKLOADS["mimo_r4_d1024_n32_b4096"] = (dict(d_model=1024, d_state=32, headdim=64, is_mimo=True, mimo_rank=4),
                                        4096, "f32")


def ssm_bytes_per_launch(m, batch: int) -> int:
    """Algorithmic HBM bytes of one state-update-only MIMO launch (fp32
    inputs): x (read), the B and C projections (read), the three head
    scalars (read), ssm_state and bx_prev (read + write), y (write) and the
    per-head parameters (D, mimo_x, mimo_o; read once)."""
    H, P, D, R = m.nheads, m.headdim, m.d_state, m.mimo_rank
    return 4 * (2 * batch * H * P + 2 * batch * R * H * D + 3 * batch * H + 4 * batch * H * D + H + 2 * H * R * P)


def run_ssm(args, kw, global_batch, dtype_name, world, rank, local):
    """The kernel-level MIMO state update (mamba3_mimo_decode_triton) on
    precomputed, already rotated B / C projections, each rank on its share
    of the batch: one launch per step, replayed from a one-node graph with
    an L2 flush before every step.  `value` = sequences updated per second;
    `roofline` is the launch's algorithmic bytes over its mean time."""
    from src.kernels.mimo_decode import mamba3_mimo_decode_triton
    from src.models.mamba3 import Mamba3

    h = Harness(world, rank, local)
    dev = h.dev
    batch = shard_rows(global_batch, world)
    m = Mamba3(**kw, device="meta")
    H, P, D, R = m.nheads, m.headdim, m.d_state, m.mimo_rank
    gen = torch.Generator(device=dev).manual_seed(1 + rank)

    def rnd(*shape, scale=1.0):
        return torch.randn(*shape, device=dev, generator=gen) * scale

    x = rnd(batch, H, P)
    Bp, Cp = rnd(batch, R, H, D), rnd(batch, R, H, D)
    DT = torch.rand(batch, H, device=dev, generator=gen) * 0.1 + 1e-3
    ADT = DT * 1e-4
    trap = torch.rand(batch, H, device=dev, generator=gen)
    Dsk = torch.ones(H, device=dev)
    mx, mo = rnd(H, R, P, scale=0.1), rnd(H, R, P, scale=0.1)
    hs, bx = rnd(batch, H, D, scale=0.5), rnd(batch, H, D, scale=0.5)
    K, W = args.steps, args.warmup
    with torch.no_grad():
        g = h.graphed(lambda: mamba3_mimo_decode_triton(x, Bp, Cp, ADT, DT, trap, Dsk, mx, mo, hs, bx), warm=W)
        h.clocks_start()
        h.barrier()
        h.clocks_mark()
        ms = h.timed_loop(lambda i: g.replay(), K)
        h.barrier()
        h.clocks_mark()
    del g
    clocks = h.clocks_stop()
    total = h.max_over_ranks(float(ms.sum()))
    mean = h.max_over_ranks(float(ms.mean()))
    p50 = h.max_over_ranks(float(np.percentile(ms, 50)))
    h.close()
    if rank == 0:
        nbytes = ssm_bytes_per_launch(m, batch)
        peak, peak_kind = hbm_peak()
        achieved = nbytes / (mean * 1e-3) / 1e9
        line = {
            "metric": "state-update sequences/s", "value": round(global_batch * K / (total / 1000.0), 1),
            "unit": "sequences/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total / K, 5),
            "p50_step_ms": round(p50, 5), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {**config_dict(args.workload, kw, global_batch, world, dtype_name),
                       "step": "one mamba3_mimo_decode_triton launch (state update + readout on precomputed "
                               "B / C projections), one-node CUDA graph, L2 flushed before every step"},
            "roofline": {"bound": "hbm", "kernel": "state update (m3_mimo_decode)", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "bytes_per_launch": nbytes, "mean_launch_ms": round(mean, 5),
                         "traffic": profile_traffic(args.workload, "ssm")},
            "gpu_launches": K,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)


def run_prefill(args, kw, global_batch, dtype_name, length, world, rank, local):
    """Prompt prefill of one layer: each rank's share of `global_batch`
    sequences of `length` tokens through Mamba3Decoder.prefill (one in_proj
    GEMM over all tokens, one prefill launch -- m3_mimo_prefill or
    m3_siso_prefill -- and one out_proj GEMM).  A step is one whole prefill.
    `roofline` is the prefill kernel alone: the in_proj rows read once, y
    written once, the state read and written once."""
    from src.kernels.linear import linear
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3

    h = Harness(world, rank, local)
    dev = h.dev
    batch = shard_rows(global_batch, world)
    wdtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    torch.manual_seed(0)
    model = Mamba3(**kw, device=dev, dtype=wdtype)
    with torch.no_grad():
        model.in_proj.weight.normal_(0.0, 0.02)
        model.out_proj.weight.normal_(0.0, 0.02)
    dec = Mamba3Decoder(model, use_triton_full_fused=True)
    state = dec.init_state(batch, device=dev)
    K, W = args.steps, args.warmup
    gen = torch.Generator(device="cpu").manual_seed(1 + rank)
    u_host = torch.randn(batch, length, kw["d_model"], generator=gen).to(wdtype).pin_memory()
    u_dev = u_host.to(dev)
    with torch.no_grad():
        for _ in range(W):
            dec.prefill(u_dev, state)

    h.clocks_start()
    h.barrier()
    h.clocks_mark()
    with torch.no_grad():
        step_ms = h.timed_loop(lambda i: dec.prefill(u_dev, state), K)
    h.barrier()
    h.clocks_mark()
    total_ms = h.max_over_ranks(float(step_ms.sum()))
    p50_all = h.max_over_ranks(float(np.percentile(step_ms, 50)))
    value = global_batch * length * K / (total_ms / 1000.0)

    # the prefill kernel alone, on prepared in_proj rows
    es = 2 if wdtype == torch.bfloat16 else 4
    with torch.no_grad():
        zx = linear(u_dev.reshape(batch * length, -1), model.in_proj.weight)
        y = torch.empty(batch * length, model.d_inner, device=dev, dtype=wdtype)
        launch = dec._fused_launch(state)
        k_ms = h.timed_loop(lambda i: launch.prefill(zx, y, length), min(K, 50))
    k_mean = h.max_over_ranks(float(k_ms.mean()))
    H, D, A = model.nheads, model.d_state, model.num_rope_angles
    R, P = model.mimo_rank, model.headdim
    # in_proj rows read once, y rows written once; h and bx_prev (MIMO: D per
    # head, SISO: P x D per head) and the angles read once and written once;
    # dt_bias, D, the norm weights, the B/C biases (and the MIMO projections)
    if model.is_mimo:
        state_elems, par_elems = H * D, 2 * H + 2 * D + 2 * H * R * D + 2 * H * R * P
    else:
        state_elems, par_elems = H * P * D, 2 * H + 2 * D + 2 * H * D
    nbytes = (batch * length * (model.d_in_proj + model.d_inner) * es + 16 * batch * state_elems
              + 8 * batch * H * A + es * par_elems)
    peak, peak_kind = hbm_peak()
    achieved = nbytes / (k_mean * 1e-3) / 1e9

    # end to end through the public API: the prompt from pinned host memory,
    # every output row back to the host
    out_host = torch.empty(batch, length, kw["d_model"], dtype=wdtype).pin_memory()
    u_stage = torch.empty_like(u_dev)

    def e2e_step(i):
        u_stage.copy_(u_host, non_blocking=True)
        out, _ = dec.prefill(u_stage, state)
        out_host.copy_(out, non_blocking=True)
        h.stream.synchronize()

    h.barrier()
    with torch.no_grad():
        e2e_ms = h.timed_loop(e2e_step, max(min(K, 50), 1), pre_sync=True)
    h.barrier()
    e2e = e2e_summary(h, e2e_ms, global_batch * length, u_stage.numel() * es, out_host.numel() * es,
                      "pinned prompt copied in, prefill, every output row copied to pinned host memory, stream sync")
    clocks = h.clocks_stop()
    cpu = None
    if rank == 0 and world == 1:
        cpu, _, _ = cpu_baseline(kw, global_batch, dtype_name, 1, budget_s=args.cpu_budget)
        cpu["sample"] += " (a prefill on the host is one decode step per prompt token)"
    h.close()
    if rank == 0:
        cfg = config_dict(args.workload, kw, global_batch, world, dtype_name)
        entry = "m3_mimo_prefill" if model.is_mimo else "m3_siso_prefill"
        cfg.update({"prompt_tokens": length, "step": "Mamba3Decoder.prefill of batch x prompt tokens: in_proj "
                    f"over all tokens, one {entry} launch, out_proj"})
        line = {
            "metric": "prefill tokens/s", "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total_ms / K, 5),
            "p50_step_ms": round(p50_all, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": dtype_name, "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": (f"{entry} (streamed kernel, sequence form)" if model.is_mimo else
                                                   f"{entry} (state tile in registers)"),
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes,
                         "mean_launch_ms": round(k_mean, 5), "traffic": profile_traffic(args.workload, "prefill")},
            "e2e": e2e,
            "gpu_launches": K,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def run_layer(args, kw, global_batch, dtype_name, world, rank, local):
    """One layer decoded through Mamba3Decoder's captured graph, each rank
    decoding its share of the global batch."""
    from src.kernels.linear import linear, uses_small_m_kernel
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3

    h = Harness(world, rank, local)
    dev = h.dev
    batch = shard_rows(global_batch, world)
    wdtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    torch.manual_seed(0)
    model = Mamba3(**kw, device=dev, dtype=wdtype)
    with torch.no_grad():
        model.in_proj.weight.normal_(0.0, 0.02)
        model.out_proj.weight.normal_(0.0, 0.02)
    gen = torch.Generator(device="cpu").manual_seed(1 + rank)
    K, W = args.steps, args.warmup
    n_inputs = 64
    u_host = torch.randn(n_inputs, batch, model.d_model, generator=gen).to(wdtype).pin_memory()
    u_dev = u_host.to(dev)
    dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
    state = dec.init_state(batch, device=dev)
    dec.warmup_cuda_graph(state, n_warmup=3)
    with torch.no_grad():
        for i in range(W):
            dec.step(u_dev[i % n_inputs], state)

    h.clocks_start()
    h.barrier()
    h.clocks_mark()
    with torch.no_grad():
        step_ms = h.timed_loop(lambda i: dec.step(u_dev[i % n_inputs], state), K)
    h.barrier()
    h.clocks_mark()
    total_ms = h.max_over_ranks(float(step_ms.sum()))
    p50 = h.max_over_ranks(float(np.percentile(step_ms, 50)))
    p99 = h.max_over_ranks(float(np.percentile(step_ms, 99)))
    value = global_batch * K / (total_ms / 1000.0)
    # our kernels per step: the single-launch step kernel, or the fused decode
    # kernel plus both projections when they run on the library's small-batch
    # GEMM (otherwise cuBLAS)
    single = dec._step_cache is not None and dec._step_cache[1] is not None
    own_gemms = int(uses_small_m_kernel(u_dev[0], model.in_proj.weight)) + int(
        uses_small_m_kernel(torch.empty(batch, model.d_inner, device=dev, dtype=wdtype), model.out_proj.weight))
    gpu_launches = K if single else K * (1 + own_gemms)

    # the fused kernel alone (roofline) and the two GEMMs, each replayed from
    # its own graph so host dispatch stays out of the device times
    with torch.no_grad():
        zx = linear(u_dev[0], model.in_proj.weight)
        y = torch.zeros(batch, model.d_inner, device=dev, dtype=wdtype)
        launch = dec._fused_launch(state)
        g_fused = h.graphed(lambda: launch.run(zx, y))
        g_in = h.graphed(lambda: linear(u_dev[0], model.in_proj.weight))
        g_out = h.graphed(lambda: linear(y, model.out_proj.weight))
        f_ms = h.timed_loop(lambda i: g_fused.replay(), K)
        gi_ms = h.timed_loop(lambda i: g_in.replay(), min(K, 500))
        go_ms = h.timed_loop(lambda i: g_out.replay(), min(K, 500))
        # the three-launch step (in_proj, fused kernel, out_proj) on its own state
        dec3 = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True, use_single_launch=False)
        st3 = dec3.init_state(batch, device=dev)
        dec3.warmup_cuda_graph(st3, n_warmup=3)
        t3_ms = h.timed_loop(lambda i: dec3.step(u_dev[i % n_inputs], st3), min(K, 500))
        dec3._cuda_graph = None
        if single:
            step_launch = dec._step_cache[1]
            out_static = torch.empty(batch, model.d_model, device=dev, dtype=wdtype)
            g_step = h.graphed(lambda: step_launch.run(u_dev[0], out_static))
            s_ms = h.timed_loop(lambda i: g_step.replay(), K)
            del g_step
    del g_fused, g_in, g_out
    es = 2 if wdtype == torch.bfloat16 else 4
    f_mean = h.max_over_ranks(float(f_ms.mean()))
    if single:
        kernel_name = "single-launch decode step (m3_mimo_step)"
        k_mean = h.max_over_ranks(float(s_ms.mean()))
        nbytes = step_bytes_per_launch(model, batch, es)
    else:
        kernel_name = "fused decode (m3_mimo_full_fused / m3_siso_full_fused)"
        k_mean = f_mean
        nbytes = fused_bytes_per_launch(model, batch, es, es)
    peak, peak_kind = hbm_peak()
    achieved = nbytes / (k_mean * 1e-3) / 1e9
    gi_mean = h.max_over_ranks(float(gi_ms.mean()))
    go_mean = h.max_over_ranks(float(go_ms.mean()))
    t3_mean = h.max_over_ranks(float(t3_ms.mean()))

    # end to end through the public API: Mamba3Decoder.step_host copies the
    # pinned input into the graph's input and returns once the host holds the
    # output rows (written by the single-launch kernel straight into pinned
    # host memory where it serves the layer, else copied back)
    h.barrier()
    with torch.no_grad():
        for i in range(W):  # the first call sets up (and captures the host-output graph)
            dec.step_host(u_host[i % n_inputs])
        torch.cuda.synchronize(dev)
        e2e_ms = h.timed_loop(lambda i: dec.step_host(u_host[i % n_inputs]), K, pre_sync=True)
    h.barrier()
    path = ("pinned input copied in; the single-launch kernel stores the output rows into pinned host memory; "
            "device synchronise" if dec._host_graph is not None else
            "pinned input copied in; graph replay; output copied to pinned host memory; device synchronise")
    e2e = e2e_summary(h, e2e_ms, global_batch, batch * model.d_model * es, batch * model.d_model * es, path)
    clocks = h.clocks_stop()
    cpu = None
    if rank == 0 and world == 1:
        cpu, _, _ = cpu_baseline(kw, global_batch, dtype_name, 1, budget_s=args.cpu_budget)
    h.close()
    if rank == 0:
        published = PUBLISHED.get(args.workload)
        line = {
            "metric": "decode tokens/s", "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total_ms / K, 5),
            "p50_step_ms": round(p50, 5), "p99_step_ms": round(p99, 5),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": round(value / published, 3) if published and world == 1 else None,
            "dtype": dtype_name, "data": "synthetic",
            "config": config_dict(args.workload, kw, global_batch, world, dtype_name),
            "roofline": {"bound": "hbm", "kernel": kernel_name,
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes,
                         "mean_launch_ms": round(k_mean, 5),
                         "traffic": profile_traffic(args.workload, "step" if single else "fused")},
            "kernels_ms": {"decode_step": round(k_mean, 5) if single else None,
                           "three_launch_step": round(t3_mean, 5),
                           "in_proj_gemm": round(gi_mean, 5),
                           "fused_decode": round(f_mean, 5),
                           "out_proj_gemm": round(go_mean, 5)},
            "e2e": e2e,
            "gpu_launches": gpu_launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    dec._cuda_graph = None


def run_sweep(args, kw, dtype_name, world, rank, local):
    """The throughput sweep of one layer (the reference's
    benchmarks/run_bench_extended.py --batch-sizes / --mimo-rank): for every
    MIMO rank and batch size, the workload's layer with that rank decoded
    through Mamba3Decoder's captured graph (full-fused path), L2 flushed
    before every timed step.  One JSON line: per point the step's mean and
    p50 / p99 ms and tokens/s (batch x steps / time).  One GPU."""
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3

    if world != 1:
        if rank == 0:
            print(json.dumps({"metric": "decode tokens/s sweep", "unavailable": "the sweep runs on one GPU"}))
        return
    h = Harness(world, rank, local)
    dev = h.dev
    wdtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    ranks = [int(r) for r in args.mimo_ranks.split(",")]
    batches = [int(b) for b in args.batch_sizes.split(",")]
    K, W = args.steps, args.warmup
    points = []
    h.clocks_start()
    h.clocks_mark()
    for R in ranks:
        lkw = dict(kw, is_mimo=True, mimo_rank=R)
        torch.manual_seed(0)
        model = Mamba3(**lkw, device=dev, dtype=wdtype)
        with torch.no_grad():
            model.in_proj.weight.normal_(0.0, 0.02)
            model.out_proj.weight.normal_(0.0, 0.02)
        for B in batches:
            gen = torch.Generator(device="cpu").manual_seed(1)
            u_dev = torch.randn(8, B, model.d_model, generator=gen).to(wdtype).to(dev)
            dec = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True)
            state = dec.init_state(B, device=dev)
            with torch.no_grad():
                dec.warmup_cuda_graph(state, n_warmup=3)
                for i in range(W):
                    dec.step(u_dev[i % 8], state)
                ms = h.timed_loop(lambda i: dec.step(u_dev[i % 8], state), K)
            single = dec._step_cache is not None and dec._step_cache[1] is not None
            points.append({"mimo_rank": R, "batch": B, "ms_per_step": round(float(ms.mean()), 5),
                           "p50_ms": round(float(np.percentile(ms, 50)), 5),
                           "p99_ms": round(float(np.percentile(ms, 99)), 5),
                           "tokens_per_s": round(B * K / (float(ms.sum()) / 1000.0), 1),
                           "path": "single launch" if single else "in_proj + fused kernel + out_proj"})
            dec._cuda_graph = None
            del dec, state
            torch.cuda.synchronize(dev)
    h.clocks_mark()
    clocks = h.clocks_stop()
    h.close()
    if rank == 0:
        print(json.dumps({
            "metric": "decode tokens/s sweep", "unit": "tokens/s", "n_gpus": 1, "steps": K, "warmup": W,
            "higher_is_better": True, "dtype": dtype_name, "data": "synthetic",
            "config": {**{k: v for k, v in kw.items() if k != "mimo_rank"}, "weights": dtype_name, "state": "f32",
                       "l2": "flushed (256 MiB write) before every timed step; per-step CUDA events",
                       "step": "CUDA-graph replay of Mamba3Decoder.step (full-fused path)"},
            "points": points, "clocks": clocks}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of reference CPU timing")
    ap.add_argument("--no-fused-rooflines", dest="fused_rooflines", action="store_false",
                    help="skip the extra fused-kernel rooflines of the default run")
    ap.add_argument("--sweep", action="store_true",
                    help="throughput sweep of the workload's layer over --batch-sizes and --mimo-ranks (one GPU)")
    ap.add_argument("--batch-sizes", default="1,8,32,128,512,1024,4096")
    ap.add_argument("--mimo-ranks", default="1,2,4,8")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    kw, global_batch, dtype_name = WORKLOADS[args.workload]

    if args.sweep:
        if args.impl == "reference" or args.workload in STACKS or args.workload in PREFILLS or \
                args.workload in PROJECTIONS or args.workload in SSM_WORKLOADS:
            raise SystemExit("--sweep takes a single-layer workload and the native implementation")
        run_sweep(args, kw, dtype_name, world, rank, local)
    elif args.impl == "reference":
        run_reference(args, kw, global_batch, dtype_name, rank)
    elif args.workload in STACKS:
        run_stack(args, kw, global_batch, dtype_name, STACKS[args.workload], world, rank, local)
    elif args.workload in PREFILLS:
        run_prefill(args, kw, global_batch, dtype_name, PREFILLS[args.workload], world, rank, local)
    elif args.workload in PROJECTIONS:
        run_projections(args, kw, global_batch, dtype_name, PROJECTIONS[args.workload], world, rank, local)
    elif args.workload in SSM_WORKLOADS:
        run_ssm(args, kw, global_batch, dtype_name, world, rank, local)
    else:
        run_layer(args, kw, global_batch, dtype_name, world, rank, local)


if __name__ == "__main__":
    main()
