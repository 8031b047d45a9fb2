"""Benchmark of the Mamba-3 single-token decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {native,reference}]
                    [--workload NAME]

Default workload: one MIMO rank-4 Mamba-3 layer, d_model=256, d_inner=512,
headdim=32 (16 heads), d_state=64, fp32 weights and state, 128 sequences per
GPU (the reference's MIMO R4 d256 decode benchmark at its largest batch).
Weights: torch.manual_seed(0), in_proj / out_proj ~ N(0, 0.02), the other
parameters per the layer's own init; inputs u ~ N(0, 1) from seed 1;
synthetic data, zero initial state.

A step is one decode step of the whole batch through the captured CUDA graph
(in_proj GEMM -> fused decode kernel -> out_proj GEMM; small fp32 batches run
the library's small-batch GEMM, larger ones cuBLAS).  Between timed steps
L2 is flushed by writing a 256 MiB buffer; each step is timed with its own
CUDA event pair on the launching stream (the flush is outside the pair).
``value`` = tokens / (sum of step times), max over ranks, all ranks' tokens.

``e2e`` times the public API end to end: per step, the pinned host input
is copied to the device, ``Mamba3Decoder.step`` replays the graph on it,
the output is copied back to pinned host memory and the stream is
synchronised so the host holds the result; the event pair brackets all of
it, after an L2 flush that has completed.

``roofline`` is for the fused decode kernel: its algorithmic HBM bytes per
launch over its mean duration in a K-launch event-timed loop with the same
L2 flush (the kernel replayed from a one-node CUDA graph, so host dispatch
stays out of the timing), against the measured HBM copy bandwidth.
``kernels_ms`` times the step's three kernels the same way.  ``cpu_baseline`` times the numpy oracle (a restatement of the
reference's PyTorch decode) on the host cores for a bounded sample.

Multi-GPU (torchrun): every rank decodes its own 128 sequences with a full
weight replica and its own graph; no collective runs on the decode path
(NCCL is used for the barrier and the max-over-ranks timing only).
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

# name -> (layer kwargs, batch per GPU, weight dtype)
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
DEFAULT_WORKLOAD = "mimo_r4_d256_b128"
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


def config_dict(workload, kw, batch, world, dtype_name, reference=False):
    published = PUBLISHED.get(workload)
    if reference:
        par, l2, step = ("rank 0 only (host cores)", "n/a (CPU)",
                         "oracle decode step (numpy restatement of the reference PyTorch decode)")
    else:
        par = f"batch-sharded x{world}, no collective on the decode path"
        l2 = "flushed (256 MiB write) before every timed step; per-step CUDA events"
        step = ("CUDA-graph replay of Mamba3Decoder.step: one single-launch kernel (in_proj, fused update, "
                "out_proj) for MIMO layers it takes, else in_proj GEMM + fused decode kernel + out_proj GEMM")
    return {"workload": workload, "batch_per_gpu": batch, "global_batch": batch * world,
            **kw, "weights": dtype_name, "state": "f32", "parallelism": par, "l2": l2, "step": step,
            "baseline": ("A100 full-fused+graph P50 0.295 ms at B=128 (reference README.md:229)"
                         if published else None)}


def run_reference(args, kw, batch, dtype_name, rank):
    """--impl reference: the oracle port of the reference's CPU decode (for a
    stack: one layer's rate divided by the number of layers)."""
    if rank != 0:
        return
    layers = STACKS.get(args.workload, 1)
    steps = args.steps if layers == 1 else min(args.steps, 3)
    cpu_oracle_rate(kw, batch, dtype_name, steps=max(min(args.warmup, steps), 1), warmup=0)  # warm-up
    rate, n, cores = cpu_oracle_rate(kw, batch, dtype_name, steps=steps, warmup=0)
    rate /= layers
    ms = 1000.0 * batch / rate
    cfg = config_dict(args.workload, kw, batch, 1, dtype_name, reference=True)
    metric, sample = "decode tokens/s", f"{n} oracle decode steps of {batch} sequences (numpy, host cores)"
    if args.workload in PREFILLS:
        # a prefill on the host is one decode step per prompt token, so its
        # tokens/s is the decode rate; ms_per_step stays one batch of tokens
        metric = "prefill tokens/s"
        cfg["prompt_tokens"] = PREFILLS[args.workload]
        sample += " (a prefill on the host steps every prompt token)"
    line = {
        "metric": metric, "value": round(rate, 1), "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": round(rate, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(rate, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_stack(args, kw, batch, dtype_name, layers, world, rank, local):
    """A residual stack of `layers` MIMO blocks decoded token by token through
    Mamba3StackDecoder, the whole stack step in one CUDA graph.  Same timing
    rules as the single-layer path: L2 flushed and a CUDA event pair around
    every timed step, max over ranks.  `roofline` is the library's fused
    decode kernel of one layer (the projections are cuBLAS bf16 GEMMs, whose
    rate is reported beside it)."""
    import datetime

    import torch.distributed as dist

    from src.kernels.linear import linear
    from src.models.lm import Mamba3LMDecoder
    from src.models.mamba3 import MambaBlock, MambaConfig, MambaLMHeadModel
    from src.models.stack import Mamba3StackDecoder

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
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
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        dec.warmup_cuda_graph(states, n_warmup=2)
        for i in range(W):
            dec.step(u_dev[i % n_inputs], states)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed_loop(fn, n, pre_sync=False):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            flush.zero_()
            if pre_sync:
                stream.synchronize()
            else:
                torch.cuda._sleep(20000)
            ev[i][0].record(stream)
            fn(i)
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        return np.array([a.elapsed_time(b) for a, b in ev])

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    try:
        gpus = [int(x) for x in vis.split(",")][:world] if vis else list(range(world))
    except ValueError:
        gpus = list(range(world))
    sampler = ClockSampler(gpus) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.2)
    barrier()
    if sampler:
        sampler.mark()
    with torch.no_grad():
        step_ms = timed_loop(lambda i: dec.step(u_dev[i % n_inputs], states), K)
    barrier()
    if sampler:
        sampler.mark()
    total_ms = max_over_ranks(float(step_ms.sum()))
    value = world * batch * K / (total_ms / 1000.0)

    # one layer's fused kernel (roofline) and its two projections
    es = 2 if wdtype == torch.bfloat16 else 4
    layer = dec.layers[0]
    xn = torch.randn(batch, kw["d_model"], device=dev).to(wdtype)
    with torch.no_grad():
        zx = linear(xn, model.in_proj.weight)
        y = torch.zeros(batch, model.d_inner, device=dev, dtype=wdtype)
        launch = layer._fused_launch(states[0])
        graphs = []
        for fn in (lambda: launch.run(zx, y), lambda: linear(xn, model.in_proj.weight),
                   lambda: linear(y, model.out_proj.weight)):
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for _ in range(2):
                    fn()
            stream.wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            graphs.append(g)
        n_k = min(K, 200)
        f_ms, gi_ms, go_ms = (timed_loop(lambda i, g=g: g.replay(), n_k) for g in graphs)
    del graphs
    k_mean = max_over_ranks(float(f_ms.mean()))
    nbytes = fused_bytes_per_launch(model, batch, es, es)
    peak, peak_kind = hbm_peak()
    achieved = nbytes / (k_mean * 1e-3) / 1e9
    gemm_flop = 2.0 * batch * model.d_model * (model.d_in_proj + model.d_inner)
    gemm_ms = float(gi_ms.mean() + go_ms.mean())

    # end to end through the public API: pinned input in, output back to the host
    out_host = torch.empty(*out_shape, dtype=wdtype).pin_memory()
    u_stage = torch.empty(u_host.shape[1:], device=dev, dtype=u_host.dtype)

    def e2e_step(i):
        u_stage.copy_(u_host[i % n_inputs], non_blocking=True)
        out, _ = dec.step(u_stage, states)
        out_host.copy_(out, non_blocking=True)
        stream.synchronize()

    barrier()
    with torch.no_grad():
        e2e_ms = timed_loop(e2e_step, min(K, 200), pre_sync=True)
    barrier()
    e2e_total = max_over_ranks(float(e2e_ms.sum()))
    e2e_value = world * batch * len(e2e_ms) / (e2e_total / 1000.0)
    clocks = sampler.stop() if sampler else None

    cpu = None
    if rank == 0 and world == 1:
        rate, n, cores = cpu_oracle_rate(kw, batch, dtype_name, budget_s=args.cpu_budget)
        cpu = {"value": round(rate / layers, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{n} oracle decode steps of one layer x {batch} sequences, rate divided by "
                         f"{layers} layers (numpy float32 restatement with bf16 rounding"
                         + ("; embedding and LM head not included" if vocab is not None else "") + ")"}
    # every rank takes part in every collective, so they all run before the
    # rank-0-only report
    p50_all = max_over_ranks(float(np.percentile(step_ms, 50)))
    if world > 1:
        dist.barrier()
    if rank == 0:
        cfg = config_dict(args.workload, kw, batch, world, dtype_name)
        cfg.update({"layers": layers, "step": "CUDA-graph replay of Mamba3StackDecoder.step: per layer "
                    "in_proj (cuBLAS bf16) + fused decode kernel + out_proj (cuBLAS bf16), residual add + "
                    "RMSNorm kernel between blocks"})
        if vocab is not None:
            cfg.update({"model": "MambaLMHeadModel", "vocab_size": vocab, "padded_vocab": lm.vocab_size,
                        "step": "CUDA-graph replay of Mamba3LMDecoder.step: token ids -> embedding, per layer "
                        "in_proj (cuBLAS bf16) + fused decode kernel + out_proj (cuBLAS bf16) + residual add "
                        "and RMSNorm kernel, final norm, LM head (cuBLAS bf16) -> logits"})
        line = {
            "metric": "decode tokens/s", "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total_ms / K, 5),
            "p50_step_ms": round(p50_all, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": dtype_name, "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": "fused decode (m3_mimo_full_fused), one layer",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes,
                         "mean_launch_ms": round(k_mean, 5),
                         "traffic": profile_traffic(LM_STACK_PROFILE.get(args.workload, args.workload), "fused")},
            "kernels_ms": {"fused_decode_per_layer": round(k_mean, 5),
                           "in_proj_gemm_per_layer": round(float(gi_ms.mean()), 5),
                           "out_proj_gemm_per_layer": round(float(go_ms.mean()), 5),
                           "projection_tflops": round(gemm_flop / (gemm_ms * 1e-3) / 1e12, 1)},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": u_stage.numel() * u_stage.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size(),
                    "ms_per_step": round(e2e_total / len(e2e_ms), 5)},
            "gpu_launches": K * (2 * layers + 1),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    dec._graph = None
    if world > 1:
        dist.destroy_process_group()


def run_prefill(args, kw, batch, dtype_name, length, world, rank, local):
    """Prompt prefill of one layer: `batch` sequences of `length` tokens
    through Mamba3Decoder.prefill (one in_proj GEMM over all tokens, one
    prefill launch -- m3_mimo_prefill or m3_siso_prefill -- and one out_proj
    GEMM).  A
    step is one whole prefill; L2 flushed and a CUDA event pair around every
    timed step, max over ranks.  `roofline` is the prefill kernel alone: the
    in_proj rows read once, y written once, the state read and written once."""
    import datetime

    import torch.distributed as dist

    from src.kernels.linear import linear
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
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
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(W):
            dec.prefill(u_dev, state)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed_loop(fn, n, pre_sync=False):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            flush.zero_()
            if pre_sync:
                stream.synchronize()
            else:
                torch.cuda._sleep(20000)
            ev[i][0].record(stream)
            fn(i)
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        return np.array([a.elapsed_time(b) for a, b in ev])

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    try:
        gpus = [int(x) for x in vis.split(",")][:world] if vis else list(range(world))
    except ValueError:
        gpus = list(range(world))
    sampler = ClockSampler(gpus) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.2)
    barrier()
    if sampler:
        sampler.mark()
    with torch.no_grad():
        step_ms = timed_loop(lambda i: dec.prefill(u_dev, state), K)
    barrier()
    if sampler:
        sampler.mark()
    total_ms = max_over_ranks(float(step_ms.sum()))
    p50_all = max_over_ranks(float(np.percentile(step_ms, 50)))
    value = world * batch * length * K / (total_ms / 1000.0)

    # the prefill kernel alone, on prepared in_proj rows
    es = 2 if wdtype == torch.bfloat16 else 4
    with torch.no_grad():
        zx = linear(u_dev.reshape(batch * length, -1), model.in_proj.weight)
        y = torch.empty(batch * length, model.d_inner, device=dev, dtype=wdtype)
        launch = dec._fused_launch(state)
        k_ms = timed_loop(lambda i: launch.prefill(zx, y, length), min(K, 50))
    k_mean = max_over_ranks(float(k_ms.mean()))
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
        stream.synchronize()

    barrier()
    with torch.no_grad():
        e2e_ms = timed_loop(e2e_step, min(K, 50), pre_sync=True)
    barrier()
    e2e_total = max_over_ranks(float(e2e_ms.sum()))
    e2e_value = world * batch * length * len(e2e_ms) / (e2e_total / 1000.0)
    clocks = sampler.stop() if sampler else None
    cpu = None
    if rank == 0 and world == 1:
        rate, n, cores = cpu_oracle_rate(kw, batch, dtype_name, budget_s=args.cpu_budget)
        cpu = {"value": round(rate, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{n} oracle decode steps of {batch} sequences (a prefill on the host is one decode "
                         f"step per prompt token; numpy float32 restatement with bf16 rounding)"}
    if world > 1:
        dist.barrier()
    if rank == 0:
        cfg = config_dict(args.workload, kw, batch, world, dtype_name)
        entry = "m3_mimo_prefill" if model.is_mimo else "m3_siso_prefill"
        cfg.update({"prompt_tokens": length, "step": "Mamba3Decoder.prefill of batch x prompt tokens: in_proj "
                    f"(cuBLAS bf16) over all tokens, one {entry} launch, out_proj (cuBLAS bf16)"})
        line = {
            "metric": "prefill tokens/s", "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total_ms / K, 5),
            "p50_step_ms": round(p50_all, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype_name, "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": (f"{entry} (streamed kernel, sequence form)" if model.is_mimo else
                                                   f"{entry} (state tile in registers)"),
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes,
                         "mean_launch_ms": round(k_mean, 5), "traffic": profile_traffic(args.workload, "prefill")},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": u_stage.numel() * es, "d2h_bytes_per_step": out_host.numel() * es,
                    "ms_per_step": round(e2e_total / len(e2e_ms), 5)},
            "gpu_launches": K,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of oracle CPU timing")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    kw, batch, dtype_name = WORKLOADS[args.workload]

    if args.impl == "reference":
        run_reference(args, kw, batch, dtype_name, rank)
        return
    if args.workload in STACKS:
        run_stack(args, kw, batch, dtype_name, STACKS[args.workload], world, rank, local)
        return
    if args.workload in PREFILLS:
        run_prefill(args, kw, batch, dtype_name, PREFILLS[args.workload], world, rank, local)
        return

    import datetime

    import torch.distributed as dist

    from src.kernels.linear import linear
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
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
    flush = torch.empty(FLUSH_BYTES // 4, device=dev, dtype=torch.float32)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed_loop(fn, n, pre_sync=False):
        """n iterations of fn, each bracketed by its own event pair after an
        L2 flush; returns per-iteration milliseconds."""
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            flush.zero_()
            if pre_sync:
                stream.synchronize()
            else:
                torch.cuda._sleep(20000)  # keep the GPU busy while the host enqueues the step
            ev[i][0].record(stream)
            fn(i)
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        return np.array([a.elapsed_time(b) for a, b in ev])

    # ---- warm-up (graph replays) ----
    with torch.no_grad():
        for i in range(W):
            dec.step(u_dev[i % n_inputs], state)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    try:
        gpus = [int(x) for x in vis.split(",")][:world] if vis else list(range(world))
    except ValueError:
        gpus = list(range(world))
    sampler = ClockSampler(gpus) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.2)

    # ---- timed region: K decode steps ----
    barrier()
    if sampler:
        sampler.mark()
    with torch.no_grad():
        step_ms = timed_loop(lambda i: dec.step(u_dev[i % n_inputs], state), K)
    barrier()
    if sampler:
        sampler.mark()
    total_ms = max_over_ranks(float(step_ms.sum()))
    p50 = max_over_ranks(float(np.percentile(step_ms, 50)))
    p99 = max_over_ranks(float(np.percentile(step_ms, 99)))
    value = world * batch * K / (total_ms / 1000.0)
    # our kernels per step: the single-launch step kernel, or the fused decode
    # kernel plus both projections when they run on the library's small-batch
    # GEMM (otherwise cuBLAS)
    single = dec._step_cache is not None and dec._step_cache[1] is not None
    from src.kernels.linear import uses_small_m_kernel
    own_gemms = int(uses_small_m_kernel(u_dev[0], model.in_proj.weight)) + int(
        uses_small_m_kernel(torch.empty(batch, model.d_inner, device=dev, dtype=wdtype), model.out_proj.weight))
    gpu_launches = K if single else K * (1 + own_gemms)

    # ---- fused kernel alone (roofline) and the two GEMMs, same flush ----
    # Each component is captured in its own CUDA graph and replayed between
    # the events, so host-side dispatch cost stays out of the device times.
    zx = linear(u_dev[0], model.in_proj.weight)
    y = torch.zeros(batch, model.d_inner, device=dev, dtype=wdtype)
    launch = dec._fused_launch(state)

    def graphed(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        stream.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    es = 2 if wdtype == torch.bfloat16 else 4
    with torch.no_grad():
        g_fused = graphed(lambda: launch.run(zx, y))
        g_in = graphed(lambda: linear(u_dev[0], model.in_proj.weight))
        g_out = graphed(lambda: linear(y, model.out_proj.weight))
        f_ms = timed_loop(lambda i: g_fused.replay(), K)
        gi_ms = timed_loop(lambda i: g_in.replay(), min(K, 500))
        go_ms = timed_loop(lambda i: g_out.replay(), min(K, 500))
        # the three-launch step (in_proj, fused kernel, out_proj) on its own state
        dec3 = Mamba3Decoder(model, use_triton_full_fused=True, use_cuda_graph=True, use_single_launch=False)
        st3 = dec3.init_state(batch, device=dev)
        dec3.warmup_cuda_graph(st3, n_warmup=3)
        t3_ms = timed_loop(lambda i: dec3.step(u_dev[i % n_inputs], st3), min(K, 500))
        dec3._cuda_graph = None
        if single:
            step_launch = dec._step_cache[1]
            out_static = torch.empty(batch, model.d_model, device=dev, dtype=wdtype)
            g_step = graphed(lambda: step_launch.run(u_dev[0], out_static))
            s_ms = timed_loop(lambda i: g_step.replay(), K)
            del g_step
    del g_fused, g_in, g_out
    f_mean = max_over_ranks(float(f_ms.mean()))
    if single:
        kernel_name = "single-launch decode step (m3_mimo_step)"
        k_mean = max_over_ranks(float(s_ms.mean()))
        nbytes = step_bytes_per_launch(model, batch, es)
    else:
        kernel_name = "fused decode (m3_mimo_full_fused / m3_siso_full_fused)"
        k_mean = f_mean
        nbytes = fused_bytes_per_launch(model, batch, es, es)
    peak, peak_kind = hbm_peak()
    achieved = nbytes / (k_mean * 1e-3) / 1e9

    # ---- end to end through the public API (pinned host in/out) ----
    # Mamba3Decoder.step_host: the pinned input is copied into the graph's
    # input, the step writes its output rows to pinned host memory (directly
    # from the single-launch kernel, else by a copy), and the call returns
    # once the host can read them
    def e2e_step(i):
        dec.step_host(u_host[i % n_inputs])

    barrier()
    with torch.no_grad():
        e2e_ms = timed_loop(e2e_step, K, pre_sync=True)
    barrier()
    e2e_total = max_over_ranks(float(e2e_ms.sum()))
    e2e_value = world * batch * K / (e2e_total / 1000.0)
    clocks = sampler.stop() if sampler else None

    cpu = None
    if rank == 0 and world == 1:
        rate, n, cores = cpu_oracle_rate(kw, batch, dtype_name, budget_s=args.cpu_budget)
        cpu = {"value": round(rate, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{n} oracle decode steps of {batch} sequences (numpy float32 restatement "
                         f"of the reference PyTorch decode; BLAS threads = host cores)"}

    # every rank takes part in every collective, so they all run before the
    # rank-0-only report
    t3_all = max_over_ranks(float(t3_ms.mean()))
    if world > 1:
        dist.barrier()
    if rank == 0:
        published = PUBLISHED.get(args.workload)
        line = {
            "metric": "decode tokens/s", "value": round(value, 1), "unit": "tokens/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(total_ms / K, 5),
            "p50_step_ms": round(p50, 5), "p99_step_ms": round(p99, 5),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / (world * published), 3) if published else None,
            "dtype": dtype_name, "data": "synthetic",
            "config": config_dict(args.workload, kw, batch, world, dtype_name),
            "roofline": {"bound": "hbm", "kernel": kernel_name,
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "bytes_per_launch": nbytes,
                         "mean_launch_ms": round(k_mean, 5),
                         "traffic": profile_traffic(args.workload, "step" if single else "fused")},
            "kernels_ms": {"decode_step": round(k_mean, 5) if single else None,
                           "three_launch_step": round(t3_all, 5),
                           "in_proj_gemm": round(float(gi_ms.mean()), 5),
                           "fused_decode": round(f_mean, 5),
                           "out_proj_gemm": round(float(go_ms.mean()), 5)},
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": batch * model.d_model * u_host.element_size(),
                    "d2h_bytes_per_step": batch * model.d_model * u_host.element_size(),
                    "ms_per_step": round(e2e_total / K, 5)},
            "gpu_launches": gpu_launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    dec._cuda_graph = None
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
