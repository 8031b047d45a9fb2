"""Time the reference's own PyTorch CPU decode on the host cores.

    python oracle/reference_cpu.py --layer '{"d_model": 2048, ...}' --dtype bf16 \
        --batch 256 --layers 24 [--steps N] [--budget SECONDS] [--warmup W] [--threads T]

Runs in its own interpreter because the reference and this package both
name their top-level package ``src``: ``baseline/_ref`` (staged by
``oracle/stage_reference.py``, checked against its manifest) goes first on
``sys.path`` and nothing of this package is imported.  Baseline
infrastructure only -- ``bench.py``'s CPU legs run it.

What is timed is the reference's public decode path, unmodified:
``Mamba3Decoder(model, use_triton=False).step`` (src/models/inference.py:
271-282 -> src/models/mamba3.py:306-353).  With ``--layers`` > 1 the layers
are the reference's ``MambaBlock`` (src/models/mamba3.py:412-421), composed
the way its ``forward`` composes them, ``x <- x + mixer_step(norm(x))``
(the reference has no stack decode API).  Weights: ``torch.manual_seed(0)``,
the reference's own init, then in_proj / out_proj ~ N(0, 0.02); inputs
u ~ N(0, 1) from seed 1, cast to the weight dtype (a bf16 model needs bf16
inputs); zero initial state.  With ``--ssm`` what is timed is the
reference's state-update-only MIMO decode, ``mamba3_mimo_decode_ref``
(src/kernels/utils.py:109-148), on random fp32 inputs of the layer's shapes.
Prints one JSON line: tokens/s (batch x timed steps / their wall time), ms
per step, p50, steps timed, threads.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layer", required=True, help="Mamba3 keyword arguments as JSON")
    ap.add_argument("--dtype", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--batch", type=int, required=True)
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="at most this many timed steps (0: no count limit)")
    ap.add_argument("--budget", type=float, default=10.0, help="stop timing after this many seconds")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--threads", type=int, default=0, help="torch threads (0: every host core)")
    ap.add_argument("--ssm", action="store_true", help="time the state-update-only MIMO decode")
    args = ap.parse_args()

    sys.dont_write_bytecode = True
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from stage_reference import verify

    why = verify(REF)
    if why:
        print(json.dumps({"unavailable": why}))
        return 0
    sys.path.insert(0, REF)
    import numpy as np
    import torch

    from src.models.inference import Mamba3Decoder  # the reference's
    from src.models.mamba3 import Mamba3, MambaBlock

    threads = args.threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    kw = json.loads(args.layer)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    torch.manual_seed(0)
    with torch.no_grad():
        if args.layers == 1:
            blocks = [None]
            mixers = [Mamba3(**kw, dtype=dtype)]
        else:
            mkw = {k: v for k, v in kw.items() if k != "d_model"}
            blocks = [MambaBlock(kw["d_model"], mkw, dtype=dtype) for _ in range(args.layers)]
            mixers = [b.mixer for b in blocks]
        for m in mixers:
            m.in_proj.weight.normal_(0.0, 0.02)
            m.out_proj.weight.normal_(0.0, 0.02)
    decs = [Mamba3Decoder(m, use_triton=False) for m in mixers]
    states = [d.init_state(args.batch) for d in decs]
    gen = torch.Generator().manual_seed(1)
    us = torch.randn(4, args.batch, kw["d_model"], generator=gen).to(dtype)
    if args.ssm:
        from src.kernels.utils import mamba3_mimo_decode_ref  # the reference's

        m = mixers[0]
        Bz, H, P, D, R = args.batch, m.nheads, m.headdim, m.d_state, m.mimo_rank
        xs = torch.randn(Bz, H, P, generator=gen)
        Bp, Cp = torch.randn(Bz, R, H, D, generator=gen), torch.randn(Bz, R, H, D, generator=gen)
        DT = torch.rand(Bz, H, generator=gen) * 0.1 + 1e-3
        ADT, trap = DT * 1e-4, torch.rand(Bz, H, generator=gen)
        mx, mo = torch.randn(H, R, P, generator=gen) * 0.1, torch.randn(H, R, P, generator=gen) * 0.1
        ssm = [torch.zeros(Bz, H, D), torch.zeros(Bz, H, D)]

    def step(u):
        if args.ssm:
            _, ssm[0], ssm[1] = mamba3_mimo_decode_ref(xs, Bp, Cp, ADT, DT, trap, m.D.float(), mx, mo, ssm[0],
                                                       ssm[1])
            return None
        if blocks[0] is None:
            out, states[0] = decs[0].step(u, states[0])
            return out
        x = u
        for i, (blk, d) in enumerate(zip(blocks, decs)):
            o, states[i] = d.step(blk.norm(x), states[i])
            x = x + o
        return x

    times = []
    with torch.no_grad():
        for i in range(args.warmup):
            step(us[i % 4])
        t_start = time.perf_counter()
        n = 0
        while True:
            t0 = time.perf_counter()
            step(us[n % 4])
            times.append(time.perf_counter() - t0)
            n += 1
            if (args.steps and n >= args.steps) or time.perf_counter() - t_start >= args.budget or n >= 10000:
                break
    total = float(sum(times))
    print(json.dumps({"tokens_per_s": args.batch * n / total, "ms_per_step": 1000.0 * total / n,
                      "p50_ms": 1000.0 * float(np.percentile(times, 50)), "steps": n, "threads": threads,
                      "batch": args.batch, "layers": args.layers, "dtype": args.dtype}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
