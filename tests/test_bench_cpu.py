"""bench.py under torchrun: every rank must take the same collective steps in
the same order, or the ranks that skip one leave the others waiting until
the process-group timeout.  bench.py needs a GPU to run, so this checks its
structure: no collective (``max_over_ranks``, ``barrier``, ``dist.*``) sits
inside a block that only some ranks enter (a test of ``rank``)."""

from __future__ import annotations

import ast
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COLLECTIVES = {"max_over_ranks", "all_reduce", "barrier", "all_gather", "broadcast", "reduce"}


def _mentions_rank(node: ast.AST) -> bool:
    return any(isinstance(n, ast.Name) and n.id == "rank" for n in ast.walk(node))


def _calls(node: ast.AST):
    for n in ast.walk(node):
        if isinstance(n, ast.Call):
            f = n.func
            name = f.id if isinstance(f, ast.Name) else f.attr if isinstance(f, ast.Attribute) else None
            if name in COLLECTIVES:
                yield name, n.lineno


def test_no_collective_inside_a_rank_dependent_branch():
    tree = ast.parse(open(os.path.join(ROOT, "bench.py")).read())
    bad = []
    for node in ast.walk(tree):
        if isinstance(node, ast.If) and _mentions_rank(node.test):
            for stmt in node.body + node.orelse:
                bad.extend(_calls(stmt))
        if isinstance(node, ast.IfExp) and _mentions_rank(node.test):
            bad.extend(_calls(node.body))
            bad.extend(_calls(node.orelse))
    assert not bad, f"collectives reached by only some ranks: {bad}"


def _json_lines(text):
    import json
    return [json.loads(ln) for ln in text.splitlines() if ln.startswith("{")]


def test_global_batch_splits_evenly_over_ranks():
    import sys

    import pytest
    sys.path.insert(0, ROOT)
    import bench
    assert [bench.shard_rows(256, n) for n in (1, 2, 4, 8)] == [256, 128, 64, 32]
    with pytest.raises(SystemExit):
        bench.shard_rows(256, 3)
    assert bench.DEFAULT_WORKLOAD == "stack24_d2048_b256_bf16"
    assert bench.WORKLOADS[bench.DEFAULT_WORKLOAD][1] == 256


def test_reference_arm_times_the_reference_cpu_decode():
    """--impl reference runs the reference's own PyTorch CPU decode (from the
    staged copy) on the workload's global batch, without a GPU; under
    torchrun only rank 0 prints."""
    import subprocess
    import sys

    import pytest
    from oracle.stage_reference import DEFAULT_OUT, verify
    why = verify(DEFAULT_OUT)
    if why:
        pytest.skip(why)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONDONTWRITEBYTECODE="1")
    args = ["bench.py", "--impl", "reference", "--workload", "mimo_r4_d256_b128", "--steps", "3", "--warmup", "1"]
    r = subprocess.run([sys.executable, *args], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    (line,) = _json_lines(r.stdout)
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "reference"
    assert line["config"]["global_batch"] == 128 and line["dtype"] == "f32" and line["steps"] == 3
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29517", *args, "--gpus", "2"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    (line,) = _json_lines(r.stdout)
    assert line["n_gpus"] == 2 and line["config"]["global_batch"] == 128


def test_sweep_takes_single_layer_workloads_only():
    """``--sweep`` runs one layer over batch sizes and MIMO ranks; a stack,
    prefill, projection or state-update workload is refused before any GPU
    work."""
    import subprocess
    import sys
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--sweep", "--workload",
                        "stack24_d2048_b256_bf16"], capture_output=True, text=True, timeout=300)
    assert r.returncode != 0 and "single-layer workload" in r.stderr + r.stdout, r.stderr[-500:]
