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
