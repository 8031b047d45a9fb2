"""Stage the unmodified reference package for the runs that need it.

    python oracle/stage_reference.py --reference <reference checkout> [--out baseline/_ref]

The reference (michaelYZh/mamba3-fused-triton-kernel) is pure Python with no
``setup.py`` or ``pyproject.toml``, so ``pip install --target baseline/_ref``
refuses it.  This recipe does what that install would have done: it copies
the reference's ``src/`` package byte for byte into ``baseline/_ref/src/``
(git-ignored, so nothing of it is committed; it travels with the working
tree to the GPU machine) and writes ``baseline/_ref/MANIFEST.json`` with the
sha256 of every file, which the users check before importing anything.

Two users, both test or baseline infrastructure, never the product path:

* ``tests/test_reference_suite_gpu.py`` runs the reference's own
  ``src/tests/test_*.py`` against this package;
* ``bench.py``'s CPU legs time the reference's own PyTorch decode
  (``Mamba3Decoder(model, use_triton=False).step``) on the host cores, in a
  separate interpreter (``oracle/reference_cpu.py``), because the reference
  and this package both name their top-level package ``src``.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEFAULT_OUT = os.path.join(ROOT, "baseline", "_ref")
MANIFEST = "MANIFEST.json"


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 16), b""):
            h.update(block)
    return h.hexdigest()


def stage(reference: str, out: str = DEFAULT_OUT) -> str:
    """Copy ``<reference>/src/**/*.py`` to ``<out>/src`` and write the
    manifest; returns ``out``.  Idempotent."""
    src = os.path.join(reference, "src")
    if not os.path.isdir(src):
        raise FileNotFoundError(f"no src/ package under {reference}")
    dst = os.path.join(out, "src")
    if os.path.isdir(dst):
        shutil.rmtree(dst)
    files = {}
    for dirpath, dirnames, filenames in os.walk(src):
        dirnames[:] = sorted(d for d in dirnames if d != "__pycache__")
        for name in sorted(filenames):
            if not name.endswith(".py"):
                continue
            s = os.path.join(dirpath, name)
            rel = os.path.relpath(s, reference)
            d = os.path.join(out, rel)
            os.makedirs(os.path.dirname(d), exist_ok=True)
            shutil.copyfile(s, d)
            files[rel] = _sha256(d)
    with open(os.path.join(out, MANIFEST), "w") as f:
        json.dump({"reference": "michaelYZh/mamba3-fused-triton-kernel", "files": files}, f, indent=1,
                  sort_keys=True)
    return out


def verify(out: str = DEFAULT_OUT) -> str | None:
    """Reason the staged copy cannot be used, or None when every file is
    present and unmodified."""
    path = os.path.join(out, MANIFEST)
    if not os.path.exists(path):
        return f"the reference is not staged ({path} is missing)"
    with open(path) as f:
        files = json.load(f)["files"]
    for rel, digest in files.items():
        p = os.path.join(out, rel)
        if not os.path.exists(p) or _sha256(p) != digest:
            return f"staged reference file {rel} is missing or modified"
    return None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout")
    ap.add_argument("--out", default=DEFAULT_OUT)
    args = ap.parse_args()
    out = stage(args.reference, args.out)
    print(f"staged {args.reference}/src -> {out}/src")
    return 0


if __name__ == "__main__":
    sys.exit(main())
