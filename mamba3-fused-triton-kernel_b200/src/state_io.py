"""Decode-state I/O: save, load, split and join the carried state of one layer
or of a stack of layers, for resuming a decode and for moving batch shards
between GPUs.

The state of a layer is the reference's cache dict ``{angle_state,
ssm_state, bx_prev}`` (src/models/inference.py:91-95,
src/models/mamba3.py:355-381): fp32 tensors whose first dimension is the
batch.  A stack is a list of such dicts, one per layer.

File format (version 1), all integers little-endian:

    bytes 0..7    magic  b"M3STATE\\x01"
    bytes 8..15   uint64 length N of the header
    bytes 16..    the header: N bytes of UTF-8 JSON
                  {"version": 1, "kind": "layer" | "stack", "layers": L,
                   "batch": B, "meta": {...},
                   "tensors": [{"layer": i, "name": "...", "dtype": "float32",
                                "shape": [...], "offset": o, "nbytes": n}, ...]}
    payload       starts at the first multiple of 64 after the header; each
                  tensor's C-contiguous bytes at payload + offset (offsets are
                  multiples of 64)

A file is checked on load (magic, version, names, dtypes, that every tensor
of a layer has the batch dimension of the file, that the payload is
complete), and a mismatch raises ``ValueError`` naming what is wrong.
"""

from __future__ import annotations

import json
import struct

import numpy as np
import torch

MAGIC = b"M3STATE\x01"
VERSION = 1
NAMES = ("angle_state", "ssm_state", "bx_prev")
_ALIGN = 64


def _pad(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def _layers(states):
    if isinstance(states, dict):
        return "layer", [states]
    if isinstance(states, (list, tuple)) and all(isinstance(s, dict) for s in states):
        return "stack", list(states)
    raise TypeError("states must be a state dict or a list of state dicts")


def _check_layer(st: dict, i: int) -> int:
    missing = [n for n in NAMES if n not in st]
    if missing:
        raise ValueError(f"layer {i}: missing {missing}")
    batch = {int(st[n].shape[0]) for n in NAMES}
    if len(batch) != 1:
        raise ValueError(f"layer {i}: batch dimensions differ {sorted(batch)}")
    for n in NAMES:
        if st[n].dtype != torch.float32:
            raise ValueError(f"layer {i}: {n} is {st[n].dtype}, the decode state is float32")
    return batch.pop()


def save_states(path: str, states, meta: dict | None = None) -> None:
    """Write one layer's state dict, or a list of them, to ``path``.  The
    tensors are copied to host memory (synchronously)."""
    kind, layers = _layers(states)
    batch = {_check_layer(st, i) for i, st in enumerate(layers)}
    if len(batch) > 1:
        raise ValueError(f"layers have different batch sizes {sorted(batch)}")
    entries, blobs, off = [], [], 0
    for i, st in enumerate(layers):
        for n in NAMES:
            a = st[n].detach().to("cpu").contiguous().numpy()
            entries.append({"layer": i, "name": n, "dtype": "float32", "shape": list(a.shape),
                            "offset": off, "nbytes": int(a.nbytes)})
            blobs.append(a)
            off = _pad(off + a.nbytes)
    header = json.dumps({"version": VERSION, "kind": kind, "layers": len(layers),
                         "batch": batch.pop() if batch else 0, "meta": meta or {},
                         "tensors": entries}).encode("utf-8")
    start = _pad(16 + len(header))
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        f.write(b"\0" * (start - 16 - len(header)))
        pos = 0
        for e, a in zip(entries, blobs):
            f.write(b"\0" * (e["offset"] - pos))
            f.write(a.astype("<f4", copy=False).tobytes())
            pos = e["offset"] + e["nbytes"]


def load_states(path: str, device=None) -> tuple:
    """Read a file written by ``save_states``; returns ``(states, meta)``
    with ``states`` a dict for a single layer or a list of dicts for a
    stack, on ``device`` (default: CPU)."""
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < 16 or raw[:8] != MAGIC:
        raise ValueError(f"{path}: not a decode-state file (bad magic)")
    (hlen,) = struct.unpack("<Q", raw[8:16])
    if 16 + hlen > len(raw):
        raise ValueError(f"{path}: truncated header")
    try:
        head = json.loads(raw[16:16 + hlen].decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise ValueError(f"{path}: unreadable header ({e})") from None
    if head.get("version") != VERSION:
        raise ValueError(f"{path}: version {head.get('version')}, this reader knows {VERSION}")
    start = _pad(16 + hlen)
    L, B = int(head["layers"]), int(head["batch"])
    layers = [dict() for _ in range(L)]
    for e in head["tensors"]:
        i, n = int(e["layer"]), e["name"]
        if not 0 <= i < L or n not in NAMES or e["dtype"] != "float32":
            raise ValueError(f"{path}: unexpected tensor entry {e}")
        shape = tuple(int(s) for s in e["shape"])
        count = int(np.prod(shape)) if shape else 1
        if not shape or shape[0] != B or count * 4 != int(e["nbytes"]):
            raise ValueError(f"{path}: tensor {n} of layer {i} has shape {shape}, batch {B}")
        lo = start + int(e["offset"])
        if lo + count * 4 > len(raw):
            raise ValueError(f"{path}: truncated payload ({n} of layer {i})")
        a = np.frombuffer(raw, dtype="<f4", count=count, offset=lo).reshape(shape)
        layers[i][n] = torch.from_numpy(a.copy()).to(device or "cpu")
    for i, st in enumerate(layers):
        _check_layer(st, i)
    return (layers[0] if head["kind"] == "layer" else layers), head.get("meta", {})


def slice_rows(states, lo: int, hi: int):
    """Batch rows [lo, hi) of a state dict or list of them, as contiguous
    copies (the rows a shard hands to another GPU)."""
    kind, layers = _layers(states)
    out = [{n: st[n][lo:hi].contiguous().clone() for n in NAMES} for st in layers]
    return out[0] if kind == "layer" else out


def concat_rows(parts: list):
    """Join state dicts (or lists of them, layer by layer) along the batch,
    in the order given; all parts on one device."""
    if not parts:
        raise ValueError("nothing to concatenate")
    kinds = {_layers(p)[0] for p in parts}
    if len(kinds) != 1:
        raise ValueError("cannot join single-layer and stack states")
    per = [_layers(p)[1] for p in parts]
    if len({len(p) for p in per}) != 1:
        raise ValueError("parts have different layer counts")
    out = [{n: torch.cat([p[i][n] for p in per], dim=0) for n in NAMES} for i in range(len(per[0]))]
    return out[0] if kinds.pop() == "layer" else out
