"""Batch sharding of decode across the ranks of a process group.

Every sequence of a decode batch is independent (the carried state is per
(batch row, head)), so a batch of ``global_batch`` sequences is split into
contiguous row ranges, one per rank; each rank decodes its own rows with a
full replica of the weights and its own state and CUDA graph, and **no
collective runs on the decode path**.  ``gather`` (an all-gather) exists for
checking and collecting results off the hot path.

The reference has no multi-GPU code; this is the batch-parallel layout the
decode path admits.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from src.models.inference import Mamba3Decoder


def shard_range(global_batch: int, world: int, rank: int) -> tuple:
    """Rows [lo, hi) of the global batch owned by ``rank``: contiguous,
    sizes differing by at most one, lower ranks take the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if global_batch < 0:
        raise ValueError("global_batch must be >= 0")
    base, rem = divmod(global_batch, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


class ShardedDecoder:
    """A ``Mamba3Decoder`` over this rank's share of a global batch.

    ``model`` must hold the same weights on every rank (seed them alike or
    broadcast them once with ``broadcast_parameters``).  ``decoder_kwargs``
    are the ``Mamba3Decoder`` flags.
    """

    def __init__(self, model, global_batch: int, group=None, **decoder_kwargs):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.global_batch = global_batch
        self.lo, self.hi = shard_range(global_batch, self.world, self.rank)
        self.decoder = Mamba3Decoder(model, **decoder_kwargs)

    @property
    def local_batch(self) -> int:
        return self.hi - self.lo

    def local_rows(self, global_tensor: torch.Tensor) -> torch.Tensor:
        """This rank's rows of a tensor indexed by the global batch."""
        return global_tensor[self.lo:self.hi]

    def init_state(self, device=None) -> dict:
        return self.decoder.init_state(self.local_batch, device=device)

    def warmup_cuda_graph(self, state: dict, n_warmup: int = 10) -> None:
        self.decoder.warmup_cuda_graph(state, n_warmup)

    def step(self, u_local: torch.Tensor, state: dict) -> tuple:
        """Decode one token for this rank's rows; no communication."""
        return self.decoder.step(u_local, state)

    def gather(self, local: torch.Tensor) -> torch.Tensor:
        """All-gather rank-local rows into the global-batch tensor (off the
        decode path).  Shards may differ in size by one row."""
        if self.world == 1:
            return local
        sizes = [shard_range(self.global_batch, self.world, r) for r in range(self.world)]
        width = max(hi - lo for lo, hi in sizes)
        pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        pad[: local.shape[0]] = local
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(parts, pad, group=self.group)
        return torch.cat([p[: hi - lo] for p, (lo, hi) in zip(parts, sizes)], dim=0)


def broadcast_parameters(model, src: int = 0, group=None) -> None:
    """Give every rank rank ``src``'s weights (once, before decoding)."""
    if not dist.is_initialized():
        return
    with torch.no_grad():
        for t in list(model.parameters()) + list(model.buffers()):
            dist.broadcast(t.data, src=src, group=group)
