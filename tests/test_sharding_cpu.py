"""Multi-process batch sharding on the CPU (gloo, world size 2).

* sharded decode == one process decoding the whole batch (no collective on
  the decode path; results gathered afterwards);
* parameter broadcast gives every rank rank 0's weights;
* a rank that dies before a collective makes the survivor's collective fail
  with an error within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import sys
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _sharded_worker(rank, world, port, global_batch, steps, out_path):
    dist = _init(rank, world, port)
    from src.models.mamba3 import Mamba3
    from src.sharding import ShardedDecoder, broadcast_parameters
    torch.manual_seed(100 + rank)  # different weights per rank ...
    model = Mamba3(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2)
    broadcast_parameters(model)  # ... until rank 0's are broadcast
    dec = ShardedDecoder(model, global_batch, use_triton=False)
    st = dec.init_state()
    g = torch.Generator().manual_seed(7)
    u = torch.randn(steps, global_batch, 64, generator=g)
    outs = []
    with torch.no_grad():
        for t in range(steps):
            o, st = dec.step(dec.local_rows(u[t]), st)
            outs.append(dec.gather(o))
    full_h = dec.gather(st["ssm_state"])
    if rank == 0:
        torch.save({"outs": torch.stack(outs), "h": full_h, "sd": model.state_dict()}, out_path)
    dist.destroy_process_group()


@pytest.mark.parametrize("global_batch", [5, 8])
def test_sharded_decode_matches_single_process(tmp_path, global_batch):
    out = str(tmp_path / "sharded.pt")
    mp.start_processes(_sharded_worker, args=(2, _free_port(), global_batch, 4, out), nprocs=2,
                       start_method="spawn", join=True)
    got = torch.load(out)
    import sys
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    from src.models.inference import Mamba3Decoder
    from src.models.mamba3 import Mamba3
    torch.manual_seed(100)
    model = Mamba3(d_model=64, d_state=16, headdim=16, is_mimo=True, mimo_rank=2)
    for k, v in model.state_dict().items():
        torch.testing.assert_close(got["sd"][k], v)  # broadcast gave rank 0's weights
    dec = Mamba3Decoder(model, use_triton=False)
    st = dec.init_state(global_batch)
    g = torch.Generator().manual_seed(7)
    u = torch.randn(4, global_batch, 64, generator=g)
    with torch.no_grad():
        ref = torch.stack([dec.step(u[t], st)[0] for t in range(4)])
    torch.testing.assert_close(got["outs"], ref)
    torch.testing.assert_close(got["h"], st["ssm_state"])


def test_shard_range_covers_the_batch():
    from src.sharding import shard_range
    for world in (1, 2, 3, 8):
        for batch in (0, 1, 7, 256, 1001):
            spans = [shard_range(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _dying_worker(rank, world, port, path):
    dist = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        os._exit(3)  # dies between steps, before the collective
    err = "no error"
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
    except Exception as e:  # the survivor learns of the failure
        err = type(e).__name__
    with open(path, "w") as f:
        f.write(err)
    os._exit(0)


def test_dead_rank_is_reported_not_hung(tmp_path):
    path = str(tmp_path / "err.txt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, path)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung after its peer died"
    assert procs[1].exitcode == 3
    assert open(path).read() != "no error"
