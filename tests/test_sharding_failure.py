"""Failure detection of the KV-head sharded step on CPU (gloo): a rank that leaves between steps,
before the one collective of the path, must not hang the others: the surviving rank's
allreduce_heads ends with an error (peer gone, or the process group's short timeout)."""
import datetime
import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, outdir):
    import torch.distributed as dist
    from actkv_open_b200 import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)                       # leaves between steps, without joining the collective
    part = torch.ones(1, 2, 64)
    try:
        sharding.allreduce_heads(part, 2, "mean")
        result = "completed"
    except Exception as e:                # noqa: BLE001 - any error ends the wait, which is the point
        result = "error: " + type(e).__name__
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(result)
    os._exit(0)


def test_a_rank_that_leaves_ends_the_others_collective_with_an_error(tmp_path):
    mp.spawn(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "rank0.txt").read_text().startswith("error:")
