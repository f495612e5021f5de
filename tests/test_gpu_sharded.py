"""KV-head sharding on GPUs (BASELINE config 4's exchange): two (or four) NCCL ranks, one GPU each,
hold their share of the KV heads of every layer and run EvictionPipeline with the process group, which all-reduces
the head reduction between scoring and ActionLRFU.  Both ranks must pick the same keep mask and
compaction plan as an unsharded pipeline over all heads (masks equal except at near-ties; tables,
free list and lengths identical), and each rank's compacted cache slice must equal the matching
heads of the unsharded cache.  Needs two (four) GPUs; the CPU tests of the same exchange are
tests/test_sharding.py."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import cases
from conftest import assert_masks_match
from gpu_util import oracle_lse, packed_region

pytestmark = pytest.mark.gpu

CASE = dict(seed=91, n_layers=2, hq=16, hkv=4, d=128, bs=16, seq_lens=[700, 400], act_lens=[40, 24],
            dtype="bfloat16", extra_blocks=6, channel_scale=True)
PROTECTED, BUDGETS, DECAY, TOP_P = 4, [120, 70], 0.9, 0.9


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(case, lse_list, dev, lo, hi, how, group, total):
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    R, W, G = len(case.seq_lens), max(case.seq_lens), case.hq // case.hkv
    cache = DevicePagedCache(case.num_blocks, case.bs, hi - lo, case.d, case.n_layers, R, W,
                             dtype=cases.DTYPES[case.dtype], device=dev)
    cache.kv.copy_(case.kv[:, :, :, :, lo:hi, :].contiguous().to(dev))
    pipe = EvictionPipeline(cache, EvictionConfig(decay=DECAY, top_p=TOP_P, head_reduce=how), group=group,
                            total_kv_heads=total)
    pipe.load(case.tables, case.seq_lens, case.free, PROTECTED)
    pipe.set_round(case.act_lens, BUDGETS)
    q, lse, _ = packed_region(case, lse_list, dev)
    pipe.step(q[:, :, lo * G:hi * G].contiguous(), lse[:, :, lo * G:hi * G].contiguous())
    torch.cuda.synchronize(dev)
    tables, seq, free = cache.state()
    ks_pre = pipe.ks[1 - pipe.cur]
    return dict(keep=pipe.keep[:R].cpu().numpy(), act=pipe.act[:R].cpu().numpy(),
                ks_mean=ks_pre[:R].mean(1).cpu().numpy(), kv=cache.kv.float().cpu().numpy(),
                tables=np.array([t + [-1] * (W // case.bs + 1 - len(t)) for t in tables]),
                seq=np.array(seq), free=np.array(free))


def _rank(rank, world, port, how, outdir):
    import torch.distributed as dist
    from actkv_open_b200 import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        case = cases.build_sessions(**CASE)
        lse_list = oracle_lse(case)
        lo, hi = sharding.head_shard(case.hkv, world, rank)
        res = _run(case, lse_list, dev, lo, hi, how, dist.group.WORLD, case.hkv)
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), lo=lo, hi=hi, **res)
        dist.barrier()
        if rank == 0:
            full = _run(case, lse_list, dev, 0, case.hkv, how, None, None)
            np.savez(os.path.join(outdir, "full.npz"), **full)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("how", ["mean", "max"])
def test_ranks_agree_with_the_unsharded_pipeline(how, world, tmp_path):
    """Two ranks of two KV heads each; four ranks of one head each (config 4's layout on 8 GPUs)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_rank, args=(world, _free_port(), how, str(tmp_path)), nprocs=world, join=True)
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    full = np.load(tmp_path / "full.npz")
    for r in range(1, world):
        for k in ("keep", "act", "tables", "seq", "free"):
            np.testing.assert_array_equal(ranks[0][k], ranks[r][k], err_msg=f"rank {r}: {k}")
    np.testing.assert_allclose(ranks[0]["act"], full["act"], rtol=1e-5, atol=1e-12)
    R = len(CASE["seq_lens"])
    same = True
    for r, n in enumerate(CASE["seq_lens"]):
        got, want = ranks[0]["keep"][r, :n].astype(bool), full["keep"][r, :n].astype(bool)
        assert_masks_match(got, want, full["ks_mean"][r, :n], what=f"session {r} keep mask")
        same &= bool(np.array_equal(got, want))
        assert got.sum() == min(n, PROTECTED + BUDGETS[r])
    if same:   # the same plan: identical tables / free list / lengths, and each slice of the cache
        for k in ("tables", "seq", "free"):
            np.testing.assert_array_equal(ranks[0][k], full[k], err_msg=k)
        for rk in ranks:
            lo, hi = int(rk["lo"]), int(rk["hi"])
            np.testing.assert_array_equal(rk["kv"], full["kv"][:, :, :, :, lo:hi, :])
    assert R == 2
