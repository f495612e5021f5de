"""KV-head sharding host logic on CPU: two gloo ranks each hold half of the KV
heads, score them (the numpy oracle stands in for the scoring kernel here, as the compute of each
rank), and exchange only the head reduction through ``actkv_open_b200.sharding``.  Both ranks must
end with the same action attention as the unsharded reference computation (the head mean or max
over all heads, actkv/eviction.py:20-33) and therefore the same ActionLRFU keep mask.  The GPU
version of the same exchange, inside EvictionPipeline, is tests/test_gpu_sharded.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from actkv_open_b200 import sharding
from cases import block_table_array, build_sessions
from conftest import assert_masks_match
from oracle import actkv_oracle as O

CASE = dict(seed=31, n_layers=2, hq=8, hkv=4, d=16, bs=16, seq_lens=[200], act_lens=[8], dtype="float32",
            extra_blocks=2)
BUDGET, PROTECTED, DECAY, TOP_P = 40, 4, 0.9, 0.9


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _head_scores():
    """Per-head scores [L, Hkv, n] of the case's session (the oracle's causal region scoring)."""
    c = build_sessions(**CASE)
    kv = c.kv.numpy()
    bt = block_table_array(c.tables)[0].astype(np.int64)
    n = c.seq_lens[0]
    q = c.q[0].numpy()
    out = []
    for l in range(c.n_layers):
        lse = O.causal_region_lse(q[l], kv[l], bt, n)
        out.append(O.layer_scores(kv[l], bt, n, q[l], lse))
    return np.stack(out)


def _keep_mask(act, how):
    """ActionLRFU round on ``act`` [L, n] and the evict keep mask of the layer-mean keep scores."""
    L, n = act.shape
    pol = O.ActionLRFU(decay=DECAY, top_p=TOP_P, head_reduce=how)
    pol.reset(L)
    pol.act = act.astype(np.float32).copy()
    pol.n_act = 1
    pol.update_scores(n, PROTECTED)
    return O.keep_mask_from_scores(pol.ks[:, :n], n, BUDGET, PROTECTED), pol.ks[:, :n].mean(0)


def _rank(rank, world, port, how, outdir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hs = _head_scores()                                          # [L, Hkv, n]
        lo, hi = sharding.head_shard(hs.shape[1], world, rank)
        mine = torch.from_numpy(np.ascontiguousarray(hs[None, :, lo:hi, :]))   # [1, L, h, n]
        part = sharding.local_head_reduce(mine, how).contiguous()
        sharding.allreduce_heads(part, hs.shape[1], how)
        act = part[0].numpy()
        keep, _ = _keep_mask(act, how)
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), act=act, keep=keep, lo=lo, hi=hi)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("how", ["mean", "max"])
def test_gloo_ranks_agree_with_the_unsharded_reduction(how, world, tmp_path):
    """Two ranks of two heads each, and four ranks of one head each (the layout of config 4 on eight
    GPUs: each rank's part of the reduction is its one head, a view)."""
    mp.spawn(_rank, args=(world, _free_port(), how, str(tmp_path)), nprocs=world, join=True)
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    per = 4 // world
    assert [(int(r["lo"]), int(r["hi"])) for r in res] == [(r * per, (r + 1) * per) for r in range(world)]
    # a collective returns the same values on every rank, so the masks agree bit for bit
    for r in range(1, world):
        np.testing.assert_array_equal(res[0]["act"], res[r]["act"])
        np.testing.assert_array_equal(res[0]["keep"], res[r]["keep"])
    hs = _head_scores()
    want = hs.mean(1, dtype=np.float32) if how == "mean" else hs.max(1)
    np.testing.assert_allclose(res[0]["act"], want, rtol=1e-6, atol=0)
    keep_want, ks_mean = _keep_mask(want, how)
    assert_masks_match(res[0]["keep"], keep_want, ks_mean, what=f"sharded keep mask ({how})")
    assert res[0]["keep"].sum() == PROTECTED + BUDGET


def test_head_shard_splits_evenly_and_rejects_the_rest():
    assert [sharding.head_shard(8, 8, r) for r in range(8)] == [(r, r + 1) for r in range(8)]
    assert [sharding.head_shard(8, 2, r) for r in range(2)] == [(0, 4), (4, 8)]
    with pytest.raises(ValueError):
        sharding.head_shard(8, 3, 0)
    with pytest.raises(ValueError):
        sharding.head_shard(8, 2, 2)


def test_local_head_reduce_is_a_view_for_one_head_and_a_sum_or_max_otherwise():
    g = torch.Generator().manual_seed(3)
    one = torch.rand(2, 3, 1, 50, generator=g)
    v = sharding.local_head_reduce(one, "mean")
    assert v.data_ptr() == one.data_ptr() and v.shape == (2, 3, 50)
    many = torch.rand(2, 3, 4, 50, generator=g)
    torch.testing.assert_close(sharding.local_head_reduce(many, "mean"), many.sum(2))
    torch.testing.assert_close(sharding.local_head_reduce(many, "max"), many.amax(2))
    out = torch.empty(2, 3, 50)
    assert sharding.local_head_reduce(many, "mean", out) is out
    with pytest.raises(ValueError):
        sharding.local_head_reduce(many, "median")
