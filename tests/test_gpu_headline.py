"""Parity at BASELINE's own shapes, through EvictionPipeline.step on the tcgen05 scoring kernels
(configs 2 and 4 on both the CTA-pair kernel and the one-CTA kernel):

  config 2   36 layers, 32768 tokens on 2048 scattered blocks, Hq/Hkv = 32/8, A = 128 (A*G = 512:
             two full 256-column query chunks, the headline kernel instantiation), 20% + 4 sinks
  config 4   one rank's KV-head shard: 80 layers, 131072 tokens, one KV head with G = 8, A = 256
             (A*G = 2048: eight chunks, the block path of both kernels), 5% + 4 sinks
  config 3   one LPT shard of the 64-session batch: 8 sessions with S in [4096, 65536] and A in
             [32, 256] (A*G up to 1024: the CTA-pair kernel's four resident query chunks), 10% + 4 sinks

Each step is checked by actkv_open_b200.check (a torch fp32 restatement of the reference's formulas,
itself checked against the pinned oracle in test_check_ref.py): per-head scores and head means
within 1e-3 relative; keep scores equal except at the nucleus boundary; keep masks equal except at
near-ties; tables, free stack, lengths, perm, every byte of every K/V plane and the permuted keep
scores and pins bit-exact.  The workloads are bench.py's builders (seeded, exact causal lse)."""
import pytest
import torch

from gpu_util import assert_device_clean, need_gpu

pytestmark = pytest.mark.gpu


def _step_and_check(pipe, q, lse, path):
    from actkv_open_b200 import check
    pipe.path = path
    before = check.capture_state(pipe)
    pipe.step(q, lse)
    torch.cuda.synchronize()
    rep = check.check_step(pipe, before, q, lse, rtol=1e-3)
    del before
    return rep


@pytest.mark.parametrize("path", ["pair", "tcgen05"])
def test_config2_full_size_step(path):
    dev = need_gpu()
    import bench
    cache, pipe, q, lse = bench.build_config2(dev, 0, 36, 32768)
    assert pipe.max_actions * (q.shape[2] // cache.n_kv_heads) == 512
    rep = _step_and_check(pipe, q, lse, path)
    assert rep["ok"] and rep["moved_rows"] > 4000, rep
    assert int(pipe.kept[0]) == bench.CFG2["BUDGET"] + bench.CFG2["P"]
    assert_device_clean(dev)
    del cache, pipe, q, lse
    torch.cuda.empty_cache()


@pytest.mark.parametrize("path", ["pair", "tcgen05"])
def test_config4_head_shard_full_size_step(path):
    dev = need_gpu()
    import bench
    cache, pipe, q, lse = bench.build_config4(dev, 0, 3, 4)          # KV head 3 of 8: G = 8, A = 256
    assert cache.n_kv_heads == 1 and pipe.max_actions * q.shape[2] == 2048
    rep = _step_and_check(pipe, q, lse, path)                # A*G = 2048: both kernels' block paths
    assert rep["ok"] and rep["moved_rows"] > 0, rep
    assert int(pipe.kept[0]) == bench.CFG4["BUDGET"] + bench.CFG4["P"]
    assert_device_clean(dev)
    del cache, pipe, q, lse
    torch.cuda.empty_cache()


def test_config3_lpt_shard_full_size_step():
    dev = need_gpu()
    import bench
    sessions = bench.config3_sessions(0)
    shard = bench.lpt_assign(sessions, 8)[0]
    items = [(i, *sessions[i]) for i in shard]
    assert any(a * 4 > 512 for _, _, a in items) and any(a * 4 <= 512 for _, _, a in items)
    cache, pipe, q, lse, budgets = bench.build_config3(dev, items, 0, pool_seed=0)
    rep = _step_and_check(pipe, q, lse, "pair")              # A*G <= 1024: four resident chunks
    assert rep["ok"] and rep["sessions"] == len(items), rep
    kept = pipe.kept[:len(items)].tolist()
    assert kept == [b + bench.CFG3["P"] for b in budgets]
    assert_device_clean(dev)
    del cache, pipe, q, lse
    torch.cuda.empty_cache()
