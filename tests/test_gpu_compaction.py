"""GPU parity of conflict-free compaction (Algorithm 4, actkv/kernels/compaction.py and
actkv/paged.py:125-157): plans, row copies, tables, free list and cache contents bit-exact against
the reference's golden outputs, including adversarial keep masks and 64-bit plane offsets."""
import math

import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_device_clean, gpu_cache, need_gpu

pytestmark = pytest.mark.gpu


def test_plans_match_reference_golden(golden):
    dev = need_gpu()
    from actkv_open_b200.kernels.compaction import plan_compaction
    g = golden("plans.npz")
    for i, (n, bs, name) in enumerate(g["meta"]["cases"]):
        p = f"p{i}_"
        plan = plan_compaction(torch.from_numpy(g[p + "keep"]).to(dev), n, torch.from_numpy(g[p + "table"]).to(dev), bs)
        np.testing.assert_array_equal(plan.src_slots.cpu().numpy(), g[p + "src"], err_msg=f"{n} {name}")
        np.testing.assert_array_equal(plan.dst_slots.cpu().numpy(), g[p + "dst"], err_msg=f"{n} {name}")
        np.testing.assert_array_equal(plan.perm.cpu().numpy(), g[p + "perm"], err_msg=f"{n} {name}")
        assert plan.drop_blocks == int(g[p + "drop"])
    assert_device_clean(dev)


def test_plan_is_conflict_free_large():
    dev = need_gpu()
    from actkv_open_b200.kernels.compaction import plan_compaction
    from oracle import actkv_oracle as O
    rng = np.random.default_rng(1)
    for n, budget, bs in [(32768, 6557, 16), (131072, 6553, 16), (5000, 4999, 8), (70000, 1, 16)]:
        keep = np.zeros(n, bool)
        keep[rng.permutation(n)[:budget]] = True
        table = rng.permutation(math.ceil(n / bs) + 9)
        plan = plan_compaction(torch.from_numpy(keep).to(dev), n, torch.from_numpy(table).to(dev), bs)
        want = O.plan_compaction(keep, n, table, bs)
        np.testing.assert_array_equal(plan.src_slots.cpu().numpy(), want.src_slots)
        np.testing.assert_array_equal(plan.dst_slots.cpu().numpy(), want.dst_slots)
        np.testing.assert_array_equal(plan.perm.cpu().numpy(), want.perm)
        assert plan.drop_blocks == want.drop_blocks
    assert_device_clean(dev)


def test_cache_compaction_matches_reference_golden(golden):
    dev = need_gpu()
    g = golden("compact.npz")
    specs = [([150], 2, 16), ([40], 2, 16), ([33, 70, 5], 2, 16), ([200, 64], 3, 8)]
    for i, (lens, layers, bs) in enumerate(specs):
        p = f"m{i}_"
        case = cases.build_sessions(300 + i, layers, 4, 2, 32, bs, lens, [1] * len(lens))
        c = gpu_cache(case, dev)
        used = c.used_blocks
        for r in range(len(lens)):
            perm = c.compact(r, torch.from_numpy(g[p + f"keep_{r}"]).to(dev))
            np.testing.assert_array_equal(perm.cpu().numpy(), g[p + f"perm_{r}"])
            assert c.tables[r] == list(g[p + f"table1_{r}"])
            assert c.seq_used[r] == int(g[p + f"seq1_{r}"])
        assert c.free == list(g[p + "free1"])
        assert cases.digest(c.kv) == str(g[p + "kv1_sha"])
        freed = sum(math.ceil(n / bs) - math.ceil(int(g[p + f"seq1_{r}"]) / bs) for r, n in enumerate(lens))
        assert used - c.used_blocks == freed
    assert_device_clean(dev)


def test_multi_round_evict_matches_reference_golden(golden):
    dev = need_gpu()
    g = golden("evict.npz")
    case = cases.build_sessions(500, 2, 4, 2, 16, 16, [90, 45], [1, 1], extra_blocks=20)
    c = gpu_cache(case, dev)
    for step in range(g["meta"]["steps"]):
        key = f"s{step}_"
        r = int(g[key + "req"])
        perm = c.evict(r, torch.from_numpy(g[key + "scores"]).to(dev), int(g[key + "budget"]), protected=5)
        np.testing.assert_array_equal(perm.cpu().numpy(), g[key + "perm"], err_msg=f"step {step}")
        np.testing.assert_array_equal(c.pinned[r].cpu().numpy(), g[key + "pinned"])
        assert c.tables[r] == list(g[key + "table"])
        assert c.free == list(g[key + "free"])
        assert cases.digest(c.kv) == str(g[key + "kv_sha"])
        c.append(r, torch.from_numpy(g[key + "newk"]), torch.from_numpy(g[key + "newv"]))
    assert_device_clean(dev)


def test_evict_keeps_protected_prefix_and_top_scored_tokens():       # test_kernels.py:157-175
    dev = need_gpu()
    case = cases.build_sessions(1, 2, 2, 2, 16, 16, [70], [1])
    c = gpu_cache(case, dev)
    k_before, v_before = c.gather(0, layer=1)
    scores = 0.1 * torch.rand(2, 2, 70, generator=torch.Generator().manual_seed(3)).to(dev)
    hot = [5, 17, 40, 69]
    scores[..., hot] += 1.0
    perm = c.evict(0, scores, budget=4, protected=3)
    assert sorted(perm.tolist()) == [0, 1, 2, *hot]
    k_after, v_after = c.gather(0, layer=1)
    assert torch.equal(k_after, k_before[perm]) and torch.equal(v_after, v_before[perm])
    assert c.seq_used[0] == 7 and len(c.tables[0]) == 1
    case = cases.build_sessions(2, 1, 2, 2, 32, 16, [20], [1])
    c = gpu_cache(case, dev)
    table = list(c.tables[0])
    assert c.evict(0, torch.rand(2, 20, device=dev), budget=20).tolist() == list(range(20))
    assert c.tables[0] == table and c.seq_used[0] == 20
    assert_device_clean(dev)


def test_copy_kernel_matches_reference():                            # test_kernels.py:94-102
    dev = need_gpu()
    from actkv_open_b200.kernels.compaction import apply_copies, apply_copies_ref
    flat = torch.randn(4, 300, 96, device=dev)
    src = torch.tensor([3, 50, 77, 299], device=dev)
    dst = torch.tensor([10, 11, 200, 0], device=dev)
    a, b = flat.clone(), flat.clone()
    apply_copies(a, src, dst)
    apply_copies_ref(b, src, dst)
    assert torch.equal(a, b)
    odd = torch.randn(3, 50, 7, dtype=torch.float16, device=dev)     # 14-byte rows: byte path
    a, b = odd.clone(), odd.clone()
    apply_copies(a, torch.tensor([1, 2], device=dev), torch.tensor([40, 41], device=dev))
    apply_copies_ref(b, torch.tensor([1, 2], device=dev), torch.tensor([40, 41], device=dev))
    assert torch.equal(a, b)
    assert_device_clean(dev)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.mem_get_info()[0] < 8 * 2**30,
                    reason="needs a CUDA GPU with 8 GB free")
def test_copy_kernel_handles_offsets_past_2_to_the_31():             # test_kernels.py:105-119
    dev = need_gpu()
    from actkv_open_b200.kernels.compaction import apply_copies
    row = 1024
    slots = 2**31 // row // 2 + 64
    flat = torch.zeros(3, slots, row, dtype=torch.float16, device=dev)
    src = torch.tensor([5, slots - 1], device=dev)
    dst = torch.tensor([7, 9], device=dev)
    flat[:, src] = torch.arange(1, 4, dtype=torch.float16, device=dev).view(3, 1, 1)
    apply_copies(flat, src, dst)
    torch.cuda.synchronize()
    assert torch.equal(flat[:, dst], flat[:, src])
    del flat
    assert_device_clean(dev)


def test_batched_compaction_with_adversarial_masks_matches_oracle():
    """The batched kernel (all sessions at once, device tables and free stack) against the
    reference's per-request loop; masks as in the agent-loop stress config."""
    dev = need_gpu()
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    from oracle import actkv_oracle as O
    lens = [1088, 517, 64, 2000, 33]
    case = cases.build_sessions(41, 2, 4, 2, 64, 16, lens, [1] * 5, dtype="bfloat16", extra_blocks=7)
    W = max(lens)
    cache = DevicePagedCache(case.num_blocks, 16, 2, 64, 2, len(lens), W, dtype=torch.bfloat16, device=dev)
    cache.kv.copy_(case.kv.to(dev))
    pipe = EvictionPipeline(cache)
    rng = np.random.default_rng(2)
    masks = []
    for i, n in enumerate(lens):
        kind = ["alternating", "all_keep", "sinks_only", "one_per_block", "random"][i]
        m = np.zeros(W, bool)
        if kind == "alternating":
            m[:n:2] = True
        elif kind == "all_keep":
            m[:n] = True
        elif kind == "sinks_only":
            m[:4] = True
        elif kind == "one_per_block":
            m[:n:16] = True
        else:
            m[rng.permutation(n)[: n // 10]] = True
        masks.append(m)
    pipe.load(case.tables, lens, case.free)
    pipe.compact_with(torch.from_numpy(np.stack(masks)).to(dev))
    tables, seq, free = cache.state()
    ref = O.PagedKVCache(case.num_blocks, 16, 2, 64, 2)
    ref.kv[:] = cases.to_np(case.kv)
    ref.free = list(case.free)
    perms = []
    for r, n in enumerate(lens):
        ref.tables[r] = list(case.tables[r])
        ref.seq_used[r] = n
    for r, n in enumerate(lens):
        perms.append(ref.compact(r, masks[r][:n]))
    assert tables == [ref.tables[r] for r in range(len(lens))]
    assert seq == [ref.seq_used[r] for r in range(len(lens))]
    assert free == ref.free
    got_perm = pipe.perm.cpu().numpy()
    for r in range(len(lens)):
        np.testing.assert_array_equal(got_perm[r, :seq[r]], perms[r])
    assert cases.digest(cache.kv) == cases.digest(torch.from_numpy(ref.kv).to(torch.bfloat16))
    assert_device_clean(dev)


def test_chunked_plan_across_chunk_boundaries_and_empty_session():
    """Sessions longer than one 4096-token plan chunk (keep-window and source runs that straddle
    chunk edges, a session of exactly one chunk, one a token past it) next to an empty session,
    against the reference's per-request loop."""
    dev = need_gpu()
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    from oracle import actkv_oracle as O
    lens = [9000, 0, 4096, 4097, 12289, 8191]
    case = cases.build_sessions(43, 2, 4, 2, 64, 16, lens, [1] * len(lens), dtype="bfloat16",
                                extra_blocks=5)
    W = max(lens)
    cache = DevicePagedCache(case.num_blocks, 16, 2, 64, 2, len(lens), W, dtype=torch.bfloat16, device=dev)
    cache.kv.copy_(case.kv.to(dev))
    pipe = EvictionPipeline(cache)
    rng = np.random.default_rng(5)
    masks = []
    for i, n in enumerate(lens):
        m = np.zeros(W, bool)
        if i == 0:
            m[:n] = rng.random(n) < 0.3
        elif i == 2:
            m[:n:2] = True
        elif i == 3:
            m[:n:16] = True
            m[4090:4097] = True                      # a kept run over the chunk edge
        elif i == 4:
            m[:8] = True
            m[4000:4200] = True
            m[8180:8200] = True
            m[12280:n] = True
        elif i == 5:
            m[:n] = rng.random(n) < 0.9
        masks.append(m)
    pipe.load(case.tables, lens, case.free)
    pipe.compact_with(torch.from_numpy(np.stack(masks)).to(dev))
    tables, seq, free = cache.state()
    ref = O.PagedKVCache(case.num_blocks, 16, 2, 64, 2)
    ref.kv[:] = cases.to_np(case.kv)
    ref.free = list(case.free)
    for r, n in enumerate(lens):
        ref.tables[r] = list(case.tables[r])
        ref.seq_used[r] = n
    perms = [ref.compact(r, masks[r][:n]) for r, n in enumerate(lens)]
    assert seq == [ref.seq_used[r] for r in range(len(lens))]
    assert tables == [ref.tables[r] for r in range(len(lens))]
    assert free == ref.free
    got_perm = pipe.perm.cpu().numpy()
    for r in range(len(lens)):
        np.testing.assert_array_equal(got_perm[r, :seq[r]], perms[r])
    assert cases.digest(cache.kv) == cases.digest(torch.from_numpy(ref.kv).to(torch.bfloat16))
    assert_device_clean(dev)
