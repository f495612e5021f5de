"""End-to-end GPU parity of one eviction step (score -> ActionLRFU -> keep mask -> compaction ->
state permutation) through actkv_open_b200.engine.EvictionPipeline, against the reference's golden
pipeline (BASELINE config 1 and a bf16 multi-layer batch) and, over several agent-loop rounds with
adversarial masks, against the CPU oracle.

Scores and keep scores must agree within 1e-3 relative; keep masks must be equal except at
near-ties (a nucleus or top-k boundary whose values agree to 1e-3); the compaction (tables, free
list, lengths, cache bytes) must be bit-exact for the mask the kernels chose."""
import numpy as np
import pytest
import torch

import cases
from conftest import assert_masks_match
from gpu_util import assert_device_clean, need_gpu, packed_region

pytestmark = pytest.mark.gpu


def _pipeline(case, dev, decay, top_p, path="auto"):
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    W = max(case.seq_lens)
    cache = DevicePagedCache(case.num_blocks, case.bs, case.hkv, case.d, case.n_layers, len(case.seq_lens), W,
                             dtype=cases.DTYPES[case.dtype], device=dev)
    cache.kv.copy_(case.kv.to(dev))
    return cache, EvictionPipeline(cache, EvictionConfig(decay=decay, top_p=top_p), path=path)


def _nucleus_near(act_row, got_ks, want_ks, rtol):
    """Entries where GPU and reference keep scores differ must sit at the nucleus boundary."""
    bad = ~np.isclose(got_ks, want_ks, rtol=rtol, atol=1e-12)
    if not bad.any():
        return
    pos = act_row[act_row > 0]
    thr_cands = np.sort(pos)
    for i in np.nonzero(bad)[0]:
        a = act_row[i]
        near = np.abs(thr_cands - a) <= rtol * a
        assert near.any() and abs(got_ks[i] - want_ks[i]) <= a * (1 + rtol), f"token {i} differs off-boundary"


@pytest.mark.parametrize("name,spec,protected,budgets,decay,top_p", [
    ("config1.npz", cases.CONFIG1, cases.CONFIG1_PROTECTED, [cases.CONFIG1_BUDGET],
     cases.CONFIG1_DECAY, cases.CONFIG1_TOP_P),
    ("pipe_bf16.npz", cases.PIPE_BF16, cases.PIPE_BF16_PROTECTED, cases.PIPE_BF16_BUDGETS,
     cases.PIPE_BF16_DECAY, cases.PIPE_BF16_TOP_P),
])
def test_pipeline_matches_reference_golden(golden, name, spec, protected, budgets, decay, top_p):
    dev = need_gpu()
    from oracle import actkv_oracle as O
    g = golden(name)
    case = cases.build_sessions(**spec)
    assert cases.digest(case.kv) == g["meta"]["kv_sha256_in"]
    R = len(case.seq_lens)
    cache, pipe = _pipeline(case, dev, decay, top_p)
    pipe.load(case.tables, case.seq_lens, case.free, protected)
    pipe.set_round(case.act_lens, budgets)
    q, lse, _ = packed_region(case, [g[f"lse_{r}"] for r in range(R)], dev)
    pipe.step(q, lse)
    torch.cuda.synchronize()
    heads = pipe.heads.cpu().numpy()
    act = pipe.act.cpu().numpy()
    keep = pipe.keep.cpu().numpy().astype(bool)
    tables, seq, free = cache.state()
    # the reference's own state transitions, replayed with the masks the kernels chose
    ref = O.PagedKVCache(case.num_blocks, case.bs, case.hkv, case.d, case.n_layers)
    ref.kv[:] = cases.to_np(case.kv)
    ref.free = list(case.free)
    for r, n in enumerate(case.seq_lens):
        ref.tables[r] = list(case.tables[r])
        ref.seq_used[r] = n
    all_equal = True
    for r, n in enumerate(case.seq_lens):
        np.testing.assert_allclose(heads[r, :, :, :n], g[f"heads_{r}"], rtol=1e-3, atol=1e-12)
        np.testing.assert_allclose(act[r, :, :n], g[f"act_{r}"], rtol=1e-3, atol=1e-12)
        # keep scores before the permutation = ks the keep mask was taken from
        ks_pre = pipe.ks[1 - pipe.cur].cpu().numpy()[r, :, :n]
        for l in range(case.n_layers):
            _nucleus_near(g[f"act_{r}"][l], ks_pre[l], g[f"ks_{r}"][l], 1e-3)
        s_ref = g[f"ks_{r}"].mean(0)
        assert_masks_match(keep[r, :n], g[f"keep_{r}"], s_ref, rtol=1e-3, what=f"session {r}")
        all_equal &= bool(np.array_equal(keep[r, :n], g[f"keep_{r}"]))
        perm = ref.compact(r, keep[r, :n])
        np.testing.assert_array_equal(pipe.perm.cpu().numpy()[r, :len(perm)], perm)
    assert tables == [ref.tables[r] for r in range(R)]
    assert seq == [ref.seq_used[r] for r in range(R)]
    assert free == ref.free
    assert cases.digest(cache.kv) == cases.digest(torch.from_numpy(ref.kv).to(cases.DTYPES[case.dtype]))
    if all_equal:    # same masks as the reference: its recorded end state must match exactly
        for r in range(R):
            assert tables[r] == list(g[f"table_{r}"]) and seq[r] == int(g[f"seq_{r}"])
        assert free == list(g["free"])
        assert cases.digest(cache.kv) == g["meta"]["kv_sha256_out"]
        pin = pipe.pinned.cpu().numpy().astype(bool)
        for r in range(R):
            np.testing.assert_array_equal(pin[r, :seq[r]], g[f"pinned_{r}"])
    assert_device_clean(dev)


def test_agent_loop_rounds_match_oracle():
    """Five rounds of append -> score -> ActionLRFU -> evict with the keep scores and pins carried
    on the device; round 3 replaces the mask with adversarial ones (alternating / one per block).
    Each round is compared with the oracle: scores and keep scores to 1e-3, masks up to near-ties,
    then the oracle replays the kernels' mask and tables, free list, lengths, cache bytes, pins and
    permuted keep scores must agree exactly."""
    dev = need_gpu()
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    from gpu_util import oracle_lse
    from oracle import actkv_oracle as O
    L, HQ, HKV, D, BS = 2, 8, 2, 128, 16
    R, NEW, ACT, BUDGET, P = 2, 96, 16, 80, 4
    W = 1024
    gen = torch.Generator().manual_seed(123)
    n_blocks = R * (W // BS)
    cache = DevicePagedCache(n_blocks, BS, HKV, D, L, R, W, dtype=torch.bfloat16, device=dev)
    pipe = EvictionPipeline(cache, EvictionConfig(decay=0.9, top_p=0.9))
    ref = O.PagedKVCache(n_blocks, BS, HKV, D, L)
    ref.free = torch.randperm(n_blocks, generator=gen).tolist()
    ks_ref = [np.zeros((L, 0), np.float32) for _ in range(R)]
    pin_ref = [np.zeros(0, bool) for _ in range(R)]
    ks_dev = torch.zeros(R, L, W, device=dev)
    pin_dev = torch.zeros(R, W, dtype=torch.uint8, device=dev)
    for rnd in range(5):
        for r in range(R):                                   # append NEW tokens (host oracle + device copy)
            k = torch.randn(L, NEW, HKV, D, generator=gen).to(torch.bfloat16).float().numpy()
            v = torch.randn(L, NEW, HKV, D, generator=gen).to(torch.bfloat16).float().numpy()
            ref.append(r, k, v)
        lens = [ref.seq_used[r] for r in range(R)]
        for r in range(R):
            first = pin_ref[r].size == 0
            pin_ref[r] = np.concatenate([pin_ref[r], np.arange(pin_ref[r].size, lens[r]) < (P if first else 0)])
            ks_ref[r] = np.concatenate([ks_ref[r], np.zeros((L, lens[r] - ks_ref[r].shape[1]), np.float32)], 1)
            if first:
                pin_dev[r, :P] = 1
        cache.kv.copy_(torch.from_numpy(ref.kv).to(torch.bfloat16).to(dev))
        pipe.load([ref.tables[r] for r in range(R)], lens, list(ref.free))
        pipe.pin[0].copy_(pin_dev)
        pipe.ks[0].copy_(ks_dev)
        if rnd == 2:                                         # adversarial masks through compact_with
            keep = np.zeros((R, W), bool)
            keep[0, :lens[0]:2] = True
            keep[1, :lens[1]:BS] = True
            keep[:, :P] = True
            pipe.compact_with(torch.from_numpy(keep).to(dev))
            from actkv_open_b200 import _native as N
            N.check(N.load().actkv_permute_tokens(
                pipe.ks[0].data_ptr(), pipe.ks[1].data_ptr(), pipe.ks[0].stride(0), pipe.ks[0].stride(1), L,
                pipe.pin[0].data_ptr(), pipe.pin[1].data_ptr(), W, pipe.perm.data_ptr(), W,
                cache.seq_used.data_ptr(), R, W, None, N.stream_ptr(dev)))
            pipe.cur = 1
        else:
            qs = [torch.randn(L, ACT, HQ, D, generator=gen).to(torch.bfloat16) for _ in range(R)]
            sc = cases.SessionCase(L, HQ, HKV, D, BS, lens, [ACT] * R, "bfloat16", n_blocks, [],
                                   torch.from_numpy(ref.kv).to(torch.bfloat16),
                                   [ref.tables[r] for r in range(R)], list(ref.free), qs)
            lse = oracle_lse(sc)
            pipe.set_round([ACT] * R, [BUDGET] * R)
            q, lse_t, _ = packed_region(sc, lse, dev)
            pipe.step(q, lse_t)
            heads = pipe.heads.cpu().numpy()
            ks_pre = pipe.ks[1 - pipe.cur].cpu().numpy()
            keep = pipe.keep.cpu().numpy().astype(bool)
            for r in range(R):
                n = lens[r]
                bt = np.asarray(ref.tables[r], np.int64)
                want_heads = np.stack([O.layer_scores(ref.kv[l], bt, n, cases.to_np(qs[r][l]), lse[r][l])
                                       for l in range(L)])
                np.testing.assert_allclose(heads[r, :, :, :n], want_heads, rtol=1e-3, atol=1e-12)
                pol = O.ActionLRFU(decay=0.9, top_p=0.9)
                pol.reset(L)
                pol.ks = ks_ref[r].copy()
                pol.act = want_heads.mean(1, dtype=np.float32)
                pol.n_act = ACT
                pol.update_scores(n, pin_ref[r])
                for l in range(L):
                    _nucleus_near(want_heads.mean(1)[l], ks_pre[r, l, :n], pol.ks[l], 1e-3)
                want_keep = O.keep_mask_from_scores(pol.ks, n, BUDGET, pin_ref[r])
                assert_masks_match(keep[r, :n], want_keep, pol.ks.mean(0), rtol=1e-3, what=f"round {rnd} r{r}")
                ks_ref[r] = ks_pre[r, :, :n].copy()          # continue from the kernels' keep scores
        for r in range(R):                                   # replay the kernels' masks on the oracle
            n = lens[r]
            if rnd != 2 and n - pin_ref[r].sum() <= BUDGET:
                continue
            perm = ref.compact(r, keep[r, :n])
            pin_ref[r] = pin_ref[r][perm]
            ks_ref[r] = ks_ref[r][:, perm]
        tables, seq, free = cache.state()
        assert tables == [ref.tables[r] for r in range(R)], f"round {rnd}"
        assert seq == [ref.seq_used[r] for r in range(R)]
        assert free == ref.free
        assert cases.digest(cache.kv) == cases.digest(torch.from_numpy(ref.kv).to(torch.bfloat16))
        ks_dev = pipe.ks[pipe.cur].clone()
        pin_dev = pipe.pin[pipe.cur].clone()
        ks_np, pin_np = ks_dev.cpu().numpy(), pin_dev.cpu().numpy().astype(bool)
        for r in range(R):
            n = seq[r]
            np.testing.assert_array_equal(pin_np[r, :n], pin_ref[r])
            np.testing.assert_array_equal(ks_np[r, :, :n], ks_ref[r])
            assert not ks_np[r, :, n:].any() and not pin_np[r, n:].any()
    assert_device_clean(dev)


def test_step_host_equals_step():
    """step_host (queries and lse in pinned host memory, copied and scored layer group by layer
    group) must leave exactly the state that step leaves."""
    dev = need_gpu()
    from gpu_util import oracle_lse
    case = cases.build_sessions(**cases.PIPE_BF16)
    lse_list = oracle_lse(case)
    results = []
    for host in (False, True):
        cache, pipe = _pipeline(case, dev, cases.PIPE_BF16_DECAY, cases.PIPE_BF16_TOP_P)
        pipe.load(case.tables, case.seq_lens, case.free, cases.PIPE_BF16_PROTECTED)
        pipe.set_round(case.act_lens, cases.PIPE_BF16_BUDGETS)
        q, lse, _ = packed_region(case, lse_list, dev)
        if host:
            pipe.step_host(q.cpu().pin_memory(), lse.cpu().pin_memory(), layer_groups=2)
        else:
            pipe.step(q, lse)
        torch.cuda.synchronize()
        results.append([pipe.heads.cpu(), pipe.keep_scores.cpu(), pipe.keep.cpu(), pipe.perm.cpu(), cache.kv.cpu(),
                        cache.block_table.cpu(), cache.seq_used.cpu(), cache.free_list.cpu(), cache.free_top.cpu()])
    for a, b in zip(*results):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):
        pipe.step_host(q.cpu(), lse.cpu())
    assert_device_clean(dev)


STREAM_CASE = dict(seed=91, n_layers=7, hq=8, hkv=2, d=128, bs=16, seq_lens=[900, 333, 1211],
                   act_lens=[40, 9, 64], dtype="bfloat16", extra_blocks=4)


@pytest.mark.parametrize("path,streamed", [("auto", True), ("pair", True), ("tcgen05", False)])
def test_step_host_streamed_groups_equal_step(path, streamed):
    """step_host's single scoring launch over streamed layer groups (seven groups of one layer,
    three sessions), and its fallback to grouped launches on the one-CTA path, leave exactly the
    state that step leaves, over two rounds with the same pinned buffers refilled in between."""
    dev = need_gpu()
    case = cases.build_sessions(**STREAM_CASE)
    g = torch.Generator(device=dev).manual_seed(5)
    sum_a = sum(case.act_lens)
    q_h = torch.empty(case.n_layers, sum_a, case.hq, case.d, dtype=torch.bfloat16).pin_memory()
    lse_h = torch.empty(case.n_layers, sum_a, case.hq).pin_memory()
    pipes = []
    for host in (False, True):
        cache, pipe = _pipeline(case, dev, 0.9, 0.9, path=path)
        pipe.load(case.tables, case.seq_lens, case.free, 4)
        pipes.append((cache, pipe))
    for rnd, budgets in enumerate([[500, 200, 700], [300, 150, 420]]):
        q = torch.randn(q_h.shape, generator=g, device=dev).to(torch.bfloat16)
        lse = torch.rand(lse_h.shape, generator=g, device=dev) * 2 + 8
        q_h.copy_(q)
        lse_h.copy_(lse)
        states = []
        for host, (cache, pipe) in zip((False, True), pipes):
            pipe.set_round(case.act_lens, budgets)
            if host:
                pipe.step_host(q_h, lse_h)
                pipe.host_inputs_read.synchronize()
            else:
                pipe.step(q, lse)
            torch.cuda.synchronize()
            states.append([pipe.heads.cpu(), pipe.keep_scores.cpu(), pipe.keep.cpu(), pipe.perm.cpu(),
                           cache.kv.cpu(), cache.block_table.cpu(), cache.seq_used.cpu(), cache.free_list.cpu(),
                           cache.free_top.cpu()])
        for a, b in zip(*states):
            assert torch.equal(a, b), f"round {rnd}"
        assert pipes[1][1]._streamed is streamed
    assert_device_clean(dev)
