"""The reference's hand-worked known answers (actkv-open tests/test_algorithms.py and
tests/test_kernels.py), restated against the CPU oracle so the oracle is pinned by them too."""
import math

import numpy as np

import cases
from oracle import actkv_oracle as O


def test_reduce_heads_max_over_group_then_mean():          # test_algorithms.py:8-12
    attn = np.array([[0.1, 0.9], [0.5, 0.2], [0.3, 0.3], [0.0, 0.6]], np.float32)
    np.testing.assert_allclose(O.reduce_heads(attn, 2, "mean"), [(0.5 + 0.3) / 2, (0.9 + 0.6) / 2], rtol=1e-6)


def test_top_p_mask_is_nucleus():                           # test_algorithms.py:15-18
    s = np.array([0.5, 0.05, 0.3, 0.15, 0.0], np.float32)
    assert O.top_p_mask(s, 0.9).tolist() == [True, False, True, True, False]


def test_lrfu_update_matches_algorithm_1():                 # test_algorithms.py:21-33
    pol = O.ActionLRFU(decay=0.5, top_p=0.9)
    pol.reset(1)
    pol.begin_action()
    pol.observe([np.array([0.05, 0.05, 0.8, 0.1], np.float32)], True)
    pol.update_scores(4, 0)
    np.testing.assert_allclose(pol.ks[0], [0.0, 0.0, 0.8, 0.1], rtol=1e-6)
    pol.begin_action()
    pol.observe([np.array([0.0, 0.0, 0.0, 0.05, 0.95, 0.0], np.float32)], True)
    pol.update_scores(6, 0)
    np.testing.assert_allclose(pol.ks[0], [0.0, 0.0, 0.4, 0.05, 0.95, 0.0], rtol=1e-6)


def test_lrfu_round_without_action_only_decays():           # test_algorithms.py:36-44
    pol = O.ActionLRFU(decay=0.5, top_p=0.9)
    pol.reset(1)
    pol.begin_action()
    pol.observe([np.array([0.05, 0.05, 0.8, 0.1], np.float32)], True)
    pol.update_scores(4, 0)
    pol.update_scores(6, 0)
    np.testing.assert_allclose(pol.ks[0], [0.0, 0.0, 0.4, 0.05, 0.0, 0.0], rtol=1e-6)


def test_lrfu_keeps_intermittent_entry_over_fresh_miss():   # test_algorithms.py:47-57
    pol = O.ActionLRFU(decay=0.5)
    pol.reset(1)
    pol.begin_action()
    pol.observe([np.array([0.9, 0.1, 0.0], np.float32)], True)
    pol.select(3, 0, budget=3)
    pol.begin_action()
    pol.observe([np.array([0.0, 0.2, 0.0, 0.8, 0.0], np.float32)], True)
    assert pol.select(5, 0, budget=2)[0].tolist() == [0, 3]


def test_action_mean_ignores_non_action_tokens():            # test_algorithms.py:60-67
    pol = O.ActionLRFU()
    pol.reset(1)
    pol.begin_action()
    pol.observe([np.array([1.0, 0.0], np.float32)], False)
    pol.observe([np.array([0.0, 1.0], np.float32)], True)
    pol.observe([np.array([0.0, 0.5, 0.5], np.float32)], True)
    np.testing.assert_allclose(pol.act[0], [0.0, 0.75, 0.25], rtol=1e-6)


def test_protected_prefix_always_kept():                     # test_algorithms.py:70-78
    pol = O.ActionLRFU()
    pol.reset(2)
    pol.begin_action()
    rng = np.random.default_rng(0)
    for _ in range(3):
        pol.observe([rng.random(20, dtype=np.float32), rng.random(20, dtype=np.float32)], True)
    keep = pol.select(20, protected=5, budget=6)
    assert keep.shape == (2, 11)
    assert (keep[:, :5] == np.arange(5)).all()


def _filled(lens, bs=16, hkv=2, d=32, layers=1, seed=0):
    case = cases.build_sessions(seed, layers, hkv, hkv, d, bs, lens, [1] * len(lens))
    c = O.PagedKVCache(case.num_blocks, bs, hkv, d, layers)
    c.kv[:] = cases.to_np(case.kv)
    c.free = list(case.free)
    for r, n in enumerate(lens):
        c.tables[r] = list(case.tables[r])
        c.seq_used[r] = n
    return c


def test_recovered_scores_are_probabilities():               # test_kernels.py:58-66
    c = _filled([50], hkv=1, d=16)
    bt, seq = c.block_table([0]), c.seq_tensor([0])
    q = np.random.default_rng(1).standard_normal((1, 1, 16)).astype(np.float32)
    _, lse = O.paged_decode_attention(q, c.kv[0], bt, seq)
    out = np.zeros((1, 1, bt.shape[1] * 16), np.float32)
    O.action_scores(q, c.kv[0], bt, seq, lse, out, np.zeros(1, np.int32))
    assert abs(float(out[0, 0, :50].sum()) - 1.0) < 1e-4
    assert float(np.abs(out[0, 0, 50:]).sum()) == 0.0


def test_plan_is_conflict_free():                            # test_kernels.py:80-91
    rng = np.random.default_rng(3)
    for seq_used, budget, bs in [(100, 40, 16), (17, 10, 16), (64, 64, 16), (200, 3, 8)]:
        keep = np.zeros(seq_used, bool)
        keep[rng.permutation(seq_used)[:budget]] = True
        table = rng.permutation(math.ceil(seq_used / bs) + 4)
        plan = O.plan_compaction(keep, seq_used, table, bs)
        src, dst = set(plan.src_slots.tolist()), set(plan.dst_slots.tolist())
        assert not (src & dst)
        assert len(src) == len(plan.src_slots) and len(dst) == len(plan.dst_slots)
        assert sorted(plan.perm.tolist()) == sorted(np.nonzero(keep)[0].tolist())
        assert plan.drop_blocks == math.ceil(seq_used / bs) - math.ceil(budget / bs)


def test_evict_keeps_the_protected_prefix_and_the_top_scored_tokens():   # test_kernels.py:157-168
    c = _filled([70], hkv=2, d=16, layers=2)
    k_before, v_before = c.gather(0, layer=1)
    scores = 0.1 * np.random.default_rng(3).random((2, 2, 70), dtype=np.float32)
    hot = [5, 17, 40, 69]
    scores[..., hot] += 1.0
    perm = c.evict(0, scores, budget=4, protected=3)
    assert sorted(perm.tolist()) == [0, 1, 2, *hot]
    k_after, v_after = c.gather(0, layer=1)
    np.testing.assert_array_equal(k_after, k_before[perm])
    np.testing.assert_array_equal(v_after, v_before[perm])
    assert c.seq_used[0] == 7 and len(c.tables[0]) == 1


def test_evict_within_budget_is_a_no_op():                   # test_kernels.py:171-175
    c = _filled([20])
    table = list(c.tables[0])
    assert c.evict(0, np.random.default_rng(0).random((2, 20)), budget=20).tolist() == list(range(20))
    assert c.tables[0] == table and c.seq_used[0] == 20


def test_keep_mask_reduces_heads_then_averages_layers():     # test_kernels.py:178-183
    scores = np.zeros((2, 2, 4), np.float32)
    scores[0, 0, 1] = 1.0
    scores[:, :, 2] = 0.3
    assert O.keep_mask_from_scores(scores, 4, budget=1).tolist() == [False, False, True, False]
    assert O.keep_mask_from_scores(scores, 4, budget=1, head_reduce="max").tolist() == [False, True, False, False]


def test_compaction_frees_blocks():                          # test_kernels.py:122-135
    for n, budget in [(150, 60), (40, 39), (33, 16)]:
        c = _filled([n], layers=2)
        k_before = [c.gather(0, l)[0].copy() for l in range(2)]
        used = c.used_blocks
        keep = np.zeros(n, bool)
        keep[np.random.default_rng(n).permutation(n)[:budget]] = True
        perm = c.compact(0, keep)
        assert c.seq_used[0] == budget
        for l in range(2):
            np.testing.assert_array_equal(c.gather(0, l)[0], k_before[l][perm])
        assert used - c.used_blocks == math.ceil(n / 16) - math.ceil(budget / 16)
