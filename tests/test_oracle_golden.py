"""Pins the CPU oracle (oracle/actkv_oracle.py) to the reference's own outputs: every fixture in
tests/golden was produced by running actkv-open's torch path (tests/golden/make_golden.py)."""
import json
import math

import numpy as np
import pytest
import torch

import cases
from conftest import assert_masks_match
from oracle import actkv_oracle as O


def _case_from(meta_shape, seed):
    lens, hq, hkv, d, bs = meta_shape
    return cases.build_sessions(seed, 1, hq, hkv, d, bs, lens, [3] * len(lens))


def test_scores_match_reference_running_mean(golden):
    g = golden("scores_small.npz")
    for i, shape in enumerate(g["meta"]["shapes"]):
        p = f"c{i}_"
        case = _case_from(shape, 100 + i)
        assert cases.digest(case.kv) == str(g[p + "kv_sha"])
        kv = cases.to_np(case.kv)[0]
        out = np.zeros_like(g[p + "out"])
        ns = np.zeros_like(g[p + "n_seen"])
        for step in range(3):
            q = g[p + "q"][step]
            _, lse = O.paged_decode_attention(q, kv, g[p + "bt"], g[p + "seq"])
            np.testing.assert_allclose(lse, g[p + "lse"][step], rtol=1e-5, atol=1e-5)
            O.action_scores(q, kv, g[p + "bt"], g[p + "seq"], g[p + "lse"][step], out, ns)
        np.testing.assert_allclose(out, g[p + "out"], rtol=1e-5, atol=1e-7)
        np.testing.assert_array_equal(ns, g[p + "n_seen"])


def test_plans_match_reference(golden):
    g = golden("plans.npz")
    for i, (n, bs, name) in enumerate(g["meta"]["cases"]):
        p = f"p{i}_"
        plan = O.plan_compaction(g[p + "keep"], n, g[p + "table"], bs)
        np.testing.assert_array_equal(plan.src_slots, g[p + "src"], err_msg=name)
        np.testing.assert_array_equal(plan.dst_slots, g[p + "dst"], err_msg=name)
        np.testing.assert_array_equal(plan.perm, g[p + "perm"], err_msg=name)
        assert plan.drop_blocks == int(g[p + "drop"])


def test_cache_compaction_matches_reference(golden):
    g = golden("compact.npz")
    specs = [([150], 2, 16), ([40], 2, 16), ([33, 70, 5], 2, 16), ([200, 64], 3, 8)]
    for i, (lens, layers, bs) in enumerate(specs):
        p = f"m{i}_"
        case = cases.build_sessions(300 + i, layers, 4, 2, 32, bs, lens, [1] * len(lens))
        assert cases.digest(case.kv) == str(g[p + "kv0_sha"])
        c = O.PagedKVCache(case.num_blocks, bs, 2, 32, layers)
        c.kv[:] = cases.to_np(case.kv)
        c.free = list(case.free)
        for r, n in enumerate(lens):
            c.tables[r] = list(case.tables[r])
            c.seq_used[r] = n
        for r in range(len(lens)):
            perm = c.compact(r, g[p + f"keep_{r}"])
            np.testing.assert_array_equal(perm, g[p + f"perm_{r}"])
            assert c.tables[r] == list(g[p + f"table1_{r}"])
            assert c.seq_used[r] == int(g[p + f"seq1_{r}"])
        assert c.free == list(g[p + "free1"])
        assert cases.digest(torch.from_numpy(c.kv)) == str(g[p + "kv1_sha"])


def test_keep_masks_match_reference(golden):
    g = golden("keep_masks.npz")
    for i, (shp, how, prot_kind, budget, si) in enumerate(g["meta"]["cases"]):
        p = f"k{i}_"
        scores = g[f"scores{si}"]
        n = shp[-1]
        prot = g[p + "prot"]
        prot = prot.astype(bool) if prot_kind == "mask" else int(prot)
        got = O.keep_mask_from_scores(scores, n, budget, prot, how)
        s = scores.astype(np.float32)
        if s.ndim >= 2:
            s = s.max(-2) if how == "max" else s.mean(-2)
            s = s.reshape(-1, n).mean(0)
        assert_masks_match(got, g[p + "keep"], s, rtol=1e-6)


def test_top_p_and_lrfu_trace_match_reference(golden):
    g = golden("lrfu.npz")
    for i, (n, p) in enumerate(g["meta"]["top_p"]):
        got = O.top_p_mask(g[f"t{i}_s"], p)
        np.testing.assert_array_equal(got, g[f"t{i}_mask"], err_msg=f"top_p n={n} p={p}")
    np.testing.assert_allclose(O.reduce_heads(g["rh_attn"], 2, "mean"), g["rh_mean"], rtol=1e-6)
    np.testing.assert_array_equal(O.reduce_heads(g["rh_attn"], 2, "max"), g["rh_max"])
    pol = O.ActionLRFU(decay=0.9, top_p=0.9)
    pol.reset(3)
    for rnd in range(g["meta"]["rounds"]):
        key = f"r{rnd}_"
        pol.begin_action()
        for obs in g[key + "obs"]:
            pol.observe(list(obs), True)
        keep = pol.select(int(g[key + "length"]), 2, 30)
        np.testing.assert_allclose(pol.ks, g[key + "ks"], rtol=1e-6, atol=1e-7)
        if keep is None:
            assert g[key + "keep"].size == 0
            continue
        np.testing.assert_array_equal(keep, g[key + "keep"])
        pol.apply_keep(keep)
        np.testing.assert_allclose(pol.ks, g[key + "ks_after"], rtol=1e-6, atol=1e-7)


def test_multi_round_evict_matches_reference(golden):
    g = golden("evict.npz")
    case = cases.build_sessions(500, 2, 4, 2, 16, 16, [90, 45], [1, 1], extra_blocks=20)
    assert cases.digest(case.kv) == str(g["kv0_sha"])
    c = O.PagedKVCache(case.num_blocks, 16, 2, 16, 2)
    c.kv[:] = cases.to_np(case.kv)
    c.free = list(case.free)
    for r, n in enumerate([90, 45]):
        c.tables[r] = list(case.tables[r])
        c.seq_used[r] = n
    for step in range(g["meta"]["steps"]):
        key = f"s{step}_"
        r = int(g[key + "req"])
        perm = c.evict(r, g[key + "scores"], int(g[key + "budget"]), protected=5)
        np.testing.assert_array_equal(perm, g[key + "perm"])
        np.testing.assert_array_equal(c.pinned[r], g[key + "pinned"])
        assert c.tables[r] == list(g[key + "table"])
        assert c.free == list(g[key + "free"])
        assert cases.digest(torch.from_numpy(c.kv)) == str(g[key + "kv_sha"])
        c.append(r, g[key + "newk"], g[key + "newv"])


@pytest.mark.parametrize("name,spec,protected,budgets,decay,top_p", [
    ("config1.npz", cases.CONFIG1, cases.CONFIG1_PROTECTED, [cases.CONFIG1_BUDGET],
     cases.CONFIG1_DECAY, cases.CONFIG1_TOP_P),
    ("pipe_bf16.npz", cases.PIPE_BF16, cases.PIPE_BF16_PROTECTED, cases.PIPE_BF16_BUDGETS,
     cases.PIPE_BF16_DECAY, cases.PIPE_BF16_TOP_P),
])
def test_pipeline_matches_reference(golden, name, spec, protected, budgets, decay, top_p):
    """Score -> ActionLRFU -> keep mask -> compaction, end to end, against the reference."""
    g = golden(name)
    case = cases.build_sessions(**spec)
    assert cases.digest(case.kv) == g["meta"]["kv_sha256_in"]
    c = O.PagedKVCache(case.num_blocks, case.bs, case.hkv, case.d, case.n_layers)
    c.kv[:] = cases.to_np(case.kv)
    c.free = list(case.free)
    for r, n in enumerate(case.seq_lens):
        c.tables[r] = list(case.tables[r])
        c.seq_used[r] = n
    for r, (n, a) in enumerate(zip(case.seq_lens, case.act_lens)):
        q = cases.to_np(case.q[r])
        lse = np.stack([O.causal_region_lse(q[l], c.kv[l], np.asarray(c.tables[r]), n)
                        for l in range(case.n_layers)])
        np.testing.assert_allclose(lse, g[f"lse_{r}"], rtol=1e-5, atol=1e-5)
        pol = O.ActionLRFU(decay=decay, top_p=top_p)
        pol.reset(case.n_layers)
        perm, heads = O.evict_session(c, pol, r, q, g[f"lse_{r}"], budgets[r], protected)
        np.testing.assert_allclose(heads, g[f"heads_{r}"], rtol=1e-4, atol=1e-9)
        np.testing.assert_array_equal(perm, g[f"perm_{r}"])
        np.testing.assert_allclose(pol.ks, g[f"ks_after_{r}"], rtol=1e-4, atol=1e-9)
        assert c.tables[r] == list(g[f"table_{r}"])
        assert c.seq_used[r] == int(g[f"seq_{r}"])
        np.testing.assert_array_equal(c.pinned[r], g[f"pinned_{r}"])
    assert c.free == list(g["free"])
    assert cases.digest(torch.from_numpy(c.kv).to(cases.DTYPES[case.dtype])) == g["meta"]["kv_sha256_out"]
