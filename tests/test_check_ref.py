"""The torch restatement that checks full-size GPU steps (actkv_open_b200.check) against the pinned
CPU oracle, on CPU tensors: region scores, nucleus, top-k and the compaction plan must agree."""
import numpy as np
import torch

import cases
from oracle import actkv_oracle as O


def test_region_scores_ref_matches_the_oracle():
    from actkv_open_b200 import check
    case = cases.build_sessions(seed=5, n_layers=2, hq=8, hkv=2, d=64, bs=16, seq_lens=[300, 77],
                                act_lens=[9, 5], dtype="float32", extra_blocks=3)
    kv_np = cases.to_np(case.kv)
    for r, n in enumerate(case.seq_lens):
        q = cases.to_np(case.q[r])
        bt = np.asarray(case.tables[r], np.int64)
        lse = np.stack([O.causal_region_lse(q[l], kv_np[l], bt, n) for l in range(case.n_layers)])
        want = np.stack([O.layer_scores(kv_np[l], bt, n, q[l], lse[l]) for l in range(case.n_layers)])
        got = check.region_scores_ref(case.kv, torch.tensor(case.tables[r], dtype=torch.int32), n, case.q[r],
                                      torch.from_numpy(lse), chunk=64)
        np.testing.assert_allclose(got.numpy(), want, rtol=1e-5, atol=1e-12)


def test_nucleus_and_topk_match_the_oracle():
    from actkv_open_b200 import check
    rng = np.random.default_rng(0)
    for n in (1, 7, 500, 4096):
        a = rng.random(n).astype(np.float32) ** 4
        a[rng.random(n) < 0.1] = 0.0
        got = check.nucleus_ref(torch.from_numpy(a), 0.9).numpy()
        np.testing.assert_array_equal(got, O.top_p_mask(a, 0.9))
        s = np.round(rng.random(n) * 50).astype(np.float32)            # many exact ties
        free = rng.random(n) < 0.8
        k = n // 3
        got = check.topk_mask_ref(torch.from_numpy(s), torch.from_numpy(free), k).numpy()
        want = np.zeros(n, bool)
        idx = np.nonzero(free)[0]
        want[idx[O.topk_lowest_index(s[idx], min(k, idx.size))]] = True
        np.testing.assert_array_equal(got, want)
    assert not check.nucleus_ref(torch.zeros(5), 0.9).any()


def test_plan_ref_matches_the_oracle_plan():
    from actkv_open_b200 import check
    rng = np.random.default_rng(1)
    for n, bs in ((1, 16), (37, 8), (500, 16), (4096, 16), (1000, 32)):
        table = rng.permutation(4 * (n // bs + 1))[: -(-n // bs)].astype(np.int64)
        for kind in range(4):
            keep = [rng.random(n) < 0.3, np.ones(n, bool), np.arange(n) < min(4, n), np.arange(n) % bs == 0][kind]
            src, dst, perm, drop = check.plan_ref(torch.from_numpy(keep), n, torch.from_numpy(table), bs)
            p = O.plan_compaction(keep, n, table, bs)
            np.testing.assert_array_equal(src.numpy(), p.src_slots)
            np.testing.assert_array_equal(dst.numpy(), p.dst_slots)
            np.testing.assert_array_equal(perm.numpy(), p.perm)
            assert drop == p.drop_blocks
