"""GPU parity of keep-mask selection (actkv/paged.py:23-46) and the ActionLRFU update with its
nucleus (actkv/eviction.py:36-50,198-224) against the reference's golden outputs and known answers.
Selections are bit-exact on the same inputs except where the reference itself leaves the order of
exact ties unspecified; those are checked as near-ties."""
import numpy as np
import pytest
import torch

from conftest import assert_masks_match
from gpu_util import assert_device_clean, need_gpu

pytestmark = pytest.mark.gpu


def test_keep_masks_match_reference_golden(golden):
    dev = need_gpu()
    from actkv_open_b200.paged import keep_mask_from_scores
    g = golden("keep_masks.npz")
    for i, (shp, how, prot_kind, budget, si) in enumerate(g["meta"]["cases"]):
        p = f"k{i}_"
        scores = g[f"scores{si}"]
        n = shp[-1]
        prot = g[p + "prot"]
        prot = torch.from_numpy(prot.astype(bool)).to(dev) if prot_kind == "mask" else int(prot)
        got = keep_mask_from_scores(torch.from_numpy(scores).to(dev), n, budget, prot, how).cpu().numpy()
        s = scores.astype(np.float32)
        if s.ndim >= 2:
            s = s.max(-2) if how == "max" else s.mean(-2)
            s = s.reshape(-1, n).mean(0)
        assert_masks_match(got, g[p + "keep"], s, rtol=1e-6, what=f"case {i} {shp} {how} {prot_kind}")
    assert_device_clean(dev)


def test_keep_mask_reduces_heads_then_averages_layers():          # test_kernels.py:178-183
    dev = need_gpu()
    from actkv_open_b200.paged import keep_mask_from_scores
    scores = torch.zeros(2, 2, 4, device=dev)
    scores[0, 0, 1] = 1.0
    scores[:, :, 2] = 0.3
    assert keep_mask_from_scores(scores, 4, budget=1).tolist() == [False, False, True, False]
    assert keep_mask_from_scores(scores, 4, budget=1, head_reduce="max").tolist() == [False, True, False, False]
    with pytest.raises(ValueError):
        keep_mask_from_scores(scores, 4, budget=1, head_reduce="median")


def test_keep_mask_ties_keep_the_lowest_index():
    dev = need_gpu()
    from actkv_open_b200.paged import keep_mask_from_scores
    s = torch.tensor([0.5, 0.2, 0.2, 0.9, 0.2, 0.2, 0.0], device=dev)
    assert keep_mask_from_scores(s, 7, 3).tolist() == [True, True, False, True, False, False, False]
    z = torch.zeros(40, device=dev)                                # all tied at zero
    m = keep_mask_from_scores(z, 40, 10, protected=3)
    assert m.tolist() == [True] * 13 + [False] * 27
    neg = torch.tensor([-1.0, -0.0, 0.0, -3.0, 2.0], device=dev)  # -0.0 == 0.0, negatives order
    assert keep_mask_from_scores(neg, 5, 3).tolist() == [False, True, True, False, True]


def test_keep_mask_edge_budgets():
    dev = need_gpu()
    from actkv_open_b200.paged import keep_mask_from_scores
    s = torch.rand(100, generator=torch.Generator().manual_seed(0)).to(dev)
    assert keep_mask_from_scores(s, 100, 0, protected=5).sum().item() == 5
    assert keep_mask_from_scores(s, 100, 95, protected=5).all()
    assert keep_mask_from_scores(s, 100, 500).all()
    assert keep_mask_from_scores(s, 1, 1).tolist() == [True]
    big = torch.rand(3, 8, 40000, generator=torch.Generator().manual_seed(1)).to(dev)
    got = keep_mask_from_scores(big, 40000, 4000, protected=4).cpu().numpy()
    from oracle import actkv_oracle as O
    want = O.keep_mask_from_scores(big.cpu().numpy(), 40000, 4000, 4)
    sref = big.cpu().numpy().mean(-2).mean(0)
    assert_masks_match(got, want, sref, rtol=1e-6)
    assert_device_clean(dev)


def test_top_p_masks_match_reference_golden(golden):
    dev = need_gpu()
    from actkv_open_b200.eviction import top_p_mask
    g = golden("lrfu.npz")
    for i, (n, p) in enumerate(g["meta"]["top_p"]):
        got = top_p_mask(torch.from_numpy(g[f"t{i}_s"]).to(dev), p).cpu().numpy()
        np.testing.assert_array_equal(got, g[f"t{i}_mask"], err_msg=f"n={n} p={p}")
    s = torch.tensor([0.5, 0.05, 0.3, 0.15, 0.0], device=dev)        # test_algorithms.py:15-18
    assert top_p_mask(s, 0.9).tolist() == [True, False, True, True, False]
    assert not top_p_mask(torch.zeros(5, device=dev), 0.9).any()
    assert_device_clean(dev)


def test_lrfu_trace_matches_reference_golden(golden):
    dev = need_gpu()
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.eviction import ActionLRFU
    g = golden("lrfu.npz")
    pol = ActionLRFU(EvictionConfig(decay=0.9, top_p=0.9))
    pol.reset(3, device=dev)
    for rnd in range(g["meta"]["rounds"]):
        key = f"r{rnd}_"
        pol.begin_action()
        for obs in g[key + "obs"]:
            pol.observe([torch.from_numpy(o).to(dev) for o in obs], True)
        keep = pol.select(int(g[key + "length"]), 2, 30)
        torch.testing.assert_close(pol.ks.cpu(), torch.from_numpy(g[key + "ks"]), rtol=1e-5, atol=1e-7)
        if keep is None:
            assert g[key + "keep"].size == 0
            continue
        np.testing.assert_array_equal(keep.cpu().numpy(), g[key + "keep"])
        pol.apply_keep(keep)
        torch.testing.assert_close(pol.ks.cpu(), torch.from_numpy(g[key + "ks_after"]), rtol=1e-5, atol=1e-7)
    assert_device_clean(dev)


def test_lrfu_known_answers():                                     # test_algorithms.py:21-78
    dev = need_gpu()
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.eviction import ActionLRFU, reduce_heads
    t = lambda *v: torch.tensor(v, device=dev)  # noqa: E731
    pol = ActionLRFU(EvictionConfig(decay=0.5, top_p=0.9))
    pol.reset(1, device=dev)
    pol.begin_action()
    pol.observe([t(0.05, 0.05, 0.8, 0.1)], True)
    pol.update_scores(4, 0)
    torch.testing.assert_close(pol.ks[0], t(0.0, 0.0, 0.8, 0.1))
    pol.begin_action()
    pol.observe([t(0.0, 0.0, 0.0, 0.05, 0.95, 0.0)], True)
    pol.update_scores(6, 0)
    torch.testing.assert_close(pol.ks[0], t(0.0, 0.0, 0.4, 0.05, 0.95, 0.0))
    pol.update_scores(6, 0)                                         # a round without action only decays
    torch.testing.assert_close(pol.ks[0], t(0.0, 0.0, 0.2, 0.025, 0.475, 0.0))
    pol = ActionLRFU(EvictionConfig(decay=0.5))
    pol.reset(1, device=dev)
    pol.begin_action()
    pol.observe([t(0.9, 0.1, 0.0)], True)
    pol.select(3, 0, budget=3)
    pol.begin_action()
    pol.observe([t(0.0, 0.2, 0.0, 0.8, 0.0)], True)
    assert pol.select(5, 0, budget=2)[0].tolist() == [0, 3]
    pol = ActionLRFU()
    pol.reset(2, device=dev)
    pol.begin_action()
    for _ in range(3):
        pol.observe([torch.rand(20, device=dev), torch.rand(20, device=dev)], True)
    keep = pol.select(20, protected=5, budget=6)
    assert keep.shape == (2, 11) and (keep[:, :5].cpu() == torch.arange(5)).all()
    attn = t([0.1, 0.9], [0.5, 0.2], [0.3, 0.3], [0.0, 0.6])
    torch.testing.assert_close(reduce_heads(attn, 2, "mean"), t((0.5 + 0.3) / 2, (0.9 + 0.6) / 2))
    assert_device_clean(dev)


def test_lrfu_update_with_pinned_mask_and_heads_matches_oracle():
    """The batched kernel: per-head input reduced on the fly, pinned tokens excluded, many rows."""
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    from oracle import actkv_oracle as O
    rng = np.random.default_rng(5)
    R, L, H, W = 3, 4, 8, 3000
    lens = [3000, 1777, 64]
    heads = (rng.random((R, L, H, W), dtype=np.float32) ** 6).astype(np.float32)
    ks0 = (rng.random((R, L, W), dtype=np.float32) * 1e-3).astype(np.float32)
    pinned = (rng.random((R, W)) < 0.05).astype(np.uint8)
    hs = torch.from_numpy(heads).to(dev)
    ks = torch.from_numpy(ks0).to(dev)
    act = torch.zeros(R, L, W, device=dev)
    pin = torch.from_numpy(pinned).to(dev)
    seq = torch.tensor(lens, dtype=torch.int32, device=dev)
    N.check(N.load().actkv_lrfu_update(hs.data_ptr(), None, hs.stride(0), hs.stride(1), hs.stride(2), H, 0,
                                       ks.data_ptr(), ks.stride(0), ks.stride(1), act.data_ptr(), act.stride(0),
                                       act.stride(1), pin.data_ptr(), pin.stride(0), 0, seq.data_ptr(), None,
                                       R, L, W, 0.9, 0.9, N.status_word(dev).data_ptr(), N.stream_ptr(dev)))
    got_ks, got_act = ks.cpu().numpy(), act.cpu().numpy()
    for r, n in enumerate(lens):
        a = heads[r, :, :, :n].mean(1, dtype=np.float32)
        np.testing.assert_allclose(got_act[r, :, :n], a, rtol=1e-6)
        pol = O.ActionLRFU(decay=0.9, top_p=0.9)
        pol.reset(L)
        pol.ks = ks0[r, :, :n].copy()
        pol.act = got_act[r, :, :n].copy()            # the same inputs: selection must agree exactly
        pol.n_act = 1
        pol.update_scores(n, pinned[r, :n].astype(bool))
        np.testing.assert_array_equal(got_ks[r, :, :n], pol.ks, err_msg=f"session {r}")
        np.testing.assert_array_equal(got_ks[r, :, n:], ks0[r, :, n:])
    assert_device_clean(dev)


def test_lrfu_ties_across_cluster_slices_match_oracle():
    """Few distinct values, so that the nucleus boundary falls on a key shared by tokens in every
    CTA slice of a row's cluster (ties go to the lowest index), at several top_p."""
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    from oracle import actkv_oracle as O
    rng = np.random.default_rng(11)
    R, L, H, W = 3, 3, 2, 4099
    lens = [4099, 2050, 9]
    levels = np.array([0.0, 1e-4, 2.5e-4, 5e-4, 1e-3], np.float32)
    heads = levels[rng.integers(0, len(levels), (R, L, H, W))].astype(np.float32)
    for top_p in (0.9, 0.5, 0.999):
        ks0 = (rng.random((R, L, W), dtype=np.float32) * 1e-3).astype(np.float32)
        hs = torch.from_numpy(heads).to(dev)
        ks = torch.from_numpy(ks0).to(dev)
        act = torch.zeros(R, L, W, device=dev)
        seq = torch.tensor(lens, dtype=torch.int32, device=dev)
        N.check(N.load().actkv_lrfu_update(hs.data_ptr(), None, hs.stride(0), hs.stride(1), hs.stride(2), H, 0,
                                           ks.data_ptr(), ks.stride(0), ks.stride(1), act.data_ptr(),
                                           act.stride(0), act.stride(1), None, 0, 3, seq.data_ptr(), None,
                                           R, L, W, 0.5, top_p, N.status_word(dev).data_ptr(), N.stream_ptr(dev)))
        got_ks, got_act = ks.cpu().numpy(), act.cpu().numpy()
        for r, n in enumerate(lens):
            pol = O.ActionLRFU(decay=0.5, top_p=top_p)
            pol.reset(L)
            pol.ks = ks0[r, :, :n].copy()
            pol.act = got_act[r, :, :n].copy()
            pol.n_act = 1
            pol.update_scores(n, 3)
            np.testing.assert_array_equal(got_ks[r, :, :n], pol.ks, err_msg=f"session {r} top_p {top_p}")
            np.testing.assert_array_equal(got_ks[r, :, n:], ks0[r, :, n:])
    assert_device_clean(dev)
