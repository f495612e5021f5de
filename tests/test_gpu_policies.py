"""FullKV, StreamingLLM and SnapKV (actkv_open_b200.eviction, kernels in csrc/policies.cu) against
the keep indices the reference produced (tests/golden/policies.npz) and the CPU oracle."""
import numpy as np
import pytest
import torch

from gpu_util import assert_device_clean, need_gpu
from oracle import actkv_oracle as O

pytestmark = pytest.mark.gpu


def _rows(g, dev):
    m = g["meta"]
    return [[torch.from_numpy(g[f"row_{i}_{l}"]).to(dev) for l in range(m["n_layers"])] for i in range(m["n_rows"])]


@pytest.mark.parametrize("max_len", [4096, 16])
def test_snapkv_matches_reference_golden(golden, max_len):
    """max_len 16 makes the row ring grow while rows are observed."""
    dev = need_gpu()
    from actkv_open_b200.eviction import SnapKV
    g = golden("policies.npz")
    rows = _rows(g, dev)
    for c, cfg in enumerate(g["meta"]["cases"]):
        pol = SnapKV(**cfg, max_len=max_len)
        pol.reset(3, dev)
        for r in rows[:10]:
            pol.observe(r, True)
        k1 = pol.select(50, 4, 20)
        np.testing.assert_array_equal(k1.cpu().numpy(), g[f"snap_{c}_k1"], err_msg=f"case {c} k1")
        pol.apply_keep(k1)
        for r in rows[10:]:
            pol.observe(r, True)
        k2 = pol.select(30, 4, 12)
        np.testing.assert_array_equal(k2.cpu().numpy(), g[f"snap_{c}_k2"], err_msg=f"case {c} k2")
        assert pol.select(30, 4, 30) is None
    assert_device_clean(dev)


def test_snapkv_rows_follow_apply_keep_like_the_oracle(golden):
    dev = need_gpu()
    from actkv_open_b200.eviction import SnapKV
    g = golden("policies.npz")
    rows = _rows(g, dev)
    pol, ref = SnapKV(window=4, pool=7), O.SnapKV(window=4, pool=7)
    pol.reset(3, dev)
    ref.reset(3)
    for r in rows[:10]:
        pol.observe(r, True)
        ref.observe([x.cpu().numpy() for x in r])
    keep = pol.select(50, 4, 20)
    pol.apply_keep(keep)
    ref.apply_keep(keep.cpu().numpy())
    got = pol.rows
    assert len(got) == len(ref.rows)
    for a, b in zip(got, ref.rows):
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x.cpu().numpy(), y)
    assert_device_clean(dev)


def test_snapkv_without_observed_rows_keeps_the_lowest_indices():
    dev = need_gpu()
    from actkv_open_b200.eviction import SnapKV
    pol, ref = SnapKV(window=4), O.SnapKV(window=4)
    pol.reset(2, dev)
    ref.reset(2)
    np.testing.assert_array_equal(pol.select(40, 3, 10).cpu().numpy(), ref.select(40, 3, 10))
    assert_device_clean(dev)


def test_streaming_and_full_match_reference(golden):
    dev = need_gpu()
    from actkv_open_b200.eviction import FullKV, StreamingLLM
    g = golden("policies.npz")
    st = StreamingLLM()
    st.reset(3, dev)
    np.testing.assert_array_equal(st.select(50, 4, 20).cpu().numpy(), g["stream_k"])
    assert st.select(24, 4, 20) is None
    full = FullKV()
    full.reset(3, dev)
    assert full.select(50, 4, 20) is None
    assert_device_clean(dev)


def test_protected_prefix_always_kept():
    """The reference's test (tests/test_algorithms.py:70-78) with every policy on the device."""
    dev = need_gpu()
    from actkv_open_b200.eviction import ActionLRFU, SnapKV, StreamingLLM
    for pol in (ActionLRFU(), StreamingLLM(), SnapKV(window=2)):
        pol.reset(2, dev)
        pol.begin_action()
        for _ in range(3):
            pol.observe([torch.rand(20, device=dev), torch.rand(20, device=dev)], True)
        keep = pol.select(20, protected=5, budget=6)
        assert keep.shape == (2, 11)
        assert (keep[:, :5].cpu() == torch.arange(5)).all()
    assert_device_clean(dev)
