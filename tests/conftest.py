import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name):
    import json
    z = np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    data = {k: z[k] for k in z.files}
    data["meta"] = json.loads(str(data["meta"]))
    return data


@pytest.fixture(scope="session")
def golden():
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = load_golden(name)
        return cache[name]
    return get


def assert_masks_match(got, want, scores=None, rtol=1e-3, what="mask"):
    """Equal bool masks, except entries whose score sits within ``rtol`` of the selection
    threshold (the smallest kept score): there the two sides may break a near-tie differently."""
    got = np.asarray(got, bool)
    want = np.asarray(want, bool)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    diff = np.nonzero(got != want)[0]
    if diff.size == 0:
        return
    assert scores is not None, f"{what}: {diff.size} entries differ at {diff[:10]}"
    s = np.asarray(scores, np.float64)
    assert got.sum() == want.sum(), f"{what}: kept counts differ {got.sum()} vs {want.sum()}"
    thr = s[want].min() if want.any() else 0.0
    near = np.abs(s[diff] - thr) <= rtol * max(abs(thr), 1e-30)
    assert near.all(), f"{what}: {diff[~near][:10]} differ and are not near-ties (thr={thr})"
