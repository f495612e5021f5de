"""Algorithm 2 (actkv/budget.py:9-104) in the CPU oracle: the reference's own known answers
(tests/test_algorithms.py:81-113 of actkv-open, restated) and the fixtures recorded by running
the reference (tests/golden/budget.npz, tests/golden/make_golden.py::gen_budget).  Also the
drop-in module's host helpers (trace_confidence, fit_slope) against the same fixtures."""

import numpy as np

from oracle import actkv_oracle as O


def test_token_confidence_higher_when_peaked():
    peaked = np.array([10.0] + [0.0] * 99)
    assert O.token_confidence(peaked, 20) > O.token_confidence(np.zeros(100), 20)


def test_trace_confidence_min_pool_and_bottom_pct():
    x, y = O.trace_confidence(list(range(100, 0, -1)), window=10, stride=5, bottom_pct=50)
    assert x.size > 1 and O.fit_slope(x, y) < 0


def test_budget_grows_on_decline_and_respects_cap():
    b = O.ConfidenceBudget(init_budget=512, scale_up=1.75, upper=1000, window=4, stride=2)
    b.tl = [float(v) for v in range(50, 0, -1)]
    assert b.next_budget() == 896
    assert b.next_budget() == 1000


def test_budget_holds_when_confidence_flat_or_rising():
    b = O.ConfidenceBudget(init_budget=512, window=4, stride=2)
    b.tl = [float(v) for v in range(50)]
    assert b.next_budget() == 512


def test_bidirectional_extension_shrinks_after_patience():
    b = O.ConfidenceBudget(init_budget=1000, window=4, stride=2, bidirectional=True, shrink_patience=2,
                           scale_down=2.0, lower=300)
    b.tl = [float(v) for v in range(50)]
    assert [b.next_budget() for _ in range(4)] == [1000, 500, 500, 300]


def replay(g, t, c, budget_cls):
    """Budgets and slopes of trace t under config c, one next_budget per recorded chunk."""
    meta = g["meta"]
    tl = g[f"trace_{t}"]
    b = budget_cls(**meta["configs"][c])
    n, got, slopes = 0, [], []
    for k in g[f"chunks_{t}"]:
        b.tl.extend(float(v) for v in tl[n:n + k])
        n += k
        got.append(b.next_budget())
        slopes.append(b.slopes[-1])
    return got, slopes


def test_oracle_matches_reference_budget_golden(golden):
    g = golden("budget.npz")
    meta = g["meta"]
    for i in range(meta["n_rows"]):
        got = [O.token_confidence(g[f"logits_{i}"], k) for k in (20, 5)]
        np.testing.assert_allclose(got, g[f"conf_{i}"], rtol=1e-6, atol=1e-5, err_msg=f"row {i}")
    for t in range(meta["n_traces"]):
        for c in range(len(meta["configs"])):
            got, slopes = replay(g, t, c, O.ConfidenceBudget)
            assert got == g[f"budgets_{t}_{c}"].tolist(), (t, c)
            np.testing.assert_allclose(slopes, g[f"slopes_{t}_{c}"], rtol=1e-9, atol=1e-12)


def test_dropin_host_helpers_match_the_oracle(golden):
    import torch

    from actkv_open_b200 import budget as B
    g = golden("budget.npz")
    for t in range(g["meta"]["n_traces"]):
        tl = g[f"trace_{t}"].tolist()
        for window, stride, pct in ((64, 8, 10.0), (4, 2, 50.0), (16, 4, 25.0)):
            x, y = B.trace_confidence(tl, window, stride, pct)
            xo, yo = O.trace_confidence(tl, window, stride, pct)
            np.testing.assert_array_equal(x.numpy(), xo)
            np.testing.assert_array_equal(y.numpy(), yo)
            assert abs(B.fit_slope(x, y) - O.fit_slope(xo, yo)) <= 1e-12
    assert B.fit_slope(torch.zeros(1), torch.zeros(1)) == 0.0
