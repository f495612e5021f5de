"""StreamingLLM and SnapKV (actkv/eviction.py:89-149) in the CPU oracle against the keep indices
the reference itself produced (tests/golden/policies.npz, tests/golden/make_golden.py::
gen_policies), and the reference's protected-prefix test (tests/test_algorithms.py:70-78)."""
import numpy as np

from oracle import actkv_oracle as O


def golden_rows(g):
    return [[g[f"row_{i}_{layer}"] for layer in range(g["meta"]["n_layers"])] for i in range(g["meta"]["n_rows"])]


def test_protected_prefix_always_kept():
    rng = np.random.default_rng(0)
    for pol in (O.StreamingLLM(), O.SnapKV(window=2)):
        pol.reset(2)
        for _ in range(3):
            if isinstance(pol, O.SnapKV):
                pol.observe([rng.random(20, dtype=np.float32), rng.random(20, dtype=np.float32)])
        keep = pol.select(20, 5, 6)
        assert keep.shape == (2, 11)
        assert (keep[:, :5] == np.arange(5)).all()


def test_oracle_policies_match_reference_golden(golden):
    g = golden("policies.npz")
    rows = golden_rows(g)
    for c, cfg in enumerate(g["meta"]["cases"]):
        pol = O.SnapKV(**cfg)
        pol.reset(3)
        for r in rows[:10]:
            pol.observe(r)
        k1 = pol.select(50, 4, 20)
        np.testing.assert_array_equal(k1, g[f"snap_{c}_k1"])
        pol.apply_keep(k1)
        for r in rows[10:]:
            pol.observe(r)
        np.testing.assert_array_equal(pol.select(30, 4, 12), g[f"snap_{c}_k2"])
        assert pol.select(30, 4, 30) is None and bool(g[f"snap_{c}_none"])
    st = O.StreamingLLM()
    st.reset(3)
    np.testing.assert_array_equal(st.select(50, 4, 20), g["stream_k"])
    assert st.select(24, 4, 20) is None and bool(g["stream_none"])
