"""Algorithm 2 on the device (actkv_token_confidence, actkv_budget_update through
actkv_open_b200.budget) against the fixtures recorded by running the reference
(tests/golden/budget.npz) and the CPU oracle."""
import math

import numpy as np
import pytest
import torch

from gpu_util import assert_device_clean, need_gpu
from oracle import actkv_oracle as O

pytestmark = pytest.mark.gpu


def test_token_confidence_matches_reference_golden(golden):
    dev = need_gpu()
    from actkv_open_b200.budget import token_confidence
    g = golden("budget.npz")
    for i in range(g["meta"]["n_rows"]):
        x = torch.from_numpy(g[f"logits_{i}"]).to(dev)
        got = [token_confidence(x, k) for k in (20, 5)]
        np.testing.assert_allclose(got, g[f"conf_{i}"], rtol=2e-6, atol=2e-5, err_msg=f"row {i}")
    assert_device_clean(dev)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_token_confidence_of_half_logits_matches_the_oracle(dtype):
    dev = need_gpu()
    from actkv_open_b200.budget import token_confidence
    g = torch.Generator().manual_seed(5)
    for V, scale in ((151_936, 3.0), (32_000, 1.0), (257, 6.0)):
        x = (torch.randn(V, generator=g) * scale).to(dtype)
        want = O.token_confidence(x.float().numpy(), 20)
        assert abs(token_confidence(x.to(dev), 20) - want) <= 2e-5 + 2e-6 * abs(want)
    assert_device_clean(dev)


def _budgets(n, cfg, dev, capacity=4096):
    from actkv_open_b200.budget import SessionBudgets
    from actkv_open_b200.config import BudgetConfig
    return SessionBudgets(n, BudgetConfig(**cfg), capacity=capacity, device=dev)


def test_budget_steps_match_reference_golden_one_session_at_a_time(golden):
    dev = need_gpu()
    g = golden("budget.npz")
    meta = g["meta"]
    for t in range(meta["n_traces"]):
        tl = torch.from_numpy(g[f"trace_{t}"])
        for c, cfg in enumerate(meta["configs"]):
            sb = _budgets(1, cfg, dev)
            got, slopes, n = [], [], 0
            for k in g[f"chunks_{t}"].tolist():
                sb.trace[0, n:n + k].copy_(tl[n:n + k])
                n += k
                sb.trace_len.fill_(n)
                sb.update()
                got.append(int(sb.budget[0].item()))
                slopes.append(float(sb.slope[0].item()))
            assert got == g[f"budgets_{t}_{c}"].tolist(), (t, c, got)
            np.testing.assert_allclose(slopes, g[f"slopes_{t}_{c}"], rtol=1e-9, atol=1e-12)
    assert_device_clean(dev)


def test_budget_update_of_many_sessions_in_one_launch(golden):
    """All traces as sessions of one SessionBudgets, stepped together, equal the one-at-a-time
    reference budgets; ``out`` receives the new budgets."""
    dev = need_gpu()
    g = golden("budget.npz")
    meta = g["meta"]
    T = meta["n_traces"]
    for c, cfg in enumerate(meta["configs"]):
        sb = _budgets(T, cfg, dev)
        out = torch.full((T,), -1, dtype=torch.int32, device=dev)
        rounds = max(len(g[f"chunks_{t}"]) for t in range(T))
        n = [0] * T
        for rnd in range(rounds):
            live = [t for t in range(T) if rnd < len(g[f"chunks_{t}"])]
            for t in live:
                k = int(g[f"chunks_{t}"][rnd])
                sb.trace[t, n[t]:n[t] + k].copy_(torch.from_numpy(g[f"trace_{t}"][n[t]:n[t] + k]))
                n[t] += k
            sb.trace_len.copy_(torch.tensor(n, dtype=torch.int32))
            before = sb.budget.clone()
            sb.update(out=out)
            now = sb.budget.cpu().tolist()
            assert out.cpu().tolist() == now
            for t in range(T):
                if t in live:
                    assert now[t] == int(g[f"budgets_{t}_{c}"][rnd]), (c, t, rnd)
                else:      # a finished trace steps again here; undo it for the comparison
                    sb.budget[t] = before[t]
    assert_device_clean(dev)


def test_record_appends_each_rows_confidence_to_its_session():
    dev = need_gpu()
    gen = torch.Generator().manual_seed(9)
    sb = _budgets(3, {}, dev)
    rows = [torch.randn(3, 5000, generator=gen) * s for s in (1.0, 4.0)]
    sb.record(rows[0].to(dev))                                               # sessions 0, 1, 2
    sb.record(rows[1][:2].to(dev), torch.tensor([2, 0], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert sb.trace_len.cpu().tolist() == [2, 1, 2]
    tr = sb.trace.cpu().numpy()
    want = {(0, 0): rows[0][0], (1, 0): rows[0][1], (2, 0): rows[0][2], (2, 1): rows[1][0], (0, 1): rows[1][1]}
    for (r, pos), x in want.items():
        assert abs(tr[r, pos] - O.token_confidence(x.numpy(), 20)) <= 2e-5
    assert_device_clean(dev)


def test_only_sessions_over_budget_are_stepped():
    """With seq_used given, a session whose unprotected length is within budget keeps it and gets
    no slope (actkv/hf/session.py:186-193)."""
    dev = need_gpu()
    sb = _budgets(2, dict(init_budget=100, window=4, stride=2), dev)
    down = torch.arange(50, 0, -1, dtype=torch.float32)
    sb.trace[:, :50].copy_(down.expand(2, 50))
    sb.trace_len.fill_(50)
    seq = torch.tensor([150, 90], dtype=torch.int32, device=dev)
    sb.update(seq_used=seq, protected=4)
    assert sb.budget.cpu().tolist() == [175, 100]
    s = sb.slope.cpu().tolist()
    assert s[0] < 0 and math.isnan(s[1])
    assert_device_clean(dev)


def test_a_full_trace_is_flagged_not_overrun():
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    sb = _budgets(1, {}, dev, capacity=2)
    x = torch.randn(1, 100, device=dev)
    for _ in range(3):
        sb.record(x)
    torch.cuda.synchronize()
    assert int(sb.trace_len[0].item()) == 2
    assert N.read_device_status(dev) & N.DEV_BAD_INDEX


def test_confidence_budget_keeps_the_reference_interface():
    """actkv-open's ConfidenceBudget tests (tests/test_algorithms.py:93-113), on the device."""
    dev = need_gpu()
    from actkv_open_b200.budget import ConfidenceBudget
    from actkv_open_b200.config import BudgetConfig
    b = ConfidenceBudget(BudgetConfig(init_budget=512, scale_up=1.75, upper=1000, window=4, stride=2), device=dev)
    b.tl = [float(v) for v in range(50, 0, -1)]
    assert b.next_budget() == 896
    assert b.next_budget() == 1000
    b = ConfidenceBudget(BudgetConfig(init_budget=512, window=4, stride=2), device=dev)
    b.tl = [float(v) for v in range(50)]
    assert b.next_budget() == 512
    b = ConfidenceBudget(BudgetConfig(init_budget=1000, window=4, stride=2, bidirectional=True, shrink_patience=2,
                                      scale_down=2.0, lower=300), device=dev)
    b.tl = [float(v) for v in range(50)]
    assert [b.next_budget() for _ in range(4)] == [1000, 500, 500, 300]
    assert b.history == [1000, 1000, 500, 500, 300]
    b.record(torch.randn(1000, device=dev))
    assert len(b.tl) == 51
    assert_device_clean(dev)
