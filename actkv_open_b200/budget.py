"""Drop-in for ``actkv.budget`` (actkv/budget.py): ActKV Algorithm 2, the confidence-driven adaptive
budget, with the per-token confidence and the budget step computed on the GPU.

``SessionBudgets`` is the device-resident form for a batch of sessions: ``record`` appends each
decode step's token confidence to the sessions' traces in device memory (one launch, no host
round trip), and ``update`` runs Algorithm 2's step for every session at once and can write the
new budgets straight into ``EvictionPipeline.budget``, so an agent loop never reads them back.
``ConfidenceBudget`` and ``FixedBudget`` keep the reference's single-session interface
(``record`` / ``next_budget`` / ``current`` / ``history`` / ``tl``); ``next_budget`` returns a
Python int, so it synchronises, as the reference's does.

``token_confidence`` runs the confidence kernel and returns a float.  ``trace_confidence`` and
``fit_slope`` are the reference's host helpers over a Python list of confidences, kept with the
same signatures for callers that import them; the budget step itself does the same arithmetic in
``actkv_budget_update`` on the device.
"""
from __future__ import annotations

import math

import torch

from . import _native as N
from .config import BudgetConfig

MAX_POOLED = 16384          # min-pooled windows a trace may have (kBudgetMaxPooled in the library)


def _rows(logits: torch.Tensor) -> torch.Tensor:
    x = logits.reshape(-1, logits.shape[-1]) if logits.dim() != 2 else logits
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def token_confidence(logits: torch.Tensor, k: int = 20) -> float:
    """T = -(1/k) * sum of the k largest log-softmax values (budget.py:9-17); for several rows,
    the mean over them, as the reference's mean over all top-k values gives."""
    x = _rows(logits)
    dev = N.require_cuda(x)
    B = x.shape[0]
    trace = torch.empty(B, 1, dtype=torch.float32, device=dev)
    tlen = torch.zeros(B, dtype=torch.int32, device=dev)
    N.check(N.load().actkv_token_confidence(x.data_ptr(), N.dtype_code(x), x.stride(0), B, x.shape[1], k, None,
                                            trace.data_ptr(), 1, tlen.data_ptr(), N.status_word(dev).data_ptr(),
                                            N.stream_ptr(dev)), "token_confidence")
    return float(trace.mean())


def trace_confidence(tl, window: int, stride: int, bottom_pct: float):
    """Sliding-window min pooling, then the pooled values at or below the bottom_pct quantile:
    (window indices, values) (budget.py:20-36).  Host helper over a list of confidences."""
    t = torch.tensor(tl, dtype=torch.float64)
    n = t.numel()
    if n == 0:
        return torch.zeros(0), torch.zeros(0)
    if n < window:
        window = n
    pooled = t.unfold(0, window, stride).amin(dim=1)
    thresh = torch.quantile(pooled, bottom_pct / 100.0)
    keep = pooled <= thresh
    x = torch.arange(pooled.numel(), dtype=torch.float64)[keep]
    return x, pooled[keep]


def fit_slope(x: torch.Tensor, y: torch.Tensor) -> float:
    """Least-squares slope; fewer than two points or no spread in x gives 0 (budget.py:39-47).
    Host helper."""
    if x.numel() < 2:
        return 0.0
    xm, ym = x.mean(), y.mean()
    var = ((x - xm) ** 2).sum()
    if var == 0:
        return 0.0
    return float(((x - xm) * (y - ym)).sum() / var)


class SessionBudgets:
    """Algorithm 2 state of R sessions in device memory: confidence traces [R, capacity] with their
    lengths, budgets and rising-slope counters.

    record(logits, sessions=None)   one decode step: row b's confidence joins session
                                    sessions[b] (default b); one launch, no synchronisation
    update(seq_used=None, protected=0, out=None)
                                    Algorithm 2's step for every session (only those over budget
                                    when seq_used is given, as the reference's end_round); the new
                                    budgets are also written to ``out`` (e.g. the pipeline's
                                    int32 budget array) when given; no synchronisation
    """

    def __init__(self, n_sessions: int, cfg: BudgetConfig | None = None, capacity: int | None = None,
                 device="cuda"):
        self.cfg = cfg or BudgetConfig()
        c = self.cfg
        max_len = c.window + c.stride * (MAX_POOLED - 1)
        if capacity is None:                      # default: 64K values, or all that can be pooled
            capacity = min(65536, max_len)
        if capacity > max_len:
            raise ValueError(f"capacity {capacity} exceeds the {max_len} values a trace can be pooled from")
        self.R, self.capacity = n_sessions, capacity
        self.device = torch.device(device)
        self.trace = torch.zeros(n_sessions, capacity, dtype=torch.float32, device=self.device)
        self.trace_len = torch.zeros(n_sessions, dtype=torch.int32, device=self.device)
        self.budget = torch.full((n_sessions,), c.init_budget, dtype=torch.int32, device=self.device)
        self.rising = torch.zeros(n_sessions, dtype=torch.int32, device=self.device)
        self.slope = torch.zeros(n_sessions, dtype=torch.float64, device=self.device)

    def record(self, logits: torch.Tensor, sessions: torch.Tensor | None = None) -> None:
        x = _rows(logits)
        N.require_cuda(x, sessions)
        if sessions is not None:
            assert sessions.dtype == torch.int32 and sessions.numel() == x.shape[0]
        elif x.shape[0] > self.R:
            raise ValueError(f"{x.shape[0]} logit rows for {self.R} sessions")
        N.check(N.load().actkv_token_confidence(
            x.data_ptr(), N.dtype_code(x), x.stride(0), x.shape[0], x.shape[1], self.cfg.top_k, N.ptr(sessions),
            self.trace.data_ptr(), self.capacity, self.trace_len.data_ptr(), N.status_word(self.device).data_ptr(),
            N.stream_ptr(self.device)), "record")

    def update(self, seq_used: torch.Tensor | None = None, protected: int = 0,
               out: torch.Tensor | None = None) -> torch.Tensor:
        c = self.cfg
        if out is not None:
            assert out.dtype == torch.int32 and out.is_contiguous() and out.numel() >= self.R
        if seq_used is not None:
            assert seq_used.dtype == torch.int32 and seq_used.numel() >= self.R
        N.require_cuda(seq_used, out)
        N.check(N.load().actkv_budget_update(
            self.trace.data_ptr(), self.capacity, self.trace_len.data_ptr(), self.R, c.window, c.stride,
            float(c.bottom_pct), float(c.scale_up), int(c.upper), int(bool(c.bidirectional)),
            int(c.shrink_patience), float(c.shrink_slope), float(c.scale_down), int(c.lower), N.ptr(seq_used),
            int(protected), self.budget.data_ptr(), self.rising.data_ptr(), self.slope.data_ptr(), N.ptr(out),
            N.status_word(self.device).data_ptr(), N.stream_ptr(self.device)), "update")
        return self.budget


class FixedBudget:
    def __init__(self, budget: int):
        self.budget = budget

    @property
    def current(self) -> int:
        return self.budget

    def record(self, logits) -> None: ...

    def next_budget(self) -> int:
        return self.budget

    @property
    def history(self):
        return [self.budget]


class ConfidenceBudget:
    """One session's Algorithm 2 (budget.py:50-104) on the device (a ``SessionBudgets`` of one)."""

    def __init__(self, cfg: BudgetConfig | None = None, device="cuda", capacity: int | None = None):
        self.cfg = cfg or BudgetConfig()
        self._s = SessionBudgets(1, self.cfg, capacity, device)
        self.budget = self.cfg.init_budget
        self.history = [self.budget]
        self.slopes: list[float] = []

    @property
    def current(self) -> int:
        return self.budget

    @property
    def tl(self) -> list[float]:
        n = int(self._s.trace_len[0].item())
        return self._s.trace[0, :n].tolist()

    @tl.setter
    def tl(self, values) -> None:
        v = torch.as_tensor(list(values), dtype=torch.float32)
        if v.numel() > self._s.capacity:
            raise ValueError(f"trace of {v.numel()} values exceeds the capacity {self._s.capacity}")
        self._s.trace[0, :v.numel()].copy_(v)
        self._s.trace_len.fill_(v.numel())

    def record(self, logits: torch.Tensor) -> None:
        self._s.record(_rows(logits)[-1:])

    def slope(self) -> float:
        return fit_slope(*trace_confidence(self.tl, self.cfg.window, self.cfg.stride, self.cfg.bottom_pct))

    def next_budget(self) -> int:
        """Called when compression is triggered (Algorithm 2, steps 3-4)."""
        self._s.update()
        self.budget = int(self._s.budget[0].item())
        a = float(self._s.slope[0].item())
        self.slopes.append(0.0 if math.isnan(a) else a)
        self.history.append(self.budget)
        return self.budget
