"""Hyperparameters of the eviction path (actkv/config.py:7-15).  Defaults match the reference."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class EvictionConfig:
    decay: float = 0.5          # lambda, keep-score decay per compression step (Algorithm 1)
    top_p: float = 0.90         # hit threshold: entries in the top-p attention mass of the action region
    head_reduce: str = "mean"   # how per-KV-head scores become one score per token: "mean" or "max"


@dataclass
class BudgetConfig:
    """Algorithm 2 hyperparameters (actkv/config.py:19-33); defaults match the reference."""
    top_k: int = 20             # top-k tokens of the token-level confidence
    window: int = 64            # sliding window of the min pooling
    stride: int = 8
    bottom_pct: float = 10.0    # pooled values kept: the bottom b%
    init_budget: int = 512
    scale_up: float = 1.75
    upper: int = 30_000
    bidirectional: bool = False  # the reference's extension: shrink while confidence keeps rising
    shrink_patience: int = 3
    shrink_slope: float = 0.0
    scale_down: float = 1.75
    lower: int = 256
