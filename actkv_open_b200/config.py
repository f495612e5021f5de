"""Hyperparameters of the eviction path (actkv/config.py:7-15).  Defaults match the reference."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class EvictionConfig:
    decay: float = 0.5          # lambda, keep-score decay per compression step (Algorithm 1)
    top_p: float = 0.90         # hit threshold: entries in the top-p attention mass of the action region
    head_reduce: str = "mean"   # how per-KV-head scores become one score per token: "mean" or "max"
