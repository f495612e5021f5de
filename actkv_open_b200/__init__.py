"""actkv_open_b200: actkv-open's eviction hot path (LSE-recovery scoring -> ActionLRFU keep scores
-> keep mask -> conflict-free in-place paged compaction) on hand-written sm_100a (B200) kernels,
behind actkv-open's own module layout:

    actkv_open_b200.kernels.lse_attn    ~ actkv.kernels.lse_attn
    actkv_open_b200.kernels.compaction  ~ actkv.kernels.compaction
    actkv_open_b200.paged               ~ actkv.paged
    actkv_open_b200.eviction            ~ actkv.eviction (ActionLRFU, reduce_heads, top_p_mask)
    actkv_open_b200.config              ~ actkv.config (EvictionConfig, BudgetConfig)
    actkv_open_b200.budget              ~ actkv.budget (Algorithm 2 on the device)
    actkv_open_b200.engine              batched, device-resident eviction of many sessions

The kernels are reached through the C ABI in include/actkv_b200.h (libactkv_b200.so).
"""
from .budget import ConfidenceBudget, FixedBudget
from .config import BudgetConfig, EvictionConfig
from .eviction import ActionLRFU, make_policy, reduce_heads, top_p_mask

__version__ = "0.1.0"
__all__ = ["ActionLRFU", "BudgetConfig", "ConfidenceBudget", "EvictionConfig", "FixedBudget", "make_policy",
           "reduce_heads", "top_p_mask", "install_as_actkv"]


def install_as_actkv() -> None:
    """Register this package under the reference's module names (``actkv``, ``actkv.kernels``,
    ``actkv.kernels.lse_attn``, ``actkv.kernels.compaction``, ``actkv.paged``, ``actkv.eviction``,
    ``actkv.config``, ``actkv.budget``) so that code written against actkv-open's eviction path
    imports these kernels unchanged.  Only call it in a process that does not also import the
    reference."""
    import sys

    from . import budget, config, engine, eviction, kernels, paged
    from .kernels import compaction, lse_attn
    pkg = sys.modules[__name__]
    for name, mod in {"actkv": pkg, "actkv.kernels": kernels, "actkv.kernels.lse_attn": lse_attn,
                      "actkv.kernels.compaction": compaction, "actkv.paged": paged,
                      "actkv.eviction": eviction, "actkv.config": config, "actkv.engine": engine,
                      "actkv.budget": budget}.items():
        sys.modules[name] = mod
