"""KV-head sharding of a session across ranks: the one exchange step of the eviction path.

A very long session (131072 tokens, 80 layers, 8 KV heads on 8 GPUs) is split
by KV head: rank r holds heads [lo, hi) of every layer -- its slice of the paged cache
``kv[L, 2, NB, BS, hi - lo, D]`` -- and the matching query heads [lo*G, hi*G).  Block tables, the
free stack and the lengths are replicated and identical on every rank.

Per step each rank scores its own heads; the only data the ranks exchange is the per-token head
reduction that ActionLRFU consumes (actkv/eviction.py:20-33, ``reduce_heads``):

  mean:  act = (sum over all KV heads) / Hkv  -> local sum over the rank's heads, all_reduce(SUM),
         one division by Hkv (the reference divides the full sum once, so does this)
  max:   act = max over all KV heads          -> local max, all_reduce(MAX)

After the all-reduce every rank holds the same ``act`` (a collective returns identical values on
all ranks), so the nucleus hits, keep scores, keep mask and compaction plan agree everywhere and
each rank compacts its own head slice with the same plan.  The collective goes through
``torch.distributed`` (NCCL over NVLink on GPUs; gloo for the CPU tests of this logic).
"""
from __future__ import annotations

import torch


def head_shard(n_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """KV heads [lo, hi) owned by ``rank`` when ``n_kv_heads`` are split evenly over ``world`` ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split evenly over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def local_head_reduce(heads: torch.Tensor, how: str, out: torch.Tensor | None = None) -> torch.Tensor:
    """This rank's part of the head reduction: heads [R, L, h, W] -> [R, L, W] (sum for "mean",
    max for "max").  With one head per rank (config 4) it is a view, no copy."""
    if how not in ("mean", "max"):
        raise ValueError(how)
    R, L, h, W = heads.shape
    if h == 1:
        part = heads.view(R, L, W) if heads.is_contiguous() else heads[:, :, 0, :]
        if out is None:
            return part if part.is_contiguous() else part.contiguous()
        out.copy_(part)
        return out
    if how == "mean":
        return torch.sum(heads, dim=2, out=out) if out is not None else heads.sum(dim=2)
    res = heads.amax(dim=2)
    if out is None:
        return res
    out.copy_(res)
    return out


def allreduce_heads(part: torch.Tensor, n_kv_heads: int, how: str, group=None) -> torch.Tensor:
    """Turn every rank's local part into the full head reduction, in place, identical on all ranks.

    ``part`` must be contiguous (the collective works on its storage); ``n_kv_heads`` is the total
    number of KV heads over all ranks (the reference's divisor for "mean")."""
    import torch.distributed as dist
    if how not in ("mean", "max"):
        raise ValueError(how)
    if not part.is_contiguous():
        raise ValueError("the all-reduced buffer must be contiguous")
    dist.all_reduce(part, op=dist.ReduceOp.SUM if how == "mean" else dist.ReduceOp.MAX, group=group)
    if how == "mean":
        part.div_(n_kv_heads)
    return part
