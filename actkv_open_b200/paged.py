"""Drop-in for ``actkv.paged`` (actkv/paged.py): a vLLM-style paged KV cache whose scoring, keep-mask
selection and compaction run on sm_100a kernels.

    kv : [n_layers, 2, num_blocks, block_size, n_kv_heads, head_dim]

The allocator keeps the reference's host model (paged.py:49-112): ``free`` is a LIFO list popped
from its end, ``tables`` maps a request to its list of physical blocks, ``seq_used`` its token
count, ``pinned`` its protected tokens.  ``evict`` needs no device->host synchronisation: the
number of tokens it keeps (pinned + budget) is known on the host, so the table and free list are
updated from it while the device computes the mask, the plan and the copies.
"""
from __future__ import annotations

import math

import torch

from . import _native as N
from ._native import OutOfBlocks
from .kernels.compaction import _keep_u8, apply_copies
from .kernels.lse_attn import action_scores, paged_decode_attention

__all__ = ["OutOfBlocks", "PagedKVCache", "keep_mask_from_scores"]


def _score_view(scores: torch.Tensor, seq_used: int):
    """(tensor, n_lead, n_red, stride_l, stride_x) so that the kernel reads (l, x, t) at
    l*stride_l + x*stride_x + t: dim -2 is reduced, the leading dims are averaged."""
    s = scores if scores.dtype == torch.float32 else scores.float()
    if s.stride(-1) != 1:
        s = s.contiguous()
    if s.dim() == 1:
        return s, 1, 1, 0, 0
    if s.dim() == 2:
        return s, 1, s.shape[0], 0, s.stride(0)
    lead = s.reshape(-1, s.shape[-2], s.shape[-1])
    return lead, lead.shape[0], lead.shape[1], lead.stride(0), lead.stride(1)


def _keep_mask_device(scores, seq_used: int, budget: int, protected, head_reduce: str) -> torch.Tensor:
    if head_reduce not in ("mean", "max"):
        raise ValueError(head_reduce)
    dev = N.require_cuda(scores)
    s, n_lead, n_red, st_l, st_x = _score_view(scores, seq_used)
    if isinstance(protected, torch.Tensor):
        pin = _keep_u8(protected.to(device=dev)[:seq_used])
        if pin.numel() < seq_used:
            pin = torch.cat([pin, pin.new_zeros(seq_used - pin.numel())])
        prefix = 0
    else:
        pin, prefix = None, int(protected)
    keep = torch.empty(max(seq_used, 1), dtype=torch.uint8, device=dev)
    small = torch.tensor([seq_used, budget], dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
    lib = N.load()
    ws = N.workspace(lib.actkv_keep_mask_workspace_bytes(1, seq_used), dev)
    N.check(lib.actkv_keep_mask(s.data_ptr(), None, 0, st_l, st_x, n_lead, n_red,
                                N.REDUCE_MAX if head_reduce == "max" else N.REDUCE_MEAN,
                                N.ptr(pin), 0, prefix, small[0:1].data_ptr(), small[1:2].data_ptr(), 0,
                                keep.data_ptr(), 0, None, 1, seq_used, ws.data_ptr(), ws.numel(),
                                N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "keep_mask_from_scores")
    return keep[:seq_used].view(torch.bool)


def keep_mask_from_scores(scores: torch.Tensor, seq_used: int, budget: int,
                          protected: int | torch.Tensor = 0, head_reduce: str = "mean") -> torch.Tensor:
    """Per-token scores -> keep mask [seq_used]: the protected tokens plus the top-``budget`` others.

    scores: [S], [Hkv, S] or [n_layers, Hkv, S]. KV heads (dim -2) are reduced with
    ``head_reduce``, then the leading dims (layers) are averaged: one block table serves every
    layer, so a paged cache keeps the same tokens in every layer (paged.py:23-46).  protected: a
    count of leading tokens, or a bool mask [seq_used].  Ties at the threshold keep the lowest index.
    """
    return _keep_mask_device(scores, int(seq_used), int(budget), protected, head_reduce)


class PagedKVCache:
    def __init__(self, num_blocks: int, block_size: int, n_kv_heads: int, head_dim: int,
                 n_layers: int = 1, dtype=torch.float16, device="cpu"):
        self.block_size, self.n_kv_heads, self.head_dim = block_size, n_kv_heads, head_dim
        self.n_layers, self.num_blocks = n_layers, num_blocks
        self.kv = torch.zeros(n_layers, 2, num_blocks, block_size, n_kv_heads, head_dim,
                              dtype=dtype, device=device)
        self.free: list[int] = list(range(num_blocks - 1, -1, -1))
        self.tables: dict[int, list[int]] = {}
        self.seq_used: dict[int, int] = {}
        self.pinned: dict[int, torch.Tensor] = {}   # per request: which logical positions evict() protects
        self._n_pinned: dict[int, int] = {}         # host count of pinned[req] (kept by every compaction)
        self.device = device

    # ---------------------------------------------------------------- allocation
    @property
    def used_blocks(self) -> int:
        return self.num_blocks - len(self.free)

    def _ensure(self, req: int, n_tokens: int) -> None:
        table = self.tables.setdefault(req, [])
        self.seq_used.setdefault(req, 0)
        need = math.ceil(n_tokens / self.block_size) - len(table)
        if need > len(self.free):
            raise OutOfBlocks(f"need {need} blocks, {len(self.free)} free")
        for _ in range(need):
            table.append(self.free.pop())

    def append(self, req: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [n_layers, n, Hkv, D] new tokens for request ``req``."""
        n = k.shape[1]
        start = self.seq_used.get(req, 0)
        self._ensure(req, start + n)
        slots = self.slot_map(req, start + n)[start:]
        flat = self.kv.view(self.n_layers, 2, -1, self.n_kv_heads, self.head_dim)
        flat[:, 0, slots] = k.to(device=self.kv.device, dtype=self.kv.dtype)
        flat[:, 1, slots] = v.to(device=self.kv.device, dtype=self.kv.dtype)
        self.seq_used[req] = start + n

    def release(self, req: int) -> None:
        self.free.extend(reversed(self.tables.pop(req, [])))
        self.seq_used.pop(req, None)
        self.pinned.pop(req, None)
        self._n_pinned.pop(req, None)

    # ---------------------------------------------------------------- views
    def _to_device(self, host: torch.Tensor) -> torch.Tensor:
        if torch.device(self.device).type == "cuda":
            return host.pin_memory().to(self.device, non_blocking=True)
        return host.to(self.device)

    def slot_map(self, req: int, n: int | None = None) -> torch.Tensor:
        n = self.seq_used[req] if n is None else n
        table = torch.tensor(self.tables[req], dtype=torch.long)
        pos = torch.arange(n)
        return self._to_device(table[pos // self.block_size] * self.block_size + pos % self.block_size)

    def block_table(self, reqs: list[int]) -> torch.Tensor:
        mb = max(len(self.tables[r]) for r in reqs)
        bt = torch.zeros(len(reqs), max(mb, 1), dtype=torch.int32)
        for i, r in enumerate(reqs):
            bt[i, : len(self.tables[r])] = torch.tensor(self.tables[r], dtype=torch.int32)
        return self._to_device(bt)

    def seq_tensor(self, reqs: list[int]) -> torch.Tensor:
        return self._to_device(torch.tensor([self.seq_used[r] for r in reqs], dtype=torch.int32))

    def gather(self, req: int, layer: int = 0):
        slots = self.slot_map(req)
        flat = self.kv[layer].view(2, -1, self.n_kv_heads, self.head_dim)
        return flat[0, slots], flat[1, slots]

    # ---------------------------------------------------------------- primitives
    def decode_attention(self, reqs, q, layer=0, scale=None):
        """Paged decode attention -> (out, lse) (paged.py:114-118): on the GPU (flash decoding,
        ``paged_decode_attention``), the role the reference's torch stand-in plays for the paged
        FA backend."""
        return paged_decode_attention(q, self.kv[layer], self.block_table(reqs), self.seq_tensor(reqs), scale)

    def cal_attn(self, reqs, q, lse, out, n_seen, layer=0, scale=None):
        """Primitive 1: AttnScore <- CalAttn(target_q, KCache) via LSE recovery (Algorithm 3)."""
        return action_scores(q, self.kv[layer], self.block_table(reqs), self.seq_tensor(reqs),
                             lse, out, n_seen, scale)

    def _compact(self, req: int, keep_u8: torch.Tensor, kept: int) -> torch.Tensor:
        """Device plan + copies for one request whose kept count is known; host table/free update."""
        n = self.seq_used[req]
        table = self.tables[req]
        dev = self.kv.device
        y, x = math.ceil(n / self.block_size), math.ceil(kept / self.block_size)
        drop = y - x
        # one host->device copy: [seq_used, free_top, table...]; the freed blocks go to a scratch
        # stack (the host list below is the allocator of record)
        meta = self._to_device(torch.tensor([n, 0] + table, dtype=torch.int32))
        scratch_free = torch.empty(max(drop, 1), dtype=torch.int32, device=dev)
        perm = torch.empty(max(n, 1), dtype=torch.int64, device=dev)
        es = self.kv.element_size()
        row = self.n_kv_heads * self.head_dim
        lib = N.load()
        ws = N.workspace(lib.actkv_compact_workspace_bytes(1, n), dev)
        N.check(lib.actkv_compact(self.kv.data_ptr(), 2 * self.n_layers, self.kv.stride(1) * es,
                                  row * es, row * es, self.num_blocks * self.block_size,
                                  keep_u8.data_ptr(), 0, meta[0:1].data_ptr(), meta[2:].data_ptr(), 0,
                                  max(len(table), 1), self.block_size, scratch_free.data_ptr(),
                                  meta[1:2].data_ptr(), max(drop, 1), perm.data_ptr(), 0, None, 1, max(n, 1),
                                  ws.data_ptr(), ws.numel(), N.status_word(dev).data_ptr(),
                                  N.stream_ptr(dev)), "compact")
        freed = table[:drop]
        self.tables[req] = table[drop:]
        self.free.extend(reversed(freed))
        self.seq_used[req] = kept
        return perm[:kept]

    def compact(self, req: int, keep_mask: torch.Tensor) -> torch.Tensor:
        """Primitive 3: KVCache <- Compaction(KVCache, KeepMask) (Algorithm 4), all layers at once.

        Returns ``perm`` (new logical position -> old logical position).  Freed blocks go straight
        back to the allocator.  Reads the kept count back from the device (the reference does too).
        """
        N.require_cuda(self.kv, keep_mask)
        n = self.seq_used[req]
        keep = _keep_u8(keep_mask[:n])
        kept = int(keep.sum().item())
        return self._compact(req, keep, kept)

    def evict(self, req: int, scores: torch.Tensor, budget: int, protected: int = 0,
              head_reduce: str = "mean") -> torch.Tensor:
        """Scores -> KeepMask -> Compaction: keep the protected tokens plus the top-``budget`` others.

        ``protected`` counts the request's first tokens the first time it is evicted; compaction
        moves them, so the cache remembers where they went (``pinned``) and keeps protecting them.
        Returns ``perm`` like compact(); a request already within budget is left untouched.
        """
        n = self.seq_used[req]
        dev = self.kv.device
        if req in self.pinned:
            pinned = self.pinned[req]
            n_pinned = self._n_pinned.get(req)
            if n_pinned is None:
                n_pinned = int(pinned.sum())
        else:
            p = max(0, min(int(protected), n))
            pinned = torch.arange(n, device=dev) < p
            n_pinned = p
        if pinned.numel() < n:
            pinned = torch.cat([pinned, pinned.new_zeros(n - pinned.numel())])   # tokens appended since
        self.pinned[req] = pinned
        self._n_pinned[req] = n_pinned
        if n - n_pinned <= budget:
            return torch.arange(n, device=dev)
        keep = _keep_mask_device(scores, n, budget, pinned, head_reduce)
        kept = n_pinned + max(0, budget)
        perm = self._compact(req, _keep_u8(keep), kept)
        self.pinned[req] = pinned[perm]
        return perm

    def apply_copies(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        """Copy slots over every layer's K and V planes (apply_copies on the cache's flat view)."""
        flat = self.kv.view(self.n_layers * 2, -1, self.n_kv_heads * self.head_dim)
        apply_copies(flat, src, dst)
