"""Drop-in for ``actkv.kernels.compaction`` (actkv/kernels/compaction.py): conflict-free in-place
paged compaction (ActKV Algorithm 4) on sm_100a kernels.

    X     = ceil(B / block_size)        blocks needed after compaction
    start = (Y - X) * block_size        Y = blocks used before compaction
    dst   = evicted slots inside [start, start + B), ascending
    src   = kept slots outside it, ascending

src and dst are disjoint, so every copy runs in parallel in one pass with no scratch buffer, and
the request's first Y - X logical blocks become free.  ``plan_compaction`` computes the plan on the
device (block-wide ballot scans instead of nonzero) and ``apply_copies`` moves the rows with one
warp per (pair, plane) and 16-byte accesses.  ``apply_copies_ref`` and ``gather_compaction`` are
the module's torch helpers (compaction.py:72-74, :109-114): a reference and the gather baseline.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import _native as N

HAS_KERNELS = __import__("os").path.exists(N.lib_path())
HAS_TRITON = HAS_KERNELS      # the reference's flag name; the kernels here are CUDA


@dataclass
class CompactionPlan:
    src_slots: torch.Tensor   # physical slots to read
    dst_slots: torch.Tensor   # physical slots to write
    perm: torch.Tensor        # [B] new logical position -> old logical position
    drop_blocks: int          # leading logical blocks that become free (Y - X)


def _keep_u8(keep: torch.Tensor) -> torch.Tensor:
    keep = keep.contiguous()
    return keep.view(torch.uint8) if keep.dtype == torch.bool else (keep != 0).to(torch.uint8)


def plan_compaction(keep_mask: torch.Tensor, seq_used: int, block_table_row: torch.Tensor,
                    block_size: int) -> CompactionPlan:
    """Algorithm 4 steps 1-5 for one request. keep_mask: [>= seq_used] bool, True = retain.

    One device->host read (the counts) sizes the returned tensors, as the reference's
    ``int(keep.sum())`` does.
    """
    dev = N.require_cuda(keep_mask, block_table_row)
    seq_used = int(seq_used)
    keep = _keep_u8(keep_mask[:seq_used])
    table = block_table_row.to(device=dev, dtype=torch.int32).contiguous()
    cap = max(seq_used, 1)
    src = torch.empty(cap, dtype=torch.int64, device=dev)
    dst = torch.empty(cap, dtype=torch.int64, device=dev)
    perm = torch.empty(cap, dtype=torch.int64, device=dev)
    counts = torch.zeros(4, dtype=torch.int32, device=dev)
    lib = N.load()
    ws = N.workspace(lib.actkv_plan_workspace_bytes(seq_used), dev)
    N.check(lib.actkv_plan_compaction(keep.data_ptr(), seq_used, table.data_ptr(), table.numel(), block_size,
                                      src.data_ptr(), dst.data_ptr(), perm.data_ptr(), counts.data_ptr(),
                                      ws.data_ptr(), ws.numel(), N.status_word(dev).data_ptr(),
                                      N.stream_ptr(dev)), "plan_compaction")
    b, n_pairs, drop, _ = counts.tolist()
    return CompactionPlan(src[:n_pairs], dst[:n_pairs], perm[:b], drop)


def apply_copies_ref(kv_flat: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
    """kv_flat [N, slots, H*D]; disjoint src/dst, so a single vectorised copy is safe."""
    kv_flat[:, dst] = kv_flat[:, src]


def apply_copies(kv_flat: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
    """kv_flat[:, dst] = kv_flat[:, src] on the device; kv_flat [planes, slots, row], row contiguous."""
    if src.numel() == 0:
        return
    assert kv_flat.stride(2) == 1
    dev = N.require_cuda(kv_flat, src, dst)
    planes, slots, row = kv_flat.shape
    es = kv_flat.element_size()
    src = src.to(torch.int64).contiguous()
    dst = dst.to(torch.int64).contiguous()
    N.check(N.load().actkv_apply_copies(kv_flat.data_ptr(), planes, kv_flat.stride(0) * es, kv_flat.stride(1) * es,
                                        row * es, slots, src.data_ptr(), dst.data_ptr(), src.numel(),
                                        N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "apply_copies")


def gather_compaction(kv_flat: torch.Tensor, keep_slots: torch.Tensor) -> torch.Tensor:
    """Gather-based baseline (paged R-KV style): survivors go into a fresh contiguous buffer."""
    return kv_flat[:, keep_slots].clone()


def blocks_after(n: int, kept: int, block_size: int) -> tuple[int, int]:
    """(Y, X): blocks used before and after compacting n tokens down to ``kept``."""
    return math.ceil(n / block_size), math.ceil(kept / block_size)
