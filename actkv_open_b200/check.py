"""Torch restatement of one eviction step, used to CHECK the kernels at full size on the GPU.

The eviction path never calls anything here: these are the reference's torch formulas (the same
role ``action_scores_ref`` and ``apply_copies_ref`` play in the reference's own modules), run on
the device in fp32 so that BASELINE-sized steps (36 layers x 32K tokens, 80 layers x 131K tokens)
can be checked in seconds.  ``check_step`` compares one ``EvictionPipeline.step`` against them:

  scores      per head and head mean, within ``rtol`` (1e-3) of fp32 torch
              (actkv/kernels/lse_attn.py:63-78: max over the GQA group of exp(q.k*scale - lse),
              running mean over the causal action region)
  keep scores ks = fl(fl(decay*ks) + act*hit), hit = nucleus of act (actkv/eviction.py:36-50,
              198-210), computed from the kernel's own act; differences allowed only at the
              nucleus boundary (values within rtol of the smallest value inside the nucleus)
  keep mask   layer mean of ks, pinned tokens + top-budget others (actkv/paged.py:23-46);
              differences allowed only at near-ties of the threshold, same kept count
  compaction  bit-exact: the kernel's mask replayed through Algorithm 4's plan
              (actkv/kernels/compaction.py:44-69): tables, free stack, lengths, perm, every byte of
              every K/V plane, and the permuted keep scores and pins (actkv/paged.py:125-157)

Every function takes device tensors and returns device tensors; only small summaries go to the
host.
"""
from __future__ import annotations

import math
from contextlib import contextmanager

import torch


@contextmanager
def _exact_fp32():
    """fp32 matmuls without TF32 (the checks need fp32 products)."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def session_slots(table: torch.Tensor, n: int, bs: int) -> torch.Tensor:
    """Physical slots [n] of a session's first n logical positions (table: its block ids)."""
    pos = torch.arange(n, device=table.device)
    return table[:math.ceil(n / bs)].long()[pos // bs] * bs + pos % bs


def region_scores_ref(kv_layers: torch.Tensor, table: torch.Tensor, n: int, q: torch.Tensor, lse: torch.Tensor,
                      scale: float | None = None, chunk: int = 8192) -> torch.Tensor:
    """Per-head scores [L, Hkv, n] of one session after its causal action region.

    kv_layers [L, 2, NB, BS, Hkv, D] (the whole cache or its layer slice), table [>= ceil(n/BS)]
    block ids, q [L, A, Hq, D], lse [L, A, Hq].  Action token j sees tokens t <= n - A + j; the
    score of t is (1/A) * sum_j max_g exp(scale * q_{j,hG+g} . k_t - lse_{j,hG+g}) -- A
    sequential ``action_scores`` calls from a zeroed running mean (lse_attn.py:63-78)."""
    L, _, nb, bs, hkv, d = kv_layers.shape
    A, hq = q.shape[1], q.shape[2]
    g = hq // hkv
    scale = d ** -0.5 if scale is None else scale
    slots = session_slots(table, n, bs)
    out = torch.empty(L, hkv, n, dtype=torch.float32, device=kv_layers.device)
    see = n - A + torch.arange(A, device=kv_layers.device)                      # last visible token
    with _exact_fp32():
        for l in range(L):
            k_all = kv_layers[l, 0].reshape(nb * bs, hkv, d)
            qq = q[l].float().view(A, hkv, g, d).permute(1, 0, 2, 3).reshape(hkv, A * g, d)
            ll = lse[l].float().view(A, hkv, g).permute(1, 0, 2).reshape(hkv, A * g, 1)
            for c0 in range(0, n, chunk):
                c1 = min(n, c0 + chunk)
                k = k_all[slots[c0:c1]].float().permute(1, 2, 0)                   # [Hkv, D, C]
                p = torch.exp(torch.bmm(qq, k) * scale - ll)                        # [Hkv, A*G, C]
                p = p.view(hkv, A, g, c1 - c0).amax(2)                              # [Hkv, A, C]
                pos = torch.arange(c0, c1, device=k.device)
                p = p.masked_fill(pos[None, None, :] > see[None, :, None], 0.0)
                out[l, :, c0:c1] = p.sum(1) / A
    return out


def nucleus_ref(a: torch.Tensor, top_p: float) -> torch.Tensor:
    """Bool nucleus mask of a 1-D row (actkv/eviction.py:36-50): the fewest largest entries holding
    >= top_p of the mass, the crossing entry included, only entries > 0; cumulative sums in fp64
    rounded to fp32, target fp32(top_p * total)."""
    if a.numel() == 0:
        return torch.zeros_like(a, dtype=torch.bool)
    total = a.sum(dtype=torch.float32)
    if not bool(total > 0):
        return torch.zeros_like(a, dtype=torch.bool)
    vals, order = torch.sort(a, descending=True, stable=True)
    csum = torch.cumsum(vals.double(), 0).float()
    target = (torch.tensor(top_p, dtype=torch.float32, device=a.device) * total).float()
    n_keep = min(int(torch.searchsorted(csum, target.view(1), right=False).item()) + 1, a.numel())
    mask = torch.zeros_like(a, dtype=torch.bool)
    mask[order[:n_keep]] = True
    return mask & (a > 0)


def topk_mask_ref(s: torch.Tensor, free: torch.Tensor, k: int) -> torch.Tensor:
    """Bool mask of the k largest s among the ``free`` entries, lowest index first among equals."""
    idx = torch.nonzero(free).flatten()
    keep = torch.zeros_like(free)
    k = min(k, idx.numel())
    if k > 0:
        vals = s[idx].double()
        order = torch.sort(-vals, stable=True).indices[:k]
        keep[idx[order]] = True
    return keep


def plan_ref(keep: torch.Tensor, n: int, table: torch.Tensor, bs: int):
    """Algorithm 4's plan for one session (actkv/kernels/compaction.py:44-69): kept tokens end in
    the window [start, start + B), start = (Y - X) * BS; kept tokens outside it move, ascending,
    into the window's holes, ascending.  Returns (src_phys, dst_phys, perm, drop)."""
    keep = keep[:n].bool()
    B = int(keep.sum().item())
    y, x = math.ceil(n / bs), math.ceil(B / bs)
    start = (y - x) * bs
    full = torch.zeros(y * bs, dtype=torch.bool, device=keep.device)
    full[:n] = keep
    dst = torch.nonzero(~full[start:start + B]).flatten() + start
    outside = full.clone()
    outside[start:start + B] = False
    src = torch.nonzero(outside).flatten()
    assert src.numel() == dst.numel(), "kept count must equal the window"
    tb = table.long()
    perm = torch.arange(start, start + B, device=keep.device)
    perm[dst - start] = src
    return tb[src // bs] * bs + src % bs, tb[dst // bs] * bs + dst % bs, perm, y - x


def _near(values: torch.Tensor, thr: float, rtol: float) -> torch.Tensor:
    return (values.double() - thr).abs() <= rtol * max(abs(thr), 1e-30)


def capture_state(pipe) -> dict:
    """Everything ``check_step`` needs from before a step: a device snapshot plus host copies of the
    small allocator state and the round's sizes."""
    c = pipe.cache
    R = c.n_sessions
    snap = pipe.snapshot()
    seq = c.seq_used[:R].tolist()
    bt = c.block_table[:R].cpu()
    top = int(c.free_top.item())
    off = pipe.act_off[:R + 1].tolist()
    return {"snap": snap, "seq": seq, "tables": [bt[r, :math.ceil(seq[r] / c.block_size)].tolist() for r in range(R)],
            "free": c.free_list[:top].tolist(), "act_off": off, "budget": pipe.budget[:R].tolist()}


def check_step(pipe, before: dict, q: torch.Tensor, lse: torch.Tensor, rtol: float = 1e-3,
               check_cache: bool = True) -> dict:
    """Compare the step ``pipe`` just ran (from state ``before`` = ``capture_state`` output, on
    inputs q [L, sumA, Hq, D] / lse [L, sumA, Hq]) with the torch restatement.  Raises
    AssertionError on a mismatch; returns a summary."""
    c = pipe.cache
    R, L, H, bs = c.n_sessions, c.n_layers, c.n_kv_heads, c.block_size
    snap = before["snap"]
    kv0 = snap["kv"]
    cfg = pipe.cfg
    ks_pre = pipe.ks[1 - pipe.cur]            # the keep scores the mask was taken from
    ks_new, pin_new = pipe.ks[pipe.cur], pipe.pin[pipe.cur]
    pin0, ks0 = snap["pin"], snap["ks"]
    rep = {"sessions": R, "layers": L, "max_rel_err_heads": 0.0, "max_rel_err_act": 0.0, "nucleus_boundary_diffs": 0,
           "mask_near_ties": 0, "moved_rows": 0}
    free_ref = list(before["free"])
    tables_now, seq_now, free_now = c.state()
    written = torch.zeros(kv0.shape[2] * bs, dtype=torch.bool, device=c.device) if check_cache else None
    for r in range(R):
        n = before["seq"][r]
        a0, a1 = before["act_off"][r], before["act_off"][r + 1]
        A = a1 - a0
        table = torch.tensor(before["tables"][r], dtype=torch.int32, device=c.device)
        pinned = pin0[r, :n].bool()
        if A > 0:
            ref = region_scores_ref(kv0, table, n, q[:, a0:a1], lse[:, a0:a1], pipe.scale)     # [L, Hkv, n]
            if pipe.heads is not None:               # this rank's heads (all of them unsharded)
                got = pipe.heads[r, :, :, :n]
                err = ((got - ref).abs() / ref.abs().clamp_min(1e-30)).masked_fill((got - ref).abs() <= 1e-12, 0)
                rep["max_rel_err_heads"] = max(rep["max_rel_err_heads"], float(err.max()))
            ref_act = ref.mean(1) if cfg.head_reduce == "mean" else ref.amax(1)
        else:
            ref_act = torch.zeros(L, n, device=c.device)
        act = pipe.act[r, :, :n]
        if pipe.group is None:
            diff = (act - ref_act).abs()
            err = (diff / ref_act.abs().clamp_min(1e-30)).masked_fill(diff <= 1e-12, 0)
            rep["max_rel_err_act"] = max(rep["max_rel_err_act"], float(err.max()))
        # ActionLRFU from the kernel's own act (pinned tokens untouched)
        free = ~pinned
        ks_ref = ks0[r, :, :n].clone()
        for l in range(L):
            a = act[l][free]
            hit = nucleus_ref(a, cfg.top_p) if A > 0 else torch.zeros_like(a, dtype=torch.bool)
            k = ks_ref[l][free] * torch.tensor(cfg.decay, dtype=torch.float32, device=c.device)
            k = torch.where(hit, k + a, k)
            row = ks_ref[l]
            row[free] = k
            bad = ks_pre[r, l, :n] != row
            if bool(bad.any()):
                pos = a[a > 0]
                thr = float(pos[hit[a > 0]].min()) if bool(hit.any()) else 0.0
                vals = torch.zeros_like(row)
                vals[free] = a
                ok = _near(vals[bad], thr, rtol) & ((ks_pre[r, l, :n][bad] - row[bad]).abs()
                                                  <= vals[bad] * (1 + rtol) + 1e-30)
                assert bool(ok.all()), f"session {r} layer {l}: keep scores differ off the nucleus boundary"
                rep["nucleus_boundary_diffs"] += int(bad.sum())
        # keep mask from the layer mean of the kernel's keep scores
        keep = pipe.keep[r, :n].bool()
        n_pin = int(pinned.sum())
        budget = before["budget"][r]
        if n - n_pin <= budget:
            want = torch.ones(n, dtype=torch.bool, device=c.device)
        else:
            s = ks_pre[r, :, :n].mean(0)
            want = pinned | topk_mask_ref(s, free, budget)
        if not torch.equal(keep, want):
            assert int(keep.sum()) == int(want.sum()), f"session {r}: kept {int(keep.sum())} != {int(want.sum())}"
            d = torch.nonzero(keep != want).flatten()
            s = ks_pre[r, :, :n].mean(0)
            thr = float(s[want & free].min())
            assert bool(_near(s[d], thr, rtol).all()), f"session {r}: masks differ off the threshold"
            rep["mask_near_ties"] += int(d.numel())
        # compaction of the kernel's mask, bit-exact
        src, dst, perm, drop = plan_ref(keep, n, table, bs)
        B = perm.numel()
        assert int(pipe.kept[r]) == B and seq_now[r] == B, f"session {r}: length {seq_now[r]} != {B}"
        assert torch.equal(pipe.perm[r, :B], perm), f"session {r}: perm differs"
        assert tables_now[r] == before["tables"][r][drop:], f"session {r}: table differs"
        free_ref.extend(reversed(before["tables"][r][:drop]))
        rep["moved_rows"] += int(src.numel())
        if check_cache and src.numel():
            flat0 = kv0.view(2 * L, -1, H * c.head_dim)
            flat1 = c.kv.view(2 * L, -1, H * c.head_dim)
            assert torch.equal(flat1[:, dst], flat0[:, src]), f"session {r}: moved rows differ"
            written[dst] = True
        # keep scores and pins follow their tokens
        assert torch.equal(ks_new[r, :, :B], ks_pre[r, :, :n][:, perm]), f"session {r}: permuted keep scores"
        assert torch.equal(pin_new[r, :B], pin0[r, :n][perm]), f"session {r}: permuted pins"
    assert free_now == free_ref, "free stack differs"
    if check_cache:
        # rows that no copy wrote are untouched: compare all slots but the destinations
        flat0 = kv0.view(2 * L, -1, H * c.head_dim)
        flat1 = c.kv.view(2 * L, -1, H * c.head_dim)
        idx = torch.nonzero(~written).flatten()
        for p in range(2 * L):
            assert torch.equal(flat1[p, idx], flat0[p, idx]), f"plane {p}: rows outside the copies changed"
    assert rep["max_rel_err_heads"] <= rtol and rep["max_rel_err_act"] <= rtol, rep
    rep["ok"] = True
    return rep
