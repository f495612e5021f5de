"""CPU oracle for the actkv eviction hot path.  TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
``--impl reference``) may import this module, and only as the checker or as the timed CPU
baseline.  The product path (``actkv_open_b200``) never imports it.

It restates, in numpy, the reference's torch path for the eviction hot path (actkv-open,
pure Python + torch; paths below are relative to that project):

    scoring        actkv/kernels/lse_attn.py:32-78   gather_kv, paged_decode_attention_ref,
                                                     action_scores_ref
    keep mask      actkv/paged.py:23-46              keep_mask_from_scores
    compaction     actkv/kernels/compaction.py:44-74 plan_compaction, apply_copies_ref
    paged cache    actkv/paged.py:49-157             PagedKVCache (allocator, tables, evict)
    ActionLRFU     actkv/eviction.py:20-50,152-224   reduce_heads, top_p_mask, ActionLRFU
    budget         actkv/budget.py:9-104             token_confidence, trace_confidence, fit_slope,
                                                     ConfidenceBudget (Algorithm 2)
    policies       actkv/eviction.py:52-56,89-149    StreamingLLM, SnapKV (keep indices per layer)

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against fixtures
produced by running the reference itself (``tests/golden/make_golden.py``), plus the
reference's own known-answer tests restated in ``tests/test_oracle_known_answers.py``.

Where the reference leaves an order unspecified (``torch.topk`` and ``torch.sort`` on exact
ties), this oracle picks the lowest index first, which is also what the CUDA kernels do.
"""
from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634


# ----------------------------------------------------------------------------- scoring

def gather_kv(kv: np.ndarray, block_table: np.ndarray, seq_used: int, row: int):
    """Contiguous K, V [S, Hkv, D] of one request (actkv/kernels/lse_attn.py:32-39)."""
    bs = kv.shape[2]
    n_blocks = math.ceil(seq_used / bs)
    blocks = block_table[row, :n_blocks].astype(np.int64)
    k = kv[0, blocks].reshape(-1, kv.shape[3], kv.shape[4])[:seq_used]
    v = kv[1, blocks].reshape(-1, kv.shape[3], kv.shape[4])[:seq_used]
    return k, v


def _group_logits(q_r: np.ndarray, k: np.ndarray, scale: float) -> np.ndarray:
    """[Hq, S] fp32 logits q.k*scale for one request; query head hq reads kv head hq // G."""
    hq, d = q_r.shape
    hkv = k.shape[1]
    g = hq // hkv
    qg = q_r.astype(np.float32).reshape(hkv, g, d)
    kt = np.ascontiguousarray(k.astype(np.float32).transpose(1, 2, 0))   # [Hkv, D, S]
    logits = np.matmul(qg, kt).reshape(hq, -1)
    return logits * np.float32(scale)


def paged_decode_attention(q, kv, block_table, seq_used, scale=None):
    """(out [R,Hq,D], lse [R,Hq]) of plain decode attention over the paged cache.

    Restates actkv/kernels/lse_attn.py:42-60.  The log-sum-exp is taken in float64 and rounded
    to float32 (torch takes it in float32; the two differ by about one ulp).
    """
    r_n, hq, d = q.shape
    scale = d ** -0.5 if scale is None else scale
    out = np.zeros((r_n, hq, d), np.float32)
    lse = np.zeros((r_n, hq), np.float32)
    for r in range(r_n):
        s = int(seq_used[r])
        k, v = gather_kv(kv, block_table, s, r)
        logits = _group_logits(q[r], k, scale).astype(np.float64)
        m = logits.max(-1, keepdims=True)
        e = np.exp(logits - m)
        z = e.sum(-1, keepdims=True)
        lse[r] = (m + np.log(z))[:, 0].astype(np.float32)
        hkv = k.shape[1]
        g = hq // hkv
        p = (e / z).reshape(hkv, g, s)
        vt = v.astype(np.float64).transpose(1, 0, 2)                         # [Hkv, S, D]
        out[r] = np.matmul(p, vt).reshape(hq, d).astype(np.float32)
    return out, lse


def causal_region_lse(q_region, kv, block_table_row, seq_len, scale=None):
    """lse [A, Hq] of the A action tokens that end a session of ``seq_len`` tokens.

    Action token j (0-based inside the region) attends to the first seq_len - A + j + 1 tokens,
    which is what the reference computes when it calls paged_decode_attention_ref once per action
    token with that seq_used (actkv/kernels/lse_attn.py:42-60).
    """
    a_n = q_region.shape[0]
    bt = block_table_row[None, :]
    lse = np.zeros(q_region.shape[:2], np.float32)
    for j in range(a_n):
        _, l = paged_decode_attention(q_region[j][None], kv, bt, [seq_len - a_n + j + 1], scale)
        lse[j] = l[0]
    return lse


def action_scores(q, kv, block_table, seq_used, lse, out, n_seen, scale=None):
    """Fold one action query per request into the running mean ``out`` (in place).

    Restates actkv/kernels/lse_attn.py:63-78: p = exp(q.k*scale - lse), max over each GQA group,
    out[r, :, :s] += (p - out) / (n_seen[r] + 1), then n_seen += 1.
    """
    r_n, hq, d = q.shape
    hkv = kv.shape[3]
    g = hq // hkv
    scale = d ** -0.5 if scale is None else scale
    for r in range(r_n):
        s = int(seq_used[r])
        k, _ = gather_kv(kv, block_table, s, r)
        logits = _group_logits(q[r], k, scale)
        p = np.exp(logits - lse[r][:, None].astype(np.float32))
        p = p.reshape(hkv, g, s).max(1)
        n = np.float32(n_seen[r])
        cur = out[r, :, :s]
        out[r, :, :s] = cur + (p - cur) / (n + np.float32(1.0))
    n_seen += 1
    return out


def action_scores_region(q_region, kv, block_table_row, seq_len, lse_region, out_row=None,
                         n_seen0=0, scale=None):
    """Scores [Hkv, W] of one session after folding its A causal action tokens, in order.

    Equivalent to A calls of action_scores where token j uses seq_used = seq_len - A + j + 1
    (the reference's per-token call sequence; the region is the last A tokens of the session).
    """
    a_n = q_region.shape[0]
    hkv = kv.shape[3]
    bs = kv.shape[2]
    width = block_table_row.shape[0] * bs
    out = np.zeros((1, hkv, width), np.float32) if out_row is None else out_row[None].copy()
    n_seen = np.array([n_seen0], np.int64)
    bt = block_table_row[None, :]
    for j in range(a_n):
        action_scores(q_region[j][None], kv, bt, [seq_len - a_n + j + 1], lse_region[j][None],
                      out, n_seen, scale)
    return out[0]


# ----------------------------------------------------------------------------- selection

def topk_lowest_index(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest entries; among equal values the lowest index wins."""
    order = np.argsort(-values.astype(np.float64), kind="stable")
    return np.sort(order[:k])


def keep_mask_from_scores(scores, seq_used, budget, protected=0, head_reduce="mean"):
    """Keep mask [seq_used]: the protected tokens plus the top-``budget`` others.

    Restates actkv/paged.py:23-46: heads (dim -2) are reduced with ``head_reduce`` then layers
    are averaged; ``protected`` is a prefix count or a bool mask.
    """
    if head_reduce not in ("mean", "max"):
        raise ValueError(head_reduce)
    s = np.asarray(scores)[..., :seq_used].astype(np.float32)
    if s.ndim >= 2:
        s = s.max(-2) if head_reduce == "max" else s.mean(-2, dtype=np.float32)
        s = s.reshape(-1, seq_used).mean(0, dtype=np.float32)
    if isinstance(protected, np.ndarray):
        keep = protected.astype(bool).copy()
    else:
        keep = np.arange(seq_used) < protected
    others = np.nonzero(~keep)[0]
    k = min(budget, others.size)
    if k > 0:
        keep[others[topk_lowest_index(s[others], k)]] = True
    return keep


def reduce_heads(attn: np.ndarray, n_kv_heads: int, how: str = "mean") -> np.ndarray:
    """[Hq, S] -> [S]: max over each GQA group, then mean/max over KV heads (eviction.py:20-33)."""
    hq, s = attn.shape
    g = hq // n_kv_heads
    per_kv = attn.reshape(n_kv_heads, g, s).max(1)
    if how == "mean":
        return per_kv.mean(0, dtype=np.float32)
    if how == "max":
        return per_kv.max(0)
    raise ValueError(how)


def top_p_mask(scores: np.ndarray, p: float) -> np.ndarray:
    """Nucleus mask (actkv/eviction.py:36-50): the fewest largest entries holding >= p of the
    mass, including the entry that crosses the threshold, and only entries > 0.

    The cumulative sum is accumulated in float64 and rounded to float32, as torch's CPU cumsum
    does; the target is float32(p * total).
    """
    scores = np.asarray(scores, np.float32)
    if scores.size == 0:
        return np.zeros(0, bool)
    total = np.float32(scores.sum(dtype=np.float32))
    if total <= 0:
        return np.zeros(scores.shape, bool)
    order = np.argsort(-scores.astype(np.float64), kind="stable")
    vals = scores[order]
    csum = np.cumsum(vals.astype(np.float64)).astype(np.float32)
    target = np.float32(np.float32(p) * total)
    n_keep = int(np.searchsorted(csum, target, side="left")) + 1
    n_keep = min(n_keep, scores.size)
    mask = np.zeros(scores.shape, bool)
    mask[order[:n_keep]] = True
    return mask & (scores > 0)


# ----------------------------------------------------------------------------- compaction

class CompactionPlan:
    """src/dst physical slots, perm (new logical -> old logical), drop_blocks
    (actkv/kernels/compaction.py:36-41)."""

    def __init__(self, src_slots, dst_slots, perm, drop_blocks):
        self.src_slots, self.dst_slots, self.perm, self.drop_blocks = src_slots, dst_slots, perm, drop_blocks


def plan_compaction(keep_mask, seq_used, block_table_row, block_size) -> CompactionPlan:
    """Algorithm 4 plan for one request (actkv/kernels/compaction.py:44-69).

    B kept tokens end up in the window [start, start + B) with start = (Y - X) * BS; kept tokens
    outside the window move, in ascending order, into the window's holes, in ascending order.
    """
    keep = np.asarray(keep_mask[:seq_used], bool)
    budget = int(keep.sum())
    y = math.ceil(seq_used / block_size)
    x = math.ceil(budget / block_size)
    start = (y - x) * block_size
    end = start + budget
    full = np.zeros(y * block_size, bool)
    full[:seq_used] = keep
    dst_logical = np.nonzero(~full[start:end])[0] + start
    outside = full.copy()
    outside[start:end] = False
    src_logical = np.nonzero(outside)[0]
    assert src_logical.size == dst_logical.size, "kept count must equal budget"
    table = np.asarray(block_table_row, np.int64)

    def to_phys(logical):
        return table[logical // block_size] * block_size + logical % block_size

    perm = np.arange(start, end, dtype=np.int64)
    perm[dst_logical - start] = src_logical
    return CompactionPlan(to_phys(src_logical), to_phys(dst_logical), perm, y - x)


def apply_copies(kv_flat: np.ndarray, src, dst) -> None:
    """kv_flat[:, dst] = kv_flat[:, src] over every plane (compaction.py:72-74)."""
    if len(src) == 0:
        return
    kv_flat[:, dst] = kv_flat[:, src]


# ----------------------------------------------------------------------------- paged cache

class OutOfBlocks(RuntimeError):
    pass


class PagedKVCache:
    """Host model of the reference's paged cache (actkv/paged.py:49-157), numpy storage.

    kv [L, 2, NB, BS, Hkv, D]; ``free`` is a LIFO list popped from its end; ``tables`` maps a
    request to its list of physical blocks; ``pinned`` holds each request's protected tokens.
    """

    def __init__(self, num_blocks, block_size, n_kv_heads, head_dim, n_layers=1, dtype=np.float32):
        self.block_size, self.n_kv_heads, self.head_dim = block_size, n_kv_heads, head_dim
        self.n_layers, self.num_blocks = n_layers, num_blocks
        self.kv = np.zeros((n_layers, 2, num_blocks, block_size, n_kv_heads, head_dim), dtype)
        self.free = list(range(num_blocks - 1, -1, -1))
        self.tables: dict[int, list[int]] = {}
        self.seq_used: dict[int, int] = {}
        self.pinned: dict[int, np.ndarray] = {}

    @property
    def used_blocks(self):
        return self.num_blocks - len(self.free)

    def _ensure(self, req, n_tokens):
        table = self.tables.setdefault(req, [])
        self.seq_used.setdefault(req, 0)
        need = math.ceil(n_tokens / self.block_size) - len(table)
        if need > len(self.free):
            raise OutOfBlocks(f"need {need} blocks, {len(self.free)} free")
        for _ in range(need):
            table.append(self.free.pop())

    def append(self, req, k, v):
        """k, v [L, n, Hkv, D] (actkv/paged.py:76-85)."""
        n = k.shape[1]
        start = self.seq_used.get(req, 0)
        self._ensure(req, start + n)
        slots = self.slot_map(req, start + n)[start:]
        flat = self.kv.reshape(self.n_layers, 2, -1, self.n_kv_heads, self.head_dim)
        flat[:, 0, slots] = k.astype(self.kv.dtype)
        flat[:, 1, slots] = v.astype(self.kv.dtype)
        self.seq_used[req] = start + n

    def release(self, req):
        self.free.extend(reversed(self.tables.pop(req, [])))
        self.seq_used.pop(req, None)
        self.pinned.pop(req, None)

    def slot_map(self, req, n=None):
        n = self.seq_used[req] if n is None else n
        table = np.asarray(self.tables[req], np.int64)
        pos = np.arange(n)
        return table[pos // self.block_size] * self.block_size + pos % self.block_size

    def block_table(self, reqs):
        mb = max(len(self.tables[r]) for r in reqs)
        bt = np.zeros((len(reqs), max(mb, 1)), np.int32)
        for i, r in enumerate(reqs):
            bt[i, :len(self.tables[r])] = self.tables[r]
        return bt

    def seq_tensor(self, reqs):
        return np.asarray([self.seq_used[r] for r in reqs], np.int32)

    def gather(self, req, layer=0):
        slots = self.slot_map(req)
        flat = self.kv[layer].reshape(2, -1, self.n_kv_heads, self.head_dim)
        return flat[0, slots], flat[1, slots]

    def compact(self, req, keep_mask):
        """Plan + copies over all 2L planes, then table/free-list update (actkv/paged.py:125-139)."""
        plan = plan_compaction(keep_mask, self.seq_used[req], self.tables[req], self.block_size)
        flat = self.kv.reshape(self.n_layers * 2, -1, self.n_kv_heads * self.head_dim)
        apply_copies(flat, plan.src_slots, plan.dst_slots)
        freed = self.tables[req][:plan.drop_blocks]
        self.tables[req] = self.tables[req][plan.drop_blocks:]
        self.free.extend(reversed(freed))
        self.seq_used[req] = plan.perm.size
        return plan.perm

    def evict(self, req, scores, budget, protected=0, head_reduce="mean"):
        """Scores -> keep mask -> compaction with pinned-token tracking (actkv/paged.py:141-157)."""
        n = self.seq_used[req]
        pinned = self.pinned.get(req, np.arange(n) < protected)
        pinned = np.concatenate([pinned, np.zeros(n - pinned.size, bool)])
        self.pinned[req] = pinned
        if n - int(pinned.sum()) <= budget:
            return np.arange(n)
        perm = self.compact(req, keep_mask_from_scores(scores, n, budget, pinned, head_reduce))
        self.pinned[req] = pinned[perm]
        return perm


# ----------------------------------------------------------------------------- ActionLRFU

class ActionLRFU:
    """ActKV Algorithm 1 (actkv/eviction.py:152-224) on numpy state ks, act [L, S].

    ``update_scores`` takes either the reference's protected prefix count or, for sessions whose
    protected tokens were moved by a paged compaction, a bool mask of the tokens to leave out
    (the prefix count is the special case mask = arange(S) < protected).
    """

    def __init__(self, decay=0.5, top_p=0.9, head_reduce="mean"):
        self.decay, self.top_p, self.head_reduce = decay, top_p, head_reduce

    def reset(self, n_layers):
        self.n_layers = n_layers
        self.ks = np.zeros((n_layers, 0), np.float32)
        self.act = np.zeros((n_layers, 0), np.float32)
        self.n_act = 0

    @staticmethod
    def _grow(t, length):
        if t.shape[1] >= length:
            return t
        return np.concatenate([t, np.zeros((t.shape[0], length - t.shape[1]), t.dtype)], 1)

    def begin_action(self):
        self.act[:] = 0
        self.n_act = 0

    def observe(self, scores, in_action):
        """Incremental mean of per-layer scores over action tokens (eviction.py:187-196)."""
        if not in_action:
            return
        length = max(s.size for s in scores)
        self.act = self._grow(self.act, length)
        cur = np.zeros_like(self.act)
        for layer, s in enumerate(scores):
            cur[layer, :s.size] = s
        self.n_act += 1
        self.act = self.act + (cur - self.act) / np.float32(self.n_act)

    def update_scores(self, length, protected=0):
        """ks = decay*ks + act*hit per layer, hit = nucleus of act (eviction.py:198-210)."""
        self.ks = self._grow(self.ks, length)[:, :length].copy()
        act = self._grow(self.act, length)[:, :length]
        if isinstance(protected, np.ndarray):
            free = ~protected[:length].astype(bool)
        else:
            free = np.arange(length) >= protected
        idx = np.nonzero(free)[0]
        decay = np.float32(self.decay)
        for layer in range(self.n_layers):
            a = act[layer, idx]
            hit = top_p_mask(a, self.top_p) if self.n_act else np.zeros(a.shape, bool)
            ks = self.ks[layer, idx] * decay
            ks[hit] = ks[hit] + a[hit]
            self.ks[layer, idx] = ks
        self.act[:] = 0
        self.n_act = 0

    def select(self, length, protected, budget):
        self.update_scores(length, protected)
        if length - protected <= budget:
            return None
        keeps = []
        for layer in range(self.n_layers):
            chosen = topk_lowest_index(self.ks[layer, protected:length], budget)
            keeps.append(np.sort(np.concatenate([np.arange(protected), chosen + protected])))
        return np.stack(keeps)

    def apply_keep(self, keep):
        self.ks = np.take_along_axis(self.ks, keep, 1)
        self.act = np.take_along_axis(self._grow(self.act, int(keep.max()) + 1), keep, 1)


# ----------------------------------------------------------------------------- pipeline glue

def layer_scores(kv_layer, block_table_row, seq_len, q_region, lse_region, scale=None):
    """Per-head scores [Hkv, S] of one layer after the session's causal action region."""
    out = action_scores_region(q_region, kv_layer, block_table_row, seq_len, lse_region,
                               scale=scale)
    return out[:, :seq_len]


def evict_session(cache: PagedKVCache, policy: ActionLRFU, req: int, q_region, lse_region,
                  budget: int, protected: int, scale=None):
    """One eviction step of one session: score every layer over the action region, fold the
    per-layer head-mean into ActionLRFU as the round's action attention, update keep scores, and
    evict with the layer-mean of the keep scores.  Returns (perm, per-layer head scores).

    q_region [L, A, Hq, D], lse_region [L, A, Hq].  ``policy`` holds this session's state and
    must have been reset to the cache's layer count; its protected tokens are the cache's pinned
    tokens (the prefix ``protected`` on a session's first eviction).
    """
    n = cache.seq_used[req]
    bt = np.asarray(cache.tables[req], np.int64)
    head_scores = np.stack([
        layer_scores(cache.kv[l], bt, n, q_region[l], lse_region[l], scale)
        for l in range(cache.n_layers)])                                  # [L, Hkv, n]
    act = head_scores.mean(1, dtype=np.float32) if policy.head_reduce == "mean" else head_scores.max(1)
    policy.act = policy._grow(policy.act, n)
    policy.act[:, :n] = act
    policy.n_act = q_region.shape[1]
    pinned = cache.pinned.get(req, np.arange(n) < protected)
    pinned = np.concatenate([pinned, np.zeros(n - pinned.size, bool)])
    policy.update_scores(n, pinned)
    perm = cache.evict(req, policy.ks[:, :n], budget, protected)
    if perm.size != n or not np.array_equal(perm, np.arange(n)):
        keep = np.broadcast_to(perm, (policy.n_layers, perm.size))
        policy.ks = np.take_along_axis(policy.ks, keep, 1)
        policy.act = np.zeros_like(policy.ks)
    return perm, head_scores


# --------------------------------------------------------------------------- adaptive budget
def token_confidence(logits, k: int = 20) -> float:
    """T = -(1/k) * sum of the k largest log-softmax values of one row (actkv/budget.py:9-17):
    large for a peaked next-token distribution.  log_softmax and the mean are taken in float32, as
    torch does for a float32 row."""
    x = np.asarray(logits, np.float32).astype(np.float64)
    m = x.max()
    logp = (x - m - np.log(np.exp(x - m).sum())).astype(np.float32)
    k = min(k, logp.size)
    top = np.sort(logp)[::-1][:k]
    return float(-np.float32(top.astype(np.float64).sum() / k))


def trace_confidence(tl, window: int, stride: int, bottom_pct: float):
    """Sliding-window min pooling of the confidence trace, then the pooled values at or below the
    bottom_pct quantile (linear interpolation, as torch.quantile): returns their window indices x
    and values y (actkv/budget.py:20-36)."""
    t = np.asarray(tl, np.float64)
    n = t.size
    if n == 0:
        return np.zeros(0), np.zeros(0)
    if n < window:
        window = n
    P = (n - window) // stride + 1
    pooled = np.array([t[i * stride:i * stride + window].min() for i in range(P)])
    v = np.sort(pooled)
    pos = (bottom_pct / 100.0) * (P - 1)
    lo = int(math.floor(pos))
    hi = min(lo + 1, P - 1)
    w = pos - lo
    thresh = v[lo] + w * (v[hi] - v[lo]) if w < 0.5 else v[hi] - (v[hi] - v[lo]) * (1 - w)
    keep = pooled <= thresh
    return np.arange(P, dtype=np.float64)[keep], pooled[keep]


def fit_slope(x, y) -> float:
    """Least-squares slope of y on x; fewer than two points or no spread in x gives 0
    (actkv/budget.py:39-47)."""
    x = np.asarray(x, np.float64)
    y = np.asarray(y, np.float64)
    if x.size < 2:
        return 0.0
    xm, ym = x.mean(), y.mean()
    var = ((x - xm) ** 2).sum()
    if var == 0:
        return 0.0
    return float(((x - xm) * (y - ym)).sum() / var)


class ConfidenceBudget:
    """Algorithm 2 (actkv/budget.py:65-104): the budget grows by scale_up (capped at upper) when
    the fitted slope of the low-confidence trace is negative; with ``bidirectional`` it shrinks by
    scale_down (floored at lower) after shrink_patience compressions in a row whose slope exceeds
    shrink_slope."""

    def __init__(self, top_k=20, window=64, stride=8, bottom_pct=10.0, init_budget=512, scale_up=1.75,
                 upper=30_000, bidirectional=False, shrink_patience=3, shrink_slope=0.0, scale_down=1.75,
                 lower=256):
        self.top_k, self.window, self.stride, self.bottom_pct = top_k, window, stride, bottom_pct
        self.scale_up, self.upper, self.bidirectional = scale_up, upper, bidirectional
        self.shrink_patience, self.shrink_slope, self.scale_down, self.lower = (shrink_patience, shrink_slope,
                                                                                scale_down, lower)
        self.budget = init_budget
        self.tl: list[float] = []
        self.history = [init_budget]
        self.slopes: list[float] = []
        self._rising = 0

    @property
    def current(self) -> int:
        return self.budget

    def record(self, logits) -> None:
        self.tl.append(token_confidence(logits, self.top_k))

    def slope(self) -> float:
        return fit_slope(*trace_confidence(self.tl, self.window, self.stride, self.bottom_pct))

    def next_budget(self) -> int:
        a = self.slope()
        self.slopes.append(a)
        if a < 0:
            self.budget = min(int(self.budget * self.scale_up), self.upper)
            self._rising = 0
        elif self.bidirectional and a > self.shrink_slope:
            self._rising += 1
            if self._rising >= self.shrink_patience:
                self.budget = max(int(self.budget / self.scale_down), self.lower)
                self._rising = 0
        else:
            self._rising = 0
        self.history.append(self.budget)
        return self.budget


# --------------------------------------------------------------------------- StreamingLLM / SnapKV
def _keep_indices(protected: int, length: int, chosen_rel: np.ndarray) -> np.ndarray:
    """Sorted keep indices: the protected prefix plus ``protected + chosen_rel`` (eviction.py:52-56)."""
    return np.sort(np.concatenate([np.arange(protected), np.asarray(chosen_rel, np.int64) + protected]))


class StreamingLLM:
    """Attention sinks plus the most recent ``budget`` tokens, the same in every layer
    (actkv/eviction.py:89-100)."""

    def reset(self, n_layers):
        self.n_layers = n_layers

    def select(self, length, protected, budget):
        if length - protected <= budget:
            return None
        keep = np.concatenate([np.arange(protected), np.arange(length - budget, length)])
        return np.tile(keep, (self.n_layers, 1))


class SnapKV:
    """Scores = attention of the last ``window`` observed query tokens, summed, avg-pooled with
    kernel ``pool`` (stride 1, zero padding pool // 2, divisor pool); the observation window
    itself is always kept, the rest of the budget goes to the top-scoring older tokens, ties to
    the lowest index (actkv/eviction.py:103-149)."""

    def __init__(self, window=32, pool=7):
        self.window, self.pool = window, pool

    def reset(self, n_layers):
        self.n_layers = n_layers
        self.rows: list[list[np.ndarray]] = []

    def observe(self, scores):
        self.rows.append([np.asarray(x, np.float32) for x in scores])
        if len(self.rows) > self.window:
            self.rows.pop(0)

    def layer_scores(self, length, w):
        out = []
        for layer in range(self.n_layers):
            acc = np.zeros(length, np.float32)
            for row in (self.rows[-w:] if w else []):
                r = row[layer]
                n = min(r.size, length)
                acc[:n] += r[:n]
            if self.pool > 1:
                pad = self.pool // 2
                padded = np.concatenate([np.zeros(pad, np.float32), acc, np.zeros(self.pool, np.float32)])
                acc = np.array([padded[t:t + self.pool].sum(dtype=np.float32) / np.float32(self.pool)
                                for t in range(length)], np.float32)
            out.append(acc)
        return out

    def select(self, length, protected, budget):
        if length - protected <= budget:
            return None
        w = min(len(self.rows), budget)
        keeps = []
        for acc in self.layer_scores(length, w):
            win_start = length - w
            cand = acc[protected:win_start]
            k = budget - w
            chosen = topk_lowest_index(cand, k) if k > 0 else np.zeros(0, np.int64)
            window_idx = np.arange(win_start - protected, length - protected)
            keeps.append(_keep_indices(protected, length, np.concatenate([chosen, window_idx])))
        return np.stack(keeps)

    def apply_keep(self, keep):
        for row in self.rows:
            for layer in range(self.n_layers):
                r = row[layer]
                idx = keep[layer][keep[layer] < r.size]
                row[layer] = r[idx]
