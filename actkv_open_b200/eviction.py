"""ActionLRFU (ActKV Algorithm 1) on device state, plus ``reduce_heads`` and ``top_p_mask``: the
eviction-policy part of ``actkv.eviction`` (actkv/eviction.py:20-50, 152-224) that the eviction
hot path uses; and the reference's baseline policies FullKV, StreamingLLM and SnapKV
(eviction.py:80-149) with their selections on the device.

Per layer and per cached token:
  act[l, i]  mean, over the action tokens of the current round, of the attention the action query
             paid to entry i (max over the GQA group, mean over KV heads)
  ks[l, i]   keep score, updated once per compression step:
             ks = decay * ks + act * hit,  hit = entry is in the top-p mass of act
``update_scores`` runs the fused nucleus + decay kernel (one CTA per layer); ``select`` runs the
top-k keep-mask kernel on every layer at once.
"""
from __future__ import annotations

import torch

from . import _native as N
from .config import EvictionConfig


def reduce_heads(attn: torch.Tensor, n_kv_heads: int, how: str = "mean") -> torch.Tensor:
    """[Hq, S] attention probs of one query token -> [S]: max over each GQA group (Algorithm 3,
    step 4), then mean or max over KV heads (eviction.py:20-33)."""
    hq, s = attn.shape
    per_kv = attn.view(n_kv_heads, hq // n_kv_heads, s).amax(dim=1)
    if how == "mean":
        return per_kv.mean(0)
    if how == "max":
        return per_kv.amax(0)
    raise ValueError(how)


def _small_i32(values, device) -> torch.Tensor:
    return torch.tensor(values, dtype=torch.int32).pin_memory().to(device, non_blocking=True)


def _lrfu(act: torch.Tensor, ks: torch.Tensor, length: int, protected, decay: float, top_p: float,
          has_action: bool, act_out: torch.Tensor | None = None) -> None:
    """ks[:, :length] (L rows, in place) <- decay*ks + act*hit on the device; protected tokens kept."""
    dev = N.require_cuda(act, ks)
    assert act.dtype == torch.float32 and ks.dtype == torch.float32
    assert act.stride(-1) == 1 and ks.stride(-1) == 1
    L = ks.shape[0]
    if isinstance(protected, torch.Tensor):
        pin = protected.to(device=dev)[:length].contiguous()
        pin = pin.view(torch.uint8) if pin.dtype == torch.bool else (pin != 0).to(torch.uint8)
        prefix = 0
    else:
        pin, prefix = None, int(protected)
    out = act_out if act_out is not None else torch.empty(L, max(length, 1), device=dev)
    meta = _small_i32([length, 0], dev)
    N.check(N.load().actkv_lrfu_update(
        act.data_ptr(), None, 0, act.stride(0), 0, 1, N.REDUCE_MEAN,
        ks.data_ptr(), 0, ks.stride(0), out.data_ptr(), 0, out.stride(0),
        N.ptr(pin), 0, prefix, meta[0:1].data_ptr(), None if has_action else meta[1:2].data_ptr(),
        1, L, length, float(decay), float(top_p), N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "lrfu_update")


def top_p_mask(scores: torch.Tensor, p: float) -> torch.Tensor:
    """Bool mask of the smallest set of largest entries holding >= p of the total score mass,
    including the crossing entry, restricted to entries > 0 (eviction.py:36-50)."""
    n = scores.numel()
    if n == 0:
        return torch.zeros_like(scores, dtype=torch.bool)
    s = scores.float().contiguous().view(1, n)
    ks = torch.zeros_like(s)
    _lrfu(s, ks, n, 0, 0.0, p, True)
    return (ks > 0).view(scores.shape)


class ActionLRFU:
    """ActKV Algorithm 1: protected prefix plus the top-``budget`` keep scores per layer."""

    name = "actkv"
    ora_only = True
    needs_attention = True

    def __init__(self, cfg: EvictionConfig | None = None):
        self.cfg = cfg or EvictionConfig()
        self.head_reduce = self.cfg.head_reduce

    def reset(self, n_layers: int, device="cuda") -> None:
        self.n_layers = n_layers
        self.device = device
        self.ks = torch.zeros(n_layers, 0, device=device)
        self.act = torch.zeros(n_layers, 0, device=device)
        self.n_act = 0

    @staticmethod
    def _grow(t: torch.Tensor, length: int) -> torch.Tensor:
        if t.shape[1] >= length:
            return t
        return torch.cat([t, t.new_zeros(t.shape[0], length - t.shape[1])], 1)

    def begin_action(self) -> None:
        # accumulated state is reset on entry to each action region
        self.act.zero_()
        self.n_act = 0

    def observe(self, scores, in_action: bool) -> None:
        """Fold one action token's per-layer scores into the running mean ``act``."""
        if not in_action:
            return
        length = max(s.numel() for s in scores)
        self.act = self._grow(self.act, length)
        L, width = self.act.shape
        if len(scores) == L and all(s.numel() == width for s in scores):
            cur = torch.stack([s.reshape(-1) for s in scores]).float()     # every layer in one launch
        else:
            cur = torch.zeros_like(self.act)
            for layer, s in enumerate(scores):
                cur[layer, : s.numel()] = s.float()
        self.n_act += 1
        self.act.add_(cur.sub_(self.act).div_(self.n_act))               # act += (cur - act) / n_act

    def update_scores(self, length: int, protected) -> None:
        """Algorithm 1 steps 2-4: nucleus hits of this round's ``act`` and the decayed keep score.

        ``protected`` is a count of leading tokens or a bool mask of tokens left untouched.
        """
        self.ks = self._grow(self.ks, length)[:, :length].contiguous()
        act = self._grow(self.act, length)[:, :length].contiguous()
        if length:
            _lrfu(act, self.ks, length, protected, self.cfg.decay, self.cfg.top_p, self.n_act > 0)
        # this round's action attention is spent; a round without an action only decays
        self.act.zero_()
        self.n_act = 0

    def select(self, length: int, protected: int, budget: int):
        """Return LongTensor [n_layers, protected + budget] of indices to keep (sorted), or None."""
        self.update_scores(length, protected)
        if length - protected <= budget:
            return None
        dev = self.ks.device
        L = self.n_layers
        keep = torch.empty(L, length, dtype=torch.uint8, device=dev)
        meta = _small_i32([length] * L + [budget] * L, dev)
        lib = N.load()
        ws = N.workspace(lib.actkv_keep_mask_workspace_bytes(L, length), dev)
        N.check(lib.actkv_keep_mask(self.ks.data_ptr(), None, self.ks.stride(0), 0, 0, 1, 1, N.REDUCE_MEAN,
                                    None, 0, int(protected), meta[:L].data_ptr(), meta[L:].data_ptr(), 0,
                                    keep.data_ptr(), length, None, L, length, ws.data_ptr(), ws.numel(),
                                    N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "select")
        idx = keep.view(torch.bool).nonzero()[:, 1]
        return idx.view(L, int(protected) + budget)

    def apply_keep(self, keep: torch.Tensor) -> None:
        """Compact the policy state after the backend kept ``keep`` [n_layers, n] (eviction.py:222-224)."""
        self.ks = torch.gather(self.ks, 1, keep)
        self.act = torch.gather(self._grow(self.act, int(keep.max()) + 1), 1, keep)


class Policy:
    """The reference's policy interface (eviction.py:58-80): backends call reset, begin_action,
    observe, select (keep indices [n_layers, protected + budget], sorted, or None when within
    budget) and apply_keep."""

    name = "base"
    ora_only = True
    needs_attention = True
    head_reduce = "mean"

    def reset(self, n_layers: int, device="cuda") -> None:
        self.n_layers = n_layers
        self.device = device

    def begin_action(self) -> None: ...

    def observe(self, scores, in_action: bool) -> None: ...

    def select(self, length: int, protected: int, budget: int):
        raise NotImplementedError

    def apply_keep(self, keep: torch.Tensor) -> None: ...


class FullKV(Policy):
    """Never evicts (eviction.py:80-86)."""

    name = "full"
    needs_attention = False

    def select(self, length, protected, budget):
        return None


class StreamingLLM(Policy):
    """Attention sinks (the protected prefix) plus the last ``budget`` tokens, the same in every
    layer (eviction.py:89-100); the indices are written on the device (actkv_streaming_keep)."""

    name = "streaming"
    ora_only = False
    needs_attention = False

    def select(self, length, protected, budget):
        if length - protected <= budget:
            return None
        dev = torch.device(self.device)
        keep = torch.empty(self.n_layers, protected + budget, dtype=torch.int64, device=dev)
        N.require_cuda(keep)
        N.check(N.load().actkv_streaming_keep(keep.data_ptr(), keep.stride(0), self.n_layers, length, protected,
                                              budget, N.stream_ptr(dev)), "streaming select")
        return keep


class SnapKV(Policy):
    """Scores = attention of the last ``window`` observed query tokens, summed and average-pooled
    (kernel ``pool``); the observation window is always kept, the rest of the budget goes to the
    top-scoring older tokens of each layer (eviction.py:103-149).

    The observed rows live on the device in a ring of ``window`` slots [slot, layer, max_len]
    (double-buffered for ``apply_keep``); select runs the pooling, keep-mask and index kernels
    with no host round trip (ties go to the lowest index)."""

    name = "snapkv"
    ora_only = False

    def __init__(self, window: int = 32, pool: int = 7, head_reduce: str = "mean", max_len: int = 4096):
        if not 1 <= window <= 64:
            raise ValueError("window must be in [1, 64]")
        if not 1 <= pool <= 64:
            raise ValueError("pool must be in [1, 64]")
        self.window, self.pool, self.head_reduce, self.max_len = window, pool, head_reduce, max_len

    def reset(self, n_layers, device="cuda"):
        super().reset(n_layers, device)
        self.order: list[int] = []          # ring slots of the stored rows, oldest first
        self._alloc(self.max_len)

    def _alloc(self, W: int) -> None:
        dev = torch.device(self.device)
        old = getattr(self, "_buf", None)
        buf = [torch.zeros(self.window, self.n_layers, W, device=dev) for _ in range(2)]
        lens = torch.zeros(self.window, self.n_layers, dtype=torch.int32, device=dev)
        if old is not None:
            w0 = old[self._cur].shape[2]
            buf[0][:, :, :w0].copy_(old[self._cur])
            lens.copy_(self._lens)
        self._buf, self._cur, self._lens, self.W = buf, 0, lens, W
        self._ws = N.workspace(N.load().actkv_snapkv_workspace_bytes(self.n_layers, W), dev)

    @property
    def rows(self) -> list[list[torch.Tensor]]:
        """The stored rows, oldest first, as [layer][S_i] tensors (a synchronising read)."""
        lens = self._lens.cpu()
        return [[self._buf[self._cur][s, l, :int(lens[s, l])] for l in range(self.n_layers)] for s in self.order]

    def observe(self, scores, in_action):
        length = max(int(x.numel()) for x in scores)
        if length > self.W:
            self._alloc(max(length, 2 * self.W))
        if len(self.order) < self.window:
            slot = len(self.order)
        else:
            slot = self.order.pop(0)
        self.order.append(slot)
        dst = self._buf[self._cur][slot]
        sizes = [int(x.numel()) for x in scores]
        if all(n == length for n in sizes):
            dst[:, :length].copy_(torch.stack([x.float() for x in scores]))
        else:
            for layer, x in enumerate(scores):
                dst[layer, :x.numel()].copy_(x.float())
        self._lens[slot].copy_(torch.tensor(sizes, dtype=torch.int32))

    def select(self, length, protected, budget):
        if length - protected <= budget:
            return None
        if length > self.W:
            self._alloc(length)
        w = min(len(self.order), budget)
        dev = torch.device(self.device)
        keep = torch.empty(self.n_layers, protected + budget, dtype=torch.int64, device=dev)
        slots = (ctypes_int_array(self.order[-w:]) if w else None)
        buf = self._buf[self._cur]
        N.check(N.load().actkv_snapkv_select(
            buf.data_ptr(), buf.stride(0), buf.stride(1), self._lens.data_ptr(), self._lens.stride(0), slots, w,
            self.n_layers, self.W, length, protected, budget, self.pool, keep.data_ptr(), keep.stride(0),
            self._ws.data_ptr(), self._ws.numel(), N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "snapkv select")
        return keep

    def apply_keep(self, keep):
        """Past rows index the old layout: gather them by the kept indices (eviction.py:143-149)."""
        if not self.order:
            return
        keep = keep.to(torch.int64).contiguous()
        dev = torch.device(self.device)
        src, dst = self._buf[self._cur], self._buf[1 - self._cur]
        N.check(N.load().actkv_snapkv_compact_rows(
            src.data_ptr(), dst.data_ptr(), src.stride(0), src.stride(1), self._lens.data_ptr(), self._lens.stride(0),
            ctypes_int_array(self.order), len(self.order), self.n_layers, keep.data_ptr(), keep.stride(0),
            keep.shape[1], N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "snapkv apply_keep")
        self._cur = 1 - self._cur


def ctypes_int_array(values):
    import ctypes
    return (ctypes.c_int * len(values))(*values)


def make_policy(name: str, cfg: EvictionConfig | None = None, **kw):
    """The reference's policy factory (eviction.py:227-237)."""
    name = name.lower()
    if name in ("full", "fullkv"):
        return FullKV()
    if name in ("actkv", "action", "lrfu"):
        return ActionLRFU(cfg)
    if name == "snapkv":
        return SnapKV(**kw)
    if name in ("streaming", "streamingllm"):
        return StreamingLLM()
    raise ValueError(f"unknown policy {name}")
