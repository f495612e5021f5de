"""ActionLRFU (ActKV Algorithm 1) on device state, plus ``reduce_heads`` and ``top_p_mask``: the
eviction-policy part of ``actkv.eviction`` (actkv/eviction.py:20-50, 152-224) that the eviction
hot path uses.

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
        cur = torch.zeros_like(self.act)
        for layer, s in enumerate(scores):
            cur[layer, : s.numel()] = s.float()
        self.n_act += 1
        self.act += (cur - self.act) / self.n_act

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


def make_policy(name: str, cfg: EvictionConfig | None = None, **kw):
    """Policy factory restricted to the eviction hot path: ActionLRFU."""
    if name.lower() in ("actkv", "action", "lrfu"):
        return ActionLRFU(cfg)
    raise ValueError(f"unknown policy {name} (this package implements the ActionLRFU eviction path)")
