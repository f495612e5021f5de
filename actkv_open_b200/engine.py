"""Device-resident eviction for a batch of sessions: the whole hot path (score -> ActionLRFU ->
keep mask -> compaction -> state permutation) as six kernel launches on one stream, with no
device->host synchronisation anywhere in a step.

``DevicePagedCache`` holds what the reference keeps in Python lists (actkv/paged.py:54-60) in device
arrays: block tables [R, MB] int32, token counts [R] int32, the free stack [NB] int32 with its top,
and each session's pinned tokens [R, W] uint8.  ``EvictionPipeline.step`` chains, for every session
at once, what the reference does per request (actkv/paged.py:120-157 and actkv/eviction.py:198-224):

  1 action_scores_region   per-head scores of every layer over the causal action region (tcgen05)
  2 lrfu_update            act = mean over KV heads; nucleus hits; ks = decay*ks + act*hit
  3 keep_mask              layer-mean of ks; pinned tokens + top-budget others; within-budget no-op
  4 compact                plan + row copies over all 2L planes + table / free-stack / length update
  5 permute                ks and pinned follow the tokens (perm), into the other buffer

Sessions are evicted as the reference's loop ``for r in reqs: cache.evict(r, ...)`` would: in
particular the freed blocks reach the free stack in session order, each session's reversed.

With a process group (``group=``), the cache holds this rank's KV-head slice and step 2 starts with
the one exchange of the path: the local head reduction is all-reduced over the group (see
``sharding``), so every rank runs the same ActionLRFU / keep mask / compaction plan on its slice.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _native as N
from . import sharding
from ._native import OutOfBlocks
from .config import EvictionConfig
from .kernels.lse_attn import (action_region_lse, action_scores_region, region_lse_workspace_bytes,
                                score_region_workspace_bytes, stream_signal)


class DevicePagedCache:
    def __init__(self, num_blocks: int, block_size: int, n_kv_heads: int, head_dim: int, n_layers: int,
                 max_sessions: int, max_tokens: int, dtype=torch.bfloat16, device="cuda", kv=None):
        self.num_blocks, self.block_size = num_blocks, block_size
        self.n_kv_heads, self.head_dim, self.n_layers = n_kv_heads, head_dim, n_layers
        self.max_sessions, self.max_tokens = max_sessions, max_tokens
        self.device = torch.device(device)
        self.max_blocks = math.ceil(max_tokens / block_size)
        self.kv = kv if kv is not None else torch.zeros(n_layers, 2, num_blocks, block_size, n_kv_heads, head_dim,
                                                        dtype=dtype, device=self.device)
        assert tuple(self.kv.shape) == (n_layers, 2, num_blocks, block_size, n_kv_heads, head_dim)
        assert self.kv.is_contiguous()
        self.block_table = torch.zeros(max_sessions, self.max_blocks, dtype=torch.int32, device=self.device)
        self.seq_used = torch.zeros(max_sessions, dtype=torch.int32, device=self.device)
        self.free_list = torch.zeros(num_blocks, dtype=torch.int32, device=self.device)
        self.free_top = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.pinned = torch.zeros(max_sessions, max_tokens, dtype=torch.uint8, device=self.device)
        self.n_sessions = 0
        self._blocks_ws = None
        # pinned staging for the small per-call inputs of append / release (offsets, masks): reused,
        # guarded by the event of the last copy out of it
        self._stage = torch.empty(max_sessions + 1, dtype=torch.int32).pin_memory()
        self._stage_dev = torch.zeros(max_sessions + 1, dtype=torch.int32, device=self.device)
        self._stage_ev = None

    def _upload(self, values) -> torch.Tensor:
        """values (host ints, at most max_sessions + 1) -> a device int32 tensor, asynchronously."""
        if self._stage_ev is not None:
            self._stage_ev.synchronize()          # the previous copy out of the staging buffer is done
        n = len(values)
        self._stage[:n] = torch.as_tensor(values, dtype=torch.int32)
        out = self._stage_dev[:n]
        out.copy_(self._stage[:n], non_blocking=True)
        self._stage_ev = torch.cuda.Event()
        self._stage_ev.record()
        return out

    def set_state(self, tables: list[list[int]], seq_lens: list[int], free: list[int], protected: int = 0):
        """Load tables / lengths / free list (one host->device copy each); pins each session's
        first ``protected`` tokens."""
        R = len(tables)
        assert R <= self.max_sessions and max(seq_lens) <= self.max_tokens
        bt = torch.zeros(R, self.max_blocks, dtype=torch.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        self.block_table[:R].copy_(bt)
        self.seq_used[:R].copy_(torch.tensor(seq_lens, dtype=torch.int32))
        self.free_list.zero_()
        if free:
            self.free_list[:len(free)].copy_(torch.tensor(free, dtype=torch.int32))
        self.free_top.fill_(len(free))
        self.pinned[:R].zero_()
        if protected:
            self.pinned[:R, :protected] = 1
        self.n_sessions = R

    def state(self):
        """(tables, seq_lens, free) read back to the host (synchronises)."""
        R = self.n_sessions
        seq = self.seq_used[:R].tolist()
        bt = self.block_table[:R].cpu()
        tables = [bt[i, :math.ceil(seq[i] / self.block_size)].tolist() for i in range(R)]
        top = int(self.free_top.item())
        return tables, seq, self.free_list[:top].tolist()

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, n_new, max_new: int | None = None,
               check: bool = True) -> None:
        """Append n_new[r] tokens to session r for every r, in session order, on the device
        (PagedKVCache.append for each request, actkv/paged.py:67-85).

        k_new / v_new [L, sum(n_new), Hkv, D] hold the new rows of all sessions packed along dim 1.
        ``n_new``: host list of counts, or a device int32 tensor of offsets [R+1] (then ``max_new``
        bounds the counts and nothing touches the host).  Sessions beyond ``n_sessions`` start
        empty.  Blocks come from the top of the device free stack, session 0 first; from the first
        session whose blocks do not fit on, nothing is appended, and with ``check`` (which
        synchronises) OutOfBlocks is raised, as the reference raises at that request."""
        lib = N.load()
        dev = self.device
        if isinstance(n_new, torch.Tensor):
            off = n_new
            R = off.numel() - 1
            if max_new is None:
                raise ValueError("max_new is required with device offsets")
        else:
            counts = [int(x) for x in n_new]
            R = len(counts)
            if R > self.max_sessions:
                raise ValueError(f"{R} sessions, room for {self.max_sessions}")
            offs = [0]
            for x in counts:
                offs.append(offs[-1] + x)
            off = self._upload(offs)
            max_new = max(counts) if counts else 0
        if R > self.max_sessions:
            raise ValueError(f"{R} sessions, room for {self.max_sessions}")
        L, H, D = self.n_layers, self.n_kv_heads, self.head_dim
        assert k_new.shape == v_new.shape and k_new.dim() == 4 and tuple(k_new.shape[::2]) == (L, H) and \
            k_new.shape[3] == D, "k_new / v_new must be [L, sum(n_new), Hkv, D]"
        assert k_new.dtype == self.kv.dtype and v_new.dtype == self.kv.dtype
        assert k_new.stride(2) == D and k_new.stride(3) == 1 and v_new.stride() == k_new.stride()
        es = self.kv.element_size()
        ws = self._blocks_workspace()
        plane, slot, row, n_slots = self.flat_planes()
        N.check(lib.actkv_append(
            self.kv.data_ptr(), L, plane, slot, row, n_slots, k_new.data_ptr(), v_new.data_ptr(),
            k_new.stride(0) * es, k_new.stride(1) * es, off.data_ptr(), int(max_new), self.seq_used.data_ptr(),
            self.block_table.data_ptr(), self.block_table.stride(0), self.max_blocks, self.block_size,
            self.free_list.data_ptr(), self.free_top.data_ptr(), self.num_blocks, R, ws.data_ptr(), ws.numel(),
            N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "append")
        self.n_sessions = max(self.n_sessions, R)
        if check:
            bits = N.read_device_status(dev)
            if bits & N.DEV_OUT_OF_BLOCKS:
                raise OutOfBlocks("append: the free stack (or a table row) ran out of blocks")
            if bits:
                raise RuntimeError(f"append: device status {bits:#x}")

    def _blocks_workspace(self) -> torch.Tensor:
        if self._blocks_ws is None:
            self._blocks_ws = N.workspace(N.load().actkv_blocks_workspace_bytes(self.max_sessions), self.device)
        return self._blocks_ws

    def release(self, sessions) -> None:
        """Release sessions (PagedKVCache.release, actkv/paged.py:87-90), in session order: their
        blocks go back onto the free stack in reverse table order, and their tables, lengths and
        pinned tokens are cleared.  No host synchronisation."""
        lib = N.load()
        dev = self.device
        R = self.n_sessions
        flags = [0] * max(R, 1)
        for r in sessions:
            if not 0 <= int(r) < R:
                raise ValueError(f"session {r} of {R}")
            flags[int(r)] = 1
        # the kernel reads release[r] as one byte: pack four flags per staged int32
        packed = [sum(flags[i + b] << (8 * b) for b in range(4) if i + b < len(flags)) for i in range(0, len(flags), 4)]
        mask = self._upload(packed).view(torch.uint8)
        ws = self._blocks_workspace()
        N.check(lib.actkv_release(
            mask.data_ptr(), self.seq_used.data_ptr(), self.block_table.data_ptr(), self.block_table.stride(0),
            self.max_blocks, self.block_size, self.free_list.data_ptr(), self.free_top.data_ptr(), self.num_blocks,
            self.pinned.data_ptr(), self.pinned.stride(0), self.max_tokens, R, ws.data_ptr(), ws.numel(),
            N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "release")

    def flat_planes(self):
        """(plane_stride_bytes, slot_stride_bytes, row_bytes, n_slots) of the [2L, NB*BS, Hkv*D] view."""
        es = self.kv.element_size()
        row = self.n_kv_heads * self.head_dim * es
        return self.kv.stride(1) * es, row, row, self.num_blocks * self.block_size


def _no_mark(name) -> None:
    pass


def _stream_groups(L: int, n: int = 16) -> list[int]:
    """Layer boundaries of step_host's streamed groups: one layer first (the only copy nothing
    hides), then the rest in up to n - 1 near-equal groups, each signalled as soon as it lands."""
    if L <= 1:
        return [0, L]
    m = min(n - 1, L - 1)
    return [0] + [1 + (L - 1) * i // m for i in range(m + 1)]


def _growing_groups(L: int, n: int, ratio: float = 1.4) -> list[int]:
    """Layer boundaries of n groups whose sizes grow by ``ratio``: the first copy, which nothing
    hides, is short, and each later group's copy (~19 us per config-2 layer at ~54 GB/s) still
    lands before the previous group's scoring (~30 us per layer) ends.  Every group costs a
    scoring launch; on config 2, 4 growing groups measured best (e2e 0.19 ms over the device
    step, against 0.24 ms for 6 equal groups)."""
    n = max(1, min(n, L))
    w = [ratio ** i for i in range(n)]
    tot = sum(w)
    bounds, acc = [0], 0.0
    for i in range(n):
        acc += w[i]
        b = L if i == n - 1 else max(bounds[-1] + 1, min(L - (n - 1 - i), round(L * acc / tot)))
        bounds.append(b)
    return bounds


class EvictionPipeline:
    def __init__(self, cache: DevicePagedCache, cfg: EvictionConfig | None = None, scale: float | None = None,
                 path: str = "auto", group=None, total_kv_heads: int | None = None):
        """``group`` / ``total_kv_heads``: KV-head sharding; ``cache`` then holds this rank's heads and
        ``total_kv_heads`` is the head count over all ranks (the divisor of the head mean)."""
        self.cache = cache
        self.group = group
        self.total_kv_heads = total_kv_heads if total_kv_heads is not None else cache.n_kv_heads
        if group is None and self.total_kv_heads != cache.n_kv_heads:
            raise ValueError("total_kv_heads differs from the cache's heads but no process group was given")
        self.cfg = cfg or EvictionConfig()
        if self.cfg.head_reduce not in ("mean", "max"):
            raise ValueError(self.cfg.head_reduce)
        self.scale = scale
        self.path = path
        c, dev = cache, cache.device
        R, L, H, W = c.max_sessions, c.n_layers, c.n_kv_heads, c.max_tokens
        self.heads = torch.zeros(R, L, H, W, device=dev)          # per-head scores of the round
        self.act = torch.zeros(R, L, W, device=dev)               # the round's action attention
        # sharded: the all-reduced head reduction (a view of ``heads`` when a rank holds one head)
        self.part = torch.zeros(R, L, W, device=dev) if group is not None and H > 1 else None
        self.ks = [torch.zeros(R, L, W, device=dev), torch.zeros(R, L, W, device=dev)]
        self.pin = [c.pinned, torch.zeros_like(c.pinned)]
        self.cur = 0
        self.keep = torch.zeros(R, W, dtype=torch.uint8, device=dev)
        self.perm = torch.zeros(R, W, dtype=torch.int64, device=dev)
        self.kept = torch.zeros(R, dtype=torch.int32, device=dev)
        self.budget = torch.zeros(R, dtype=torch.int32, device=dev)
        self.act_off = torch.zeros(R + 1, dtype=torch.int32, device=dev)
        lib = N.load()
        self.ws_keep = N.workspace(lib.actkv_keep_mask_workspace_bytes(R, W), dev)
        self.ws_compact = N.workspace(lib.actkv_compact_workspace_bytes(R, W), dev)
        self.max_actions = 0
        self.sum_actions = 0
        self._q_dev = self._lse_dev = None        # step_host's device copies of the queries / lse
        self._copy_stream = None
        self.host_inputs_read = None              # event: step_host's last copy out of host memory done
        self._ready = None                        # step_host's streamed mode: copied-groups counter
        self._ready_base = 0
        self._streamed = None                     # None: not tried yet; False: the grouped launches
        self._lse_own = None                      # lse computed here when a step gets none
        self._lse_ws = None
        self._score_ws = None                     # the CTA-pair scoring kernel's lse operand rows
        self._graphs = {}                         # captured steps, see graph_step
        self._graph_pool = None
        self._warm = set()                        # kinds of step run eagerly once (lazy set-up done)

    def load(self, tables, seq_lens, free, protected: int = 0) -> None:
        """Start from a fresh cache state: tables / lengths / free list, first ``protected`` tokens
        pinned, keep scores zero."""
        self.cur = 0
        self.cache.pinned = self.pin[0]
        self.cache.set_state(tables, seq_lens, free, protected)
        for k in self.ks:
            k.zero_()
        self.pin[1].zero_()

    def snapshot(self, with_kv: bool = True) -> dict:
        """Device copies of the whole mutable state: the cache contents (``with_kv``), tables,
        lengths, free stack, pins and keep scores.  Without the contents, ``restore`` puts back
        the allocator and policy state only (every row keeps whatever the last compaction left)."""
        c = self.cache
        return {"kv": c.kv.clone() if with_kv else None, "bt": c.block_table.clone(), "seq": c.seq_used.clone(),
                "free": c.free_list.clone(), "top": c.free_top.clone(), "pin": self.pin[self.cur].clone(),
                "ks": self.ks[self.cur].clone(), "n": c.n_sessions}

    def restore(self, snap: dict) -> None:
        """Device-to-device restore of a snapshot (no host round trip)."""
        c = self.cache
        if snap["kv"] is not None:
            c.kv.copy_(snap["kv"])
        c.block_table.copy_(snap["bt"])
        c.seq_used.copy_(snap["seq"])
        c.free_list.copy_(snap["free"])
        c.free_top.copy_(snap["top"])
        self.cur = 0
        self.pin[0].copy_(snap["pin"])
        self.ks[0].copy_(snap["ks"])
        c.pinned = self.pin[0]
        c.n_sessions = snap["n"]

    @property
    def keep_scores(self) -> torch.Tensor:
        """Current ActionLRFU keep scores [R, L, W] (after the last step's permutation)."""
        return self.ks[self.cur]

    @property
    def pinned(self) -> torch.Tensor:
        return self.pin[self.cur]

    def set_round(self, act_lens: list[int], budgets: list[int]) -> None:
        """Action-region lengths and budgets of the next step (one small host->device copy)."""
        R = self.cache.n_sessions
        assert len(act_lens) == R and len(budgets) == R
        off = [0]
        for a in act_lens:
            off.append(off[-1] + a)
        host = torch.tensor(off + list(budgets), dtype=torch.int32).pin_memory()
        dev = host.to(self.cache.device, non_blocking=True)
        self.act_off[:R + 1].copy_(dev[:R + 1])
        self.budget[:R].copy_(dev[R + 1:])
        self.max_actions = max(act_lens) if act_lens else 0
        self.sum_actions = off[-1]

    def step(self, q: torch.Tensor, lse: torch.Tensor | None = None, on_phase=None) -> None:
        """One eviction step for every session.  q [L, sumA, Hq, D], lse [L, sumA, Hq] fp32; when
        lse is None it is computed here from the cache (``region_lse``).

        ``on_phase(name)``, if given, is called on the host just before each phase's launches
        ("score", "exchange" with a process group, "lrfu", "keep_mask", "compact", "permute") and
        once with None after the last one, e.g. to record CUDA events between them."""
        if self.cache.n_sessions == 0:
            return
        if lse is None:
            lse = self.region_lse(q)
        mark = on_phase or _no_mark
        mark("score")
        self._score_layers(q, lse, 0, self.cache.n_layers)
        self._finish_step(mark)
        mark(None)

    def _graph_key(self, kind, *tensors):
        c = self.cache
        return (kind, self.cur, c.n_sessions, self.max_actions, self.sum_actions, self.path, self.scale) + tuple(
            (t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype) for t in tensors)

    def _replay(self, key, run) -> None:
        """Replay the CUDA graph of ``run`` for ``key``, capturing it first if needed.  A captured
        step bakes in the current keep-score / pin buffers, so there is one graph per buffer
        parity; the host-side flip that ``step`` does is repeated after each replay."""
        if self.group is not None:
            raise RuntimeError("graph replay is not used with a process group (the all-reduce runs eagerly)")
        g = self._graphs.get(key)
        cur0 = self.cur
        if g is None:
            if key[0] not in self._warm:         # first call: load and set up every kernel eagerly
                run()
                self._warm.add(key[0])
                return
            g = torch.cuda.CUDAGraph()
            if self._graph_pool is None:
                self._graph_pool = torch.cuda.graph_pool_handle()
            # thread-local capture: other threads' CUDA calls (e.g. a process group's watchdog)
            # must not invalidate it
            with torch.cuda.graph(g, pool=self._graph_pool, capture_error_mode="thread_local"):
                run()
            self.cur = cur0                      # capture launched nothing: undo the host-side flip
            self.cache.pinned = self.pin[cur0]
            self._graphs[key] = g
        g.replay()
        self.cur = 1 - cur0
        self.cache.pinned = self.pin[self.cur]

    def graph_step(self, q: torch.Tensor, lse: torch.Tensor) -> None:
        """``step`` replayed from a CUDA graph: the same kernels and results, without a launch gap
        between them (config-5-sized steps measured 12% faster).  Every kernel reads the sizes that
        change from step to step (lengths, tables, offsets, budgets) from device memory, so one
        capture serves every later step with the same q / lse buffers (fill them in place), the
        same session count and the same action-region sizes (``set_round`` values may change
        otherwise).  The first call runs eagerly, the second captures; a new key captures again."""
        self._replay(self._graph_key("step", q, lse), lambda: self.step(q, lse))

    def region_lse(self, q: torch.Tensor) -> torch.Tensor:
        """Causal lse [L, sumA, Hq] of every session's action region, on the tensor cores: the LSE
        by-product the reference takes from paged_decode_attention_ref per action token
        (actkv/kernels/lse_attn.py:42-60)."""
        c = self.cache
        R, L = c.n_sessions, c.n_layers
        shape = (L, q.shape[1], q.shape[2])
        if self._lse_own is None or tuple(self._lse_own.shape) != shape:
            self._lse_own = torch.empty(shape, dtype=torch.float32, device=c.device)
            need = region_lse_workspace_bytes(L, q.shape[1], q.shape[2], c.max_tokens)
            self._lse_ws = N.workspace(need, c.device)
        return action_region_lse(q, self.act_off[:R + 1], c.kv, c.block_table[:R], c.seq_used[:R],
                                 scale=self.scale, max_seq=c.max_tokens, out=self._lse_own, workspace=self._lse_ws)

    def step_host(self, q_host: torch.Tensor, lse_host: torch.Tensor, layer_groups: int = 4) -> None:
        """``step`` with the action queries and their lse in pinned host memory.

        The host->device copies go on a side stream one group of layers at a time.  Where the
        CTA-pair scorer applies, one scoring launch takes every group as it lands: after each
        group's copy the copy stream advances a device counter (a stream memory write, no kernel),
        and the scorer's CTA pairs, which take their share of group 0, then of group 1, ..., wait
        on it before reading a group's queries -- the first group is one layer, so little of the
        transfer stays unhidden.  Elsewhere (``layer_groups`` growing groups) each group is scored
        by its own launch once its copy has landed.  The rest of the step follows, replayed from a
        CUDA graph (see ``graph_step``; the first call runs it eagerly).  Nothing synchronises with
        the host.

        Buffer contract: the copies out of ``q_host`` / ``lse_host`` are still in flight when this
        returns.  The caller must not write into those pinned buffers (e.g. refill them for the
        next step) before ``host_inputs_read`` (a CUDA event recorded after the last copy) has
        completed -- ``pipe.host_inputs_read.synchronize()`` or a stream wait on it; otherwise the
        step may read a mix of old and new inputs."""
        c = self.cache
        if c.n_sessions == 0:
            return
        if not (q_host.is_pinned() and lse_host.is_pinned()):
            raise ValueError("step_host needs pinned host tensors (tensor.pin_memory())")
        dev, L = c.device, c.n_layers
        if (self._q_dev is None or self._q_dev.shape != q_host.shape or self._q_dev.dtype != q_host.dtype
                or self._lse_dev.shape != lse_host.shape):
            self._q_dev = torch.empty(q_host.shape, dtype=q_host.dtype, device=dev)
            self._lse_dev = torch.empty(lse_host.shape, dtype=lse_host.dtype, device=dev)
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(dev)
        cur, cs = torch.cuda.current_stream(dev), self._copy_stream
        cs.wait_stream(cur)                      # the previous step's reads of the buffers come first
        if self._streamed is not False and self._step_host_streamed(q_host, lse_host, cur, cs):
            return
        bounds = _growing_groups(L, layer_groups)
        n = len(bounds) - 1
        landed = []
        with torch.cuda.stream(cs):
            for g in range(n):
                l0, l1 = bounds[g], bounds[g + 1]
                self._q_dev[l0:l1].copy_(q_host[l0:l1], non_blocking=True)
                self._lse_dev[l0:l1].copy_(lse_host[l0:l1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(cs)
                landed.append(ev)
        self.host_inputs_read = landed[-1]
        for g in range(n):
            cur.wait_event(landed[g])
            self._score_layers(self._q_dev, self._lse_dev, bounds[g], bounds[g + 1])
        if self.group is None:
            # the rest of the step (its inputs are the pipeline's own buffers) from a CUDA graph
            self._replay(self._graph_key("finish"), self._finish_step)
        else:
            self._finish_step()

    def _step_host_streamed(self, q_host, lse_host, cur, cs) -> bool:
        """step_host in one scoring launch over streamed layer groups; False (nothing enqueued) where
        the stream signal or the CTA-pair path is not available."""
        c = self.cache
        dev, L = c.device, c.n_layers
        if self._ready is None:
            self._ready = torch.zeros(1, dtype=torch.int32, device=dev)
            try:
                stream_signal(self._ready, 0, cs)
            except NotImplementedError:
                self._streamed = False
                return False
        bounds = _stream_groups(L)
        base = self._ready_base
        n = len(bounds) - 1
        # the lse and the first group (one layer), the scoring launch, then the other groups: each
        # group's copy and signal queued natively (a few microseconds each, against tens from
        # Python), and the kernel waits on the device counter, not on the copy stream
        with torch.cuda.stream(cs):
            self._lse_dev.copy_(lse_host, non_blocking=True)
            lse_landed = torch.cuda.Event()
            lse_landed.record(cs)
        gl = (ctypes.c_int32 * (n + 1))(*bounds)
        layer_bytes = q_host[0].numel() * q_host.element_size()
        lib = N.load()

        def copy_groups(g0: int, g1: int) -> None:
            N.check(lib.actkv_stream_copy_groups(self._q_dev.data_ptr(), q_host.data_ptr(), layer_bytes, gl, g0, g1,
                                                 self._ready.data_ptr(), base, cs.cuda_stream),
                    "step_host: stream_copy_groups")

        copy_groups(0, 1)
        self._ready_base = (base + n) & 0xFFFFFFFF
        cur.wait_event(lse_landed)
        try:
            self._score_layers(self._q_dev, self._lse_dev, 0, L, streamed=(self._ready, base, bounds))
            self._streamed = True
            fallback = False
        except NotImplementedError:
            # another scoring path (nothing was launched): score this step once every group has
            # landed, and take the grouped launches from the next step on
            self._streamed = False
            fallback = True
        copy_groups(1, n)
        done = torch.cuda.Event()
        done.record(cs)
        self.host_inputs_read = done
        if fallback:
            cur.wait_event(done)
            self._score_layers(self._q_dev, self._lse_dev, 0, L)
        if self.group is None:
            self._replay(self._graph_key("finish"), self._finish_step)
        else:
            self._finish_step()
        return True

    def _score_layers(self, q, lse, l0: int, l1: int, streamed=None) -> None:
        """1 scores of every head of layers [l0, l1) and every session over the causal action region."""
        c = self.cache
        R = c.n_sessions
        need = score_region_workspace_bytes(c.n_layers, q.shape[1], q.shape[2])
        if self._score_ws is None or self._score_ws.numel() < need:
            self._score_ws = N.workspace(need, c.device)
        action_scores_region(q[l0:l1], lse[l0:l1], self.act_off[:R + 1], c.kv[l0:l1], c.block_table[:R],
                             c.seq_used[:R], self.heads[:R, l0:l1], scale=self.scale, path=self.path,
                             max_actions=self.max_actions, workspace=self._score_ws, streamed=streamed)

    def _finish_step(self, mark=None) -> None:
        """Steps 2-5 of ``step`` (everything after the scores)."""
        mark = mark or _no_mark
        c = self.cache
        R, L, H, W = c.n_sessions, c.n_layers, c.n_kv_heads, c.max_tokens
        dev = c.device
        lib = N.load()
        st = N.stream_ptr(dev)
        status = N.status_word(dev).data_ptr()
        ks, pin = self.ks[self.cur], self.pin[self.cur]
        # 2 ActionLRFU: act = head-reduced scores, ks = decay*ks + act*hit (pinned tokens untouched)
        hs, n_red, how = self.heads, H, (N.REDUCE_MAX if self.cfg.head_reduce == "max" else N.REDUCE_MEAN)
        if self.group is not None:
            mark("exchange")
            part = sharding.local_head_reduce(self.heads[:R], self.cfg.head_reduce,
                                              None if self.part is None else self.part[:R])
            sharding.allreduce_heads(part, self.total_kv_heads, self.cfg.head_reduce, self.group)
            hs, n_red, how = part.view(R, L, 1, W), 1, N.REDUCE_MEAN     # one (already reduced) head
        mark("lrfu")
        N.check(lib.actkv_lrfu_update(
            hs.data_ptr(), None, hs.stride(0), hs.stride(1), hs.stride(2), n_red, how,
            ks.data_ptr(), ks.stride(0), ks.stride(1), self.act.data_ptr(), self.act.stride(0),
            self.act.stride(1), pin.data_ptr(), pin.stride(0), 0, c.seq_used.data_ptr(),
            None, R, L, W, float(self.cfg.decay), float(self.cfg.top_p),
            status, st), "lrfu_update")
        # 3 keep mask from the layer-mean of the keep scores (dim -2 of [L, S] is the layer dim)
        mark("keep_mask")
        N.check(lib.actkv_keep_mask(
            ks.data_ptr(), None, ks.stride(0), 0, ks.stride(1), 1, L, N.REDUCE_MEAN,
            pin.data_ptr(), pin.stride(0), 0, c.seq_used.data_ptr(), self.budget.data_ptr(), 1,
            self.keep.data_ptr(), self.keep.stride(0), None, R, W, self.ws_keep.data_ptr(), self.ws_keep.numel(),
            status, st), "keep_mask")
        # 4 compaction: plan, copies over all planes, table / free stack / length update
        mark("compact")
        self.compact_with(self.keep)
        # 5 keep scores and pins follow their tokens
        mark("permute")
        self._permute_state()

    def _permute_state(self) -> None:
        """Keep scores and pins follow their tokens (perm of the last compaction), into the other
        buffer, which becomes the current one."""
        c = self.cache
        R, L, W = c.n_sessions, c.n_layers, c.max_tokens
        dev = c.device
        ks, pin = self.ks[self.cur], self.pin[self.cur]
        nxt = 1 - self.cur
        N.check(N.load().actkv_permute_tokens(
            ks.data_ptr(), self.ks[nxt].data_ptr(), ks.stride(0), ks.stride(1), L,
            pin.data_ptr(), self.pin[nxt].data_ptr(), pin.stride(0), self.perm.data_ptr(), self.perm.stride(0),
            c.seq_used.data_ptr(), R, W, N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "permute")
        self.cur = nxt
        c.pinned = self.pin[nxt]

    def evict_with_mask(self, keep: torch.Tensor) -> None:
        """Evict every session by an explicit keep mask [R, W] instead of the ActionLRFU one
        (PagedKVCache.compact with a caller's mask, actkv/paged.py:125-139): compaction, then the
        keep scores and pins follow their tokens as after ``step``."""
        self.compact_with(keep)
        self._permute_state()

    def compact_with(self, keep: torch.Tensor) -> None:
        """Compaction of every session by an explicit keep mask [R, W] (uint8/bool, 1 = keep)."""
        c = self.cache
        R = c.n_sessions
        dev = c.device
        keep = keep.view(torch.uint8) if keep.dtype == torch.bool else keep
        plane, slot, row, n_slots = c.flat_planes()
        N.check(N.load().actkv_compact(
            c.kv.data_ptr(), 2 * c.n_layers, plane, slot, row, n_slots, keep.data_ptr(), keep.stride(0),
            c.seq_used.data_ptr(), c.block_table.data_ptr(), c.block_table.stride(0), c.max_blocks, c.block_size,
            c.free_list.data_ptr(), c.free_top.data_ptr(), c.num_blocks, self.perm.data_ptr(), self.perm.stride(0),
            self.kept.data_ptr(), R, c.max_tokens, self.ws_compact.data_ptr(), self.ws_compact.numel(),
            N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "compact")
