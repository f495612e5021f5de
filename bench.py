#!/usr/bin/env python
"""Benchmark of the eviction hot path: one eviction step = score every layer over the causal action
region -> ActionLRFU keep-score update -> keep mask -> in-place paged compaction -> state
permutation.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Headline (the JSON line's value): the BASELINE config-2 session (Qwen3-8B shape: 36 layers, 32/8
heads, head_dim 128, bf16 paged cache, block 16, 32768 tokens, 128-token action region, budget 20%
+ 4 sinks, ActionLRFU decay 0.9 / top_p 0.9), one session per GPU (N>1: every rank evicts its own
session, no collective, weak scaling; step time = max over ranks).  The step is checked once,
outside the timed region, against a torch fp32 restatement (``parity``).

Two more records ride on the same line, both measured at every N:
  config3_batch  BASELINE config 3: all 64 mixed sessions (S in [4096, 65536], A in [32, 256],
                 10% budget) LPT-assigned over the N ranks, no collective; a rank whose sessions do
                 not fit in HBM evicts them in resident waves (each wave built untimed); value =
                 algorithmic bytes of the whole batch / the slowest rank's summed step times
  config4        BASELINE config 4: one 131072-token, 80-layer session with 8 KV heads split over
                 the N ranks (8 / N heads each; strong scaling), the per-token head sum
                 all-reduced over NCCL before ActionLRFU; the all-reduce is timed apart

Inputs are synthetic and seeded (no dataset exists for this path).  Caches are larger than L2;
the headline restores its 4.8 GB cache from a device snapshot between timed steps (this also
flushes L2); the records restore the allocator and policy state (tables, lengths, free stack,
pins, keep scores) between steps and leave the rows where the last compaction put them.

One JSON line on rank 0: value = algorithmic HBM bytes of the step / step time (GB/s, whole job),
ms_per_step (evict latency), per-phase times, the roofline of the dominant kernel (the tcgen05
scoring kernel), the end-to-end number through the public API with host buffers, and the CPU
baseline (the CPU oracle of the reference's torch path on the host cores, one full layer).
``--impl reference`` times that CPU implementation alone on the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "evict() step throughput, score+LRFU+mask+compact (algorithmic HBM GB/s)"
UNIT = "GB/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# BASELINE config 2
CFG2 = dict(L=36, HQ=32, HKV=8, D=128, BS=16, S=32768, A=128, P=4, BUDGET=int(0.2 * 32768), DECAY=0.9,
            TOP_P=0.9)
# 64 sessions of the config-2 model, S ~ U[4096, 65536] rounded to 16,
# A ~ U[32, 256], budget 10% of S + 4 sinks, assigned to ranks by LPT on S * max(1, A / 63)
CFG3 = dict(L=36, HQ=32, HKV=8, D=128, BS=16, SESSIONS=64, S_MIN=4096, S_MAX=65536, A_MIN=32, A_MAX=256,
            P=4, BUDGET_FRAC=0.1, DECAY=0.9, TOP_P=0.9)
# one 131072-token session, 80 layers, 64 query / 8 KV heads, the KV heads split
# over the ranks, 256 action tokens, per-token scores all-reduced before a 5% keep mask
CFG4 = dict(L=80, HQ=64, HKV=8, D=128, BS=16, S=131072, A=256, P=4, BUDGET=int(0.05 * 131072), DECAY=0.9, TOP_P=0.9)
# BASELINE config 5 (agent loop): 2 sessions per GPU, 50 rounds of 1024 + 64 appended tokens (the
# 64 action tokens last), budget 10% of the full trace, adversarial masks every 5th round
CFG5 = dict(L=36, HQ=32, HKV=8, D=128, BS=16, NEW=1024, A=64, ROUNDS=50, SESSIONS=2, P=4, DECAY=0.9, TOP_P=0.9,
            BUDGET=int(0.1 * 50 * (1024 + 64)), ADV_EVERY=5)
LAYERS_CONFIG2 = CFG2["L"]


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--path", choices=["auto", "simt", "tcgen05", "pair"], default="auto")
    ap.add_argument("--layers", type=int, default=CFG2["L"], help="smaller headline cases for profiling only")
    ap.add_argument("--seq", type=int, default=CFG2["S"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-aux", action="store_true", help="skip the region-lse and decode-attention lines")
    ap.add_argument("--records", default="config3,config4,dropin",
                    help="comma list of extra records on the headline line (config3, config4, dropin; '' for none)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workload", choices=["config2", "config3", "config4", "config5"], default="config2",
                    help="config2: the headline line with its records (default); config3 / config4: that "
                         "record alone as the line; config5: the agent loop")
    ap.add_argument("--rounds", type=int, default=CFG5["ROUNDS"], help="config5 rounds")
    ap.add_argument("--c4-layers", type=int, default=CFG4["L"], help="smaller config-4 cases for profiling only")
    return ap.parse_args(argv)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


# --------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of this GPU, sampled every ~2 ms by NVML
    from a thread while ``active`` (the timed regions); nvidia-smi every 100 ms if NVML is missing."""

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str):
        self.index = index
        self.samples = []           # (sm MHz, max sm MHz, power W, reason names)
        self.active = False
        self._stop = False
        self._thread = None
        self._proc = None
        self._file = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                h = pynvml.nvmlDeviceGetHandleByPciBusId(self.index)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(int(self.index) if self.index.isdigit() else 0)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self._stop:
                    if self.active:
                        try:
                            sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                            pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                            bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                            self.samples.append((sm, mx, pw, [n for b, n in self.REASONS.items() if bits & b]))
                        except Exception:
                            pass
                    time.sleep(0.002)

            self._thread = threading.Thread(target=poll, daemon=True)
            self._thread.start()
            self.source = "nvml every 2 ms"
        except Exception:
            self._start_smi()
        return self

    def _start_smi(self):
        self.source = "nvidia-smi every 100 ms"
        try:
            self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self._proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                           "--format=csv,noheader,nounits", "-lms", "100"],
                                          stdout=self._file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self._proc = None

    def stop(self):
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=5)
        elif self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            self._file.flush()
            self._file.seek(0)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in (l.strip().split(", ") for l in self._file.read().splitlines() if l.strip()):
                if len(r) >= 9 and r[1].replace(".", "").isdigit():
                    self.samples.append((float(r[1]), float(r[2]), float(r[3]) if r[3].replace(".", "").isdigit()
                                         else 0.0, [n for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"]))
            os.unlink(self._file.name)
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"], "samples": 0}
        sm = [x[0] for x in self.samples]
        reasons = sorted({n for x in self.samples for n in x[3]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(x[1] for x in self.samples) if sm else None,
                "sm_mhz_min": min(sm) if sm else None,
                "power_w_median": round(statistics.median(x[2] for x in self.samples), 1) if sm else None,
                "reasons": reasons, "samples": len(sm), "source": self.source}


# --------------------------------------------------------------------------------------- workloads
# The BASELINE workloads built on the device.  The full-size parity tests (tests/test_gpu_headline.py)
# build the same ones through these functions.

def chunked_causal_lse(torch, k, q, A, scale, chunk=16384):
    """Exact causal lse [A, Hq] of the last A of n tokens for one layer: k [n, Hkv, D], q [A, Hq, D],
    streamed over key chunks with a running logsumexp (untimed set-up, fp32 without TF32)."""
    n, hkv, d = k.shape
    hq = q.shape[1]
    qq = q.float().view(A, hkv, hq // hkv, d)
    see = n - A + torch.arange(A, device=k.device)
    acc = torch.full((A, hkv, hq // hkv), float("-inf"), device=k.device)
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for c0 in range(0, n, chunk):
            kk = k[c0:c0 + chunk].float()
            logits = torch.einsum("ahgd,nhd->ahgn", qq, kk) * scale
            pos = c0 + torch.arange(kk.shape[0], device=k.device)
            logits.masked_fill_(pos[None, None, None, :] > see[:, None, None, None], float("-inf"))
            acc = torch.logaddexp(acc, torch.logsumexp(logits, -1))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    return acc.reshape(A, hq)


def build_config2(dev, seed: int, L: int, S: int):
    """Config-2 session on the device: K/V ~ N(0,1) * c (c per layer / head / channel in U(0.5,2)),
    scattered physical blocks, 128 N(0,1) action queries per layer, exact causal lse (untimed)."""
    import torch

    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    c = CFG2
    HQ, HKV, D, BS, A = c["HQ"], c["HKV"], c["D"], c["BS"], c["A"]
    nb = math.ceil(S / BS)
    gen = torch.Generator(device=dev).manual_seed(1000 + seed)
    cache = DevicePagedCache(nb, BS, HKV, D, L, 1, S, dtype=torch.bfloat16, device=dev)
    for l in range(L):
        scale = torch.rand(1, 1, 1, HKV, D, generator=gen, device=dev) * 1.5 + 0.5
        for kv in range(2):
            x = torch.randn(nb, BS, HKV, D, generator=gen, device=dev)
            cache.kv[l, kv].copy_((x * scale[0]).to(torch.bfloat16))
    free = torch.randperm(nb, generator=torch.Generator().manual_seed(seed)).tolist()
    table = [free.pop() for _ in range(nb)]
    q = torch.randn(L, A, HQ, D, generator=gen, device=dev).to(torch.bfloat16)
    bt = torch.tensor(table, dtype=torch.long, device=dev)
    pos = torch.arange(S, device=dev)
    slots = bt[pos // BS] * BS + pos % BS
    lse = torch.empty(L, A, HQ, device=dev)
    for l in range(L):
        lse[l] = chunked_causal_lse(torch, cache.kv[l, 0].view(nb * BS, HKV, D)[slots], q[l], A, D ** -0.5)
    pipe = EvictionPipeline(cache, EvictionConfig(decay=c["DECAY"], top_p=c["TOP_P"]))
    pipe.load([table], [S], free, c["P"])
    pipe.set_round([A], [c["BUDGET"]])
    torch.cuda.synchronize(dev)
    return cache, pipe, q.contiguous(), lse.contiguous()


def config3_sessions(seed: int = 0):
    """The 64 (S_i, A_i) of config 3 (the same for every rank count)."""
    import numpy as np
    c = CFG3
    rng = np.random.default_rng(3000 + seed)
    S = (rng.integers(c["S_MIN"], c["S_MAX"] + 1, c["SESSIONS"]) // c["BS"]) * c["BS"]
    A = rng.integers(c["A_MIN"], c["A_MAX"] + 1, c["SESSIONS"])
    return [(int(s), int(a)) for s, a in zip(S, A)]


def lpt_cost(S: int, A: int, G: int = CFG3["HQ"] // CFG3["HKV"]) -> float:
    """Relative step time of one config-3 session: its 256-token tiles times (a per-tile cost, the
    K stream and the tail, + the tile's MMA columns / 256 over its query chunks of 256 / G tokens,
    each padded to 32 columns).  The per-tile term, 2.03 column-chunks, is the ratio of the two
    coefficients fitted to the measured per-rank times at N = 2 and 4 (0.00584 ms per tile, 0.00288
    ms per 256 columns of a tile), which also reproduce the N = 1 batch time within 0.3%."""
    tiles = math.ceil(S / 256)
    cols, a, qpc = 0, A, 256 // G
    while a > 0:
        cols += (min(256, a * G) + 31) // 32 * 32
        a -= qpc
    return tiles * (2.03 + cols / 256)


def lpt_assign(sessions, n_ranks: int):
    """Longest-processing-time assignment of sessions to ranks by lpt_cost.  Returns each rank's
    session indices, ascending."""
    w = [lpt_cost(s, a) for s, a in sessions]
    load = [0.0] * n_ranks
    out = [[] for _ in range(n_ranks)]
    for i in sorted(range(len(sessions)), key=lambda i: (-w[i], i)):
        k = min(range(n_ranks), key=lambda k: (load[k], k))
        out[k].append(i)
        load[k] += w[i]
    return [sorted(x) for x in out]


def build_config3(dev, items, seed: int = 0, pool_seed: int = 0):
    """Sessions ``items`` = [(index, S, A)] of config 3 on one GPU: one shuffled block pool, each
    session's K/V (N(0,1) times per-layer channel scales in U(0.5, 2)) and N(0,1) queries drawn
    from a generator seeded by its index (so a session's data does not depend on the rank count),
    exact causal lse.  Returns (cache, pipe, q, lse, budgets)."""
    import torch

    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    c = CFG3
    L, HQ, HKV, D, BS = c["L"], c["HQ"], c["HKV"], c["D"], c["BS"]
    R = len(items)
    W = max(s for _, s, _ in items)
    nbs = [math.ceil(s / BS) for _, s, _ in items]
    NB = sum(nbs)
    cache = DevicePagedCache(NB, BS, HKV, D, L, R, W, dtype=torch.bfloat16, device=dev)
    flat = cache.kv.view(L, 2, NB * BS, HKV, D)
    free = torch.randperm(NB, generator=torch.Generator().manual_seed(7919 * pool_seed + 1)).tolist()
    tables = [[free.pop() for _ in range(nb)] for nb in nbs]
    qs, lses = [], []
    for (idx, S, A), table in zip(items, tables):
        gen = torch.Generator(device=dev).manual_seed(30000 + 1000 * seed + idx)
        bt = torch.tensor(table, dtype=torch.long, device=dev)
        pos = torch.arange(S, device=dev)
        slots = bt[pos // BS] * BS + pos % BS
        q = torch.randn(L, A, HQ, D, generator=gen, device=dev).to(torch.bfloat16)
        lse = torch.empty(L, A, HQ, device=dev)
        for l in range(L):
            scale = torch.rand(HKV, D, generator=gen, device=dev) * 1.5 + 0.5
            for kv in range(2):
                flat[l, kv, slots] = (torch.randn(S, HKV, D, generator=gen, device=dev) * scale).to(torch.bfloat16)
            lse[l] = chunked_causal_lse(torch, flat[l, 0, slots], q[l], A, D ** -0.5)
        qs.append(q)
        lses.append(lse)
    q = torch.cat(qs, 1).contiguous()
    lse = torch.cat(lses, 1).contiguous()
    budgets = [int(c["BUDGET_FRAC"] * s) for _, s, _ in items]
    pipe = EvictionPipeline(cache, EvictionConfig(decay=c["DECAY"], top_p=c["TOP_P"]))
    pipe.load(tables, [s for _, s, _ in items], free, c["P"])
    pipe.set_round([a for _, _, a in items], budgets)
    torch.cuda.synchronize(dev)
    return cache, pipe, q, lse, budgets


def build_config4(dev, seed: int, lo: int, hi: int, group=None, L: int | None = None, S: int | None = None):
    """KV heads [lo, hi) of the config-4 session on this GPU: its paged K/V [L, 2, NB, BS, hi-lo, D]
    (each head's data drawn from a generator seeded by the head, so it does not depend on the rank
    count), the replicated block table (one permutation on every rank), the matching query heads
    and their exact causal lse.  ``group``: the process group of a head-sharded run (None: the
    heads are all local and reduced inside ActionLRFU's kernel)."""
    import torch

    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    c = CFG4
    L = c["L"] if L is None else L
    S = c["S"] if S is None else S
    HKV, D, BS, A, P = c["HKV"], c["D"], c["BS"], c["A"], c["P"]
    G = c["HQ"] // HKV
    h = hi - lo
    nb = S // BS
    cache = DevicePagedCache(nb, BS, h, D, L, 1, S, dtype=torch.bfloat16, device=dev)
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.tensor(table, dtype=torch.long, device=dev)
    pos = torch.arange(S, device=dev)
    slots = bt[pos // BS] * BS + pos % BS
    q = torch.empty(L, A, G * h, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(L, A, G * h, device=dev)
    for j, head in enumerate(range(lo, hi)):
        gen = torch.Generator(device=dev).manual_seed(4000 + 100 * seed + head)
        for l in range(L):
            for kv in range(2):
                cache.kv[l, kv, :, :, j].copy_(torch.randn(nb, BS, D, generator=gen, device=dev).to(torch.bfloat16))
        q[:, :, j * G:(j + 1) * G] = torch.randn(L, A, G, D, generator=gen, device=dev).to(torch.bfloat16)
        for l in range(L):
            k = cache.kv[l, 0, :, :, j].reshape(nb * BS, 1, D)[slots]
            lse[l, :, j * G:(j + 1) * G] = chunked_causal_lse(torch, k, q[l, :, j * G:(j + 1) * G], A, D ** -0.5)
    pipe = EvictionPipeline(cache, EvictionConfig(decay=c["DECAY"], top_p=c["TOP_P"]), group=group,
                            total_kv_heads=HKV if group is not None else None)
    pipe.load([table], [S], [], P)
    pipe.set_round([A], [c["BUDGET"]])
    torch.cuda.synchronize(dev)
    return cache, pipe, q, lse


def committed_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` from the ncu summary committed in profiles/traffic.txt."""
    p = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        f = line.split()
        if len(f) == 3 and not line.startswith("#") and f[0] == kernel and f[1] == workload:
            return int(f[2])
    return None


def gpu_smi_id(torch, dev, local):
    """nvidia-smi --id for this device: its PCI bus id (independent of CUDA_VISIBLE_DEVICES)."""
    p = torch.cuda.get_device_properties(dev)
    if all(hasattr(p, a) for a in ("pci_domain_id", "pci_bus_id", "pci_device_id")):
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    return str(local)



def step_bytes(L, S, A, n_moved, hq, hkv, d=128):
    """Bytes one session's step must touch at minimum: K once per layer, its queries + lse, keep
    scores / action means (read + write), and each moved row read and written in all 2L planes."""
    parts = {"k_read": L * S * hkv * d * 2, "q_lse": L * A * hq * (d * 2 + 4), "state": 4 * L * S * 4,
             "moves": 2 * n_moved * 2 * L * hkv * d * 2}
    return sum(parts.values()), parts


def algorithmic_bytes(L, S, n_moved, c=CFG2):
    return step_bytes(L, S, c["A"], n_moved, c["HQ"], c["HKV"], c["D"])


def score_flops(L, S, c=CFG2):
    return 2 * L * c["HQ"] * c["A"] * c["D"] * S


# --------------------------------------------------------------------------------------- timing
class PhaseTimer:
    """The ``on_phase`` hook of EvictionPipeline.step: a CUDA event on the launching stream before
    each phase and after the last one."""

    def __init__(self, torch):
        self.torch = torch
        self.pool = []
        self.names = []

    def start(self):
        self.names = []

    def __call__(self, name):
        i = len(self.names)
        if i == len(self.pool):
            self.pool.append(self.torch.cuda.Event(enable_timing=True))
        self.pool[i].record()
        self.names.append(name)

    def times(self) -> dict:
        return {self.names[i]: self.pool[i].elapsed_time(self.pool[i + 1]) for i in range(len(self.names) - 1)}


def timed_steps(torch, pipe, q, lse, snap, n, dev, clocks=None):
    """n eviction steps, each from the state ``snap`` (restored untimed), timed phase by phase with
    CUDA events; returns the list of {phase: ms}."""
    timer = PhaseTimer(torch)
    out = []
    for _ in range(n):
        pipe.restore(snap)
        torch.cuda.synchronize(dev)
        if clocks is not None:
            clocks.active = True
        timer.start()
        pipe.step(q, lse, on_phase=timer)
        torch.cuda.synchronize(dev)
        if clocks is not None:
            clocks.active = False
        out.append(timer.times())
    return out


def med(xs):
    return statistics.median(xs) if xs else 0.0


def phase_medians(runs):
    names = list(runs[0]) if runs else []
    return {k: round(med([r[k] for r in runs]), 4) for k in names}


def phase_spread(runs):
    """[min, median, max] ms of every phase over the timed steps."""
    names = list(runs[0]) if runs else []
    return {k: [round(min(r[k] for r in runs), 4), round(med([r[k] for r in runs]), 4),
                round(max(r[k] for r in runs), 4)] for k in names}


def moved_rows(perm, n, bs):
    """Rows the compaction moved: new position j holds old position perm[j]; it stayed in place
    when perm[j] == start + j (start = first logical slot of the kept window)."""
    kept = len(perm)
    start = (math.ceil(n / bs) - math.ceil(kept / bs)) * bs
    return sum(1 for j, p in enumerate(perm) if p != start + j)


# lse_split, score_pair, lrfu_select (with the head mean), keep_reduce, keep_select, count_chunks, plan_chunks,
# copy_pairs, finish, permute
LAUNCHES_PER_STEP = 10


def run_headline(args, dev, world, rank, clocks, peaks):
    """The config-2 step of this rank's session: warm-up, one parity check, eager phase timing, then
    the CUDA-graph step (the headline ms), region lse, decode attention and the end-to-end line."""
    import torch
    import torch.distributed as dist

    from actkv_open_b200 import _native as N
    from actkv_open_b200 import check
    L, S = args.layers, args.seq
    cache, pipe, q, lse = build_config2(dev, args.seed + rank, L, S)
    pipe.path = args.path
    snap = pipe.snapshot()
    timed_steps(torch, pipe, q, lse, snap, args.warmup, dev)
    kept = int(pipe.kept[0].item())
    n_moved = moved_rows(pipe.perm[0, :kept].cpu().tolist(), S, CFG2["BS"])
    parity = None
    if not args.no_parity:
        # the step that is timed, once, against the torch fp32 restatement (outside the timing)
        pipe.restore(snap)
        before = check.capture_state(pipe)
        pipe.step(q, lse)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        try:
            parity = check.check_step(pipe, before, q, lse)
        except AssertionError as e:
            parity = {"ok": False, "error": str(e)[:400]}
        parity["check_s"] = round(time.perf_counter() - t0, 2)
        parity["against"] = ("actkv_open_b200.check: torch fp32 scores (rtol 1e-3), nucleus / top-k masks "
                             "(near-ties only), Algorithm-4 plan, tables, free stack, perm and every cache "
                             "byte bit-exact")
        del before
        torch.cuda.empty_cache()
    status = N.read_device_status(dev)
    if world > 1:
        dist.barrier()
    runs = timed_steps(torch, pipe, q, lse, snap, args.steps, dev, clocks)
    eager_ms = med([sum(r.values()) for r in runs])
    # the step as a serving loop runs it: replayed from a CUDA graph (EvictionPipeline.graph_step,
    # the same eight kernels without launch gaps); the first calls set up and capture it
    for _ in range(max(2, args.warmup)):
        pipe.restore(snap)
        pipe.graph_step(q, lse)
    torch.cuda.synchronize(dev)
    graph_ms = []
    if world > 1:
        dist.barrier()
    for _ in range(args.steps):
        pipe.restore(snap)
        torch.cuda.synchronize(dev)
        clocks.active = True
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        pipe.graph_step(q, lse)
        e.record()
        torch.cuda.synchronize(dev)
        clocks.active = False
        graph_ms.append(s.elapsed_time(e))
    status |= N.read_device_status(dev)
    ms = med(graph_ms)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
        dist.barrier()
    nbytes, parts = algorithmic_bytes(L, S, n_moved)
    phases = phase_medians(runs)
    flops = score_flops(L, S)
    ach = flops / (phases["score"] * 1e-3) / 1e12
    clocks.active = True
    e2e = None if args.no_e2e else e2e_measure(torch, pipe, snap, q, lse, args, dev, world, nbytes)
    clocks.active = False
    aux = {}
    if not args.no_aux:
        aux["region_lse"] = region_lse_measure(torch, pipe, snap, q, lse, args, dev)
        aux["decode_attention"] = decode_measure(torch, pipe, q, args, dev)
        aux["kv_gather"] = kv_gather_measure(torch, pipe, dev)
        one = aux["kv_gather"]["one_head_per_cta_gbs"]
        aux["decode_attention"]["frac_of_one_head_gather_rate"] = round(aux["decode_attention"]["achieved_gbs"] / one, 4)
    status |= N.read_device_status(dev)
    res = {"value": world * nbytes / (ms * 1e-3) / 1e9, "ms": ms, "eager_ms": eager_ms, "phases": phases,
           "phase_spread": phase_spread(runs),
           "kept": kept, "n_moved": n_moved, "nbytes": nbytes, "parts": parts, "flops": flops, "ach": ach,
           "e2e": e2e, "parity": parity, "status": status, "graph_ms_min_median_max":
           [round(min(graph_ms), 4), round(ms, 4), round(max(graph_ms), 4)], **aux}
    del cache, pipe, q, lse, snap
    torch.cuda.empty_cache()
    return res


def config3_batch(args, dev, world, rank, clocks, peaks):
    """BASELINE config 3 over the N ranks: the 64 sessions LPT-assigned to ranks, each rank's share
    evicted in resident waves (as many sessions as fit in ~55% of the free HBM per wave, built
    untimed), every wave timed over ``--steps`` steps from its restored allocator state.  The
    rank's time is the sum of its waves' median step times; the job's is the max over ranks."""
    import torch
    import torch.distributed as dist

    from actkv_open_b200 import _native as N
    c = CFG3
    L, HQ, HKV, D, BS = c["L"], c["HQ"], c["HKV"], c["D"], c["BS"]
    sessions = config3_sessions(args.seed)
    mine = lpt_assign(sessions, world)[rank]
    cap = int(0.55 * torch.cuda.mem_get_info(dev)[0])
    row = L * 2 * HKV * D * 2                                     # cache bytes per token slot
    waves, cur, used = [], [], 0
    for i in sorted(mine, key=lambda i: -sessions[i][0]):
        b = math.ceil(sessions[i][0] / BS) * BS * row
        if cur and used + b > cap:
            waves.append(cur)
            cur, used = [], 0
        cur.append(i)
        used += b
    if cur:
        waves.append(cur)
    rank_ms = score_ms = 0.0
    nbytes = flops = 0
    roof_ms = 0.0                     # the rank's serial roofline: per session, scoring then copies
    wave_info = []
    status = 0
    t_build = 0.0
    for w, wave in enumerate(waves):
        items = [(i, *sessions[i]) for i in sorted(wave)]
        t0 = time.perf_counter()
        cache, pipe, q, lse, budgets = build_config3(dev, items, args.seed, pool_seed=1000 * rank + w)
        t_build += time.perf_counter() - t0
        meta = pipe.snapshot(with_kv=False)
        timed_steps(torch, pipe, q, lse, meta, max(1, min(args.warmup, 2)), dev)
        kept = pipe.kept[:len(items)].tolist()
        for r, (i, S, A) in enumerate(items):
            m = moved_rows(pipe.perm[r, :kept[r]].cpu().tolist(), S, BS)
            tot, parts = step_bytes(L, S, A, m, HQ, HKV, D)
            nbytes += tot
            fl = 2 * L * HQ * A * D * S
            flops += fl
            # small A (A*G <= ~250 columns) makes a session's scoring HBM-bound, large A tensor-bound
            roof_ms += 1e3 * (max((tot - parts["moves"]) / (peaks["hbm_gbs"] * 1e9), fl / (peaks["bf16_tflops"] * 1e12))
                              + parts["moves"] / (peaks["hbm_gbs"] * 1e9))
        runs = timed_steps(torch, pipe, q, lse, meta, max(1, args.steps), dev, clocks)
        ms = med([sum(r.values()) for r in runs])
        sc = med([r["score"] for r in runs])
        rank_ms += ms
        score_ms += sc
        status |= N.read_device_status(dev)
        wave_info.append({"sessions": len(items), "tokens": sum(s for _, s, _ in items), "ms": round(ms, 4),
                          "score_ms": round(sc, 4), "phases_ms": phase_medians(runs)})
        del cache, pipe, q, lse, meta
        torch.cuda.empty_cache()
    per_rank = [rank_ms]
    if world > 1:
        t = torch.tensor([rank_ms, score_ms, float(nbytes), float(flops), float(len(waves)), roof_ms], device=dev,
                         dtype=torch.float64)
        allt = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        per_rank = [float(x[0]) for x in allt]
        total_bytes = sum(float(x[2]) for x in allt)
        total_flops = sum(float(x[3]) for x in allt)
        score_max = max(float(x[1]) for x in allt)
        n_waves = [int(x[4]) for x in allt]
        roof_max = max(float(x[5]) for x in allt)
    else:
        total_bytes, total_flops, score_max, n_waves = float(nbytes), float(flops), score_ms, [len(waves)]
        roof_max = roof_ms
    job_ms = max(per_rank)
    ach = total_flops / world / (score_max * 1e-3) / 1e12 if score_max else 0.0
    return {"workload": "BASELINE config 3: 64 sessions (S in [4096, 65536], A in [32, 256], 10% budget + 4 "
                        "sinks), LPT over the ranks on lpt_cost (tiles x (2.03 + MMA columns / 256)), no collective",
            "value": round(total_bytes / (job_ms * 1e-3) / 1e9, 2), "unit": UNIT, "ms_per_batch_step": round(job_ms, 4),
            "scaling": "strong (the 64-session batch is fixed; it is split over the N ranks)",
            "per_rank_ms": [round(x, 4) for x in per_rank],
            "imbalance": round(job_ms / (sum(per_rank) / len(per_rank)), 4) if sum(per_rank) else None,
            "waves_per_rank": n_waves, "algorithmic_bytes": total_bytes, "score_flops": total_flops,
            "score_tflops_per_gpu": round(ach, 1), "score_frac_of_bf16_peak": round(ach / peaks["bf16_tflops"], 4),
            "serial_roofline_ms": round(roof_max, 4),
            "frac_of_serial_roofline": round(roof_max / job_ms, 4) if job_ms else None,
            "serial_roofline": "per session: max(its bytes other than the copies / measured HBM, its QK^T flops / "
                               "measured bf16 burst peak) + its moved rows / measured HBM; summed over the rank's "
                               "sessions, max over ranks",
            "rank0_waves": wave_info, "rank0_build_s": round(t_build, 1),
            "timing": "each wave: allocator / policy state restored untimed before every step, rows left where the "
                      "last compaction put them; the wave's caches are built untimed; rank time = sum over its "
                      "waves of the median step; job time = max over ranks",
            "limiter": "max-rank load imbalance (per_rank_ms) at N>1; HBM capacity (waves) at N=1",
            "device_status": status}


def config4_record(args, dev, world, rank, clocks, peaks):
    """BASELINE config 4 with its 8 KV heads split over the N ranks (N in 1, 2, 4, 8): scoring of the
    local heads, all_reduce(SUM) of the per-token [1, 80, 131072] fp32 head sums over NCCL and the
    division by 8 (the 'exchange' phase), then identical ActionLRFU, keep mask (5% + 4 sinks) and
    local compaction on every rank.  N=1 holds all 8 heads and reduces them inside ActionLRFU's
    kernel (no exchange)."""
    import torch
    import torch.distributed as dist

    from actkv_open_b200 import _native as N
    from actkv_open_b200 import sharding
    c = CFG4
    L, HKV, D, S, A, BS = args.c4_layers, c["HKV"], c["D"], c["S"], c["A"], c["BS"]
    G = c["HQ"] // HKV
    if HKV % world:
        return {"skipped": f"{HKV} KV heads do not split evenly over {world} ranks"}
    lo, hi = sharding.head_shard(HKV, world, rank)
    group = dist.group.WORLD if world > 1 else None
    cache, pipe, q, lse = build_config4(dev, args.seed, lo, hi, group, L=L)
    meta = pipe.snapshot(with_kv=False)
    timed_steps(torch, pipe, q, lse, meta, max(1, min(args.warmup, 2)), dev)
    kept = int(pipe.kept[0].item())
    n_moved = moved_rows(pipe.perm[0, :kept].cpu().tolist(), S, BS)
    if world > 1:
        dist.barrier()
    runs = timed_steps(torch, pipe, q, lse, meta, max(1, args.steps), dev, clocks)
    status = N.read_device_status(dev)
    ms = med([sum(r.values()) for r in runs])
    ex = med([r.get("exchange", 0.0) for r in runs])
    sc = med([r["score"] for r in runs])
    phases = phase_medians(runs)
    del cache, pipe, q, lse, meta
    torch.cuda.empty_cache()
    act_bytes = L * S * 4
    ar = 0.0
    if world > 1:
        # the all_reduce alone, on a buffer of the head sums' size, every rank in step (after a
        # barrier): the exchange phase above also holds the wait for the slowest rank's scoring
        buf = torch.ones(L * S, device=dev)
        for _ in range(3):
            dist.all_reduce(buf)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_ar = 10
        e0.record()
        for _ in range(n_ar):
            dist.all_reduce(buf)
        e1.record()
        torch.cuda.synchronize()
        ar = e0.elapsed_time(e1) / n_ar
        del buf
        t = torch.tensor([ms, ex, sc, ar], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ex, sc, ar = (float(x) for x in t)
    k_read = L * S * HKV * D * 2
    nbytes = k_read + L * A * G * HKV * (D * 2 + 4) + 4 * act_bytes + 2 * n_moved * 2 * L * HKV * D * 2
    flops = 2 * L * G * HKV * A * D * S
    tf = flops / world / (sc * 1e-3) / 1e12
    return {"workload": f"BASELINE config 4: one 131072-token, {L}-layer session, 64/8 heads, A=256, 5% budget; "
                        f"{hi - lo} KV head(s) per rank", "value": round(nbytes / (ms * 1e-3) / 1e9, 2), "unit": UNIT,
            "ms_per_step": round(ms, 4), "scaling": "strong (one session; its heads are split over the N ranks)",
            "kv_heads_per_rank": hi - lo, "score_ms_max_rank": round(sc, 4),
            "exchange_ms_max_rank": round(ex, 4), "exchange_share": round(ex / ms, 4) if ms else None,
            "allreduce_bytes": act_bytes if world > 1 else 0,
            "allreduce_alone_ms": round(ar, 4) if world > 1 else None,
            "allreduce_alone_algbw_gbs": round(act_bytes / (ar * 1e-3) / 1e9, 1) if ar else None,
            "allreduce_alone_busbw_gbs": round(act_bytes * 2 * (world - 1) / world / (ar * 1e-3) / 1e9, 1)
            if ar else None,
            "exchange_wait_ms": round(max(0.0, ex - ar), 4) if world > 1 else None,
            "exchange_note": "exchange_ms_max_rank is the phase in the step (its all_reduce also waits for the "
                             "slowest rank's scoring); allreduce_alone_ms times the same all_reduce after a "
                             "barrier (CUDA events, max over ranks)" if world > 1 else None,
            "phases_ms_rank0": phases, "kept": kept, "moved_rows": n_moved, "algorithmic_bytes": nbytes,
            "score_flops": flops, "score_tflops_per_gpu": round(tf, 1),
            "score_frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4),
            "step_roofline_ms": round(max(nbytes / world / (peaks["hbm_gbs"] * 1e9),
                                          flops / world / (peaks["bf16_tflops"] * 1e12)) * 1e3, 4),
            "limiter": "the exchange (NCCL all_reduce of the head sums) and the per-rank scoring" if world > 1
                       else "scoring (tensor-bound)",
            "device_status": status}


# The reference's published per-step times of its own benchmark (benchmarks/bench_kernels.py, A100
# SXM4 80 GB, compiled Triton kernels, fp16, one layer, median of 5 after 1 warm-up; its
# results/bench_kernels.txt:1-14): ms per compression step of r requests, "actkv" column.
REF_A100_STEP_MS = {(1024, 512): {1: 1.233, 4: 4.128, 16: 15.690, 64: 61.856},
                    (2048, 1536): {1: 1.248, 4: 4.290, 16: 16.214, 64: 63.968},
                    (6144, 4096): {1: 1.394, 4: 4.753, 16: 18.111, 64: 71.083}}


def dropin_reference_shape(dev, iters: int = 5, warmup: int = 1):
    """The reference's own benchmark step through the drop-in API (benchmarks/bench_kernels.py:81-89,
    actkv_step): for r requests of n fp16 tokens (block 16, 8 KV / 32 query heads, head_dim 128,
    one layer, scattered blocks), PagedKVCache.cal_attn scores one action query per request
    against the cache with a precomputed lse, then PagedKVCache.evict keeps the top `budget`
    tokens of each request in turn (keep mask + in-place compaction + block reclamation).  Timed
    as the reference times it: wall clock with a device sync, median of `iters` fresh caches after
    `warmup` untimed steps, the lse (from PagedKVCache.decode_attention) outside the timer."""
    import torch

    from actkv_open_b200.paged import PagedKVCache
    bs, hkv, hq, d = 16, 8, 32, 128
    rows = []

    def build(r, n, seed=0):
        nb = r * math.ceil(n / bs) + 4
        cache = PagedKVCache(nb, bs, hkv, d, dtype=torch.float16, device=dev)
        cache.free = torch.randperm(nb, generator=torch.Generator().manual_seed(seed)).tolist()
        g = torch.Generator(device=dev).manual_seed(seed)
        for i in range(r):
            k = torch.randn(1, n, hkv, d, generator=g, device=dev, dtype=torch.float16)
            cache.append(i, k, torch.randn(k.shape, generator=g, device=dev, dtype=torch.float16))
        return cache

    for (n, budget), ref in REF_A100_STEP_MS.items():
        for r in (1, 4, 16, 64):
            reqs = list(range(r))
            q = torch.randn(r, hq, d, generator=torch.Generator(device=dev).manual_seed(1), device=dev,
                            dtype=torch.float16)
            _, lse = build(r, n).decode_attention(reqs, q)

            def step(cache):
                bt = cache.block_table(reqs)
                out = torch.zeros(r, hkv, bt.shape[1] * bs, device=dev)
                nseen = torch.zeros(r, dtype=torch.int32, device=dev)
                cache.cal_attn(reqs, q, lse, out, nseen)
                for i in reqs:
                    cache.evict(i, out[i], budget)

            for _ in range(warmup):
                step(build(r, n))
            times = []
            for _ in range(iters):
                cache = build(r, n)
                torch.cuda.synchronize(dev)
                t = time.perf_counter()
                step(cache)
                torch.cuda.synchronize(dev)
                times.append((time.perf_counter() - t) * 1e3)
                left = [cache.seq_used[i] for i in reqs]
                assert left == [budget] * r, left
            ms = med(times)
            rows.append({"case": f"{n}->{budget}", "requests": r, "ms": round(ms, 3), "ref_a100_ms": ref[r],
                         "speedup_vs_ref_a100": round(ref[r] / ms, 2)})
    return {"workload": "the reference's benchmarks/bench_kernels.py step (cal_attn + per-request evict, fp16, 1 layer, "
                        "A = 1) through actkv_open_b200.paged.PagedKVCache", "rows": rows,
            "timing": f"wall clock with device sync, median of {iters} fresh caches after {warmup} warm-up step(s); "
                      "lse outside the timer, as the reference times it",
            "ref_source": "the reference's published A100 numbers (results/bench_kernels.txt)"}


def run_ours(args):
    import datetime

    import torch
    import torch.distributed as dist

    from actkv_open_b200 import _native as N
    world, rank, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    N.load()
    peaks, peak_kind = measured_peaks()
    clocks = ClockSampler(gpu_smi_id(torch, dev, local)).start()
    if args.workload in ("config3", "config4"):
        rec = (config3_batch if args.workload == "config3" else config4_record)(args, dev, world, rank, clocks, peaks)
        clk = clocks.stop()
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            ms = rec.get("ms_per_batch_step", rec.get("ms_per_step"))
            print(json.dumps({"metric": METRIC, "value": rec.get("value"), "unit": UNIT, "n_gpus": world,
                              "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                              "data": "synthetic (seeded)", "config": {"workload": rec.get("workload")},
                              "record": rec, "clocks": clk}))
        return
    h = run_headline(args, dev, world, rank, clocks, peaks)
    records = {}
    wanted = [x for x in args.records.split(",") if x]
    if "config3" in wanted:
        records["config3_batch"] = config3_batch(args, dev, world, rank, clocks, peaks)
    if "config4" in wanted:
        records["config4"] = config4_record(args, dev, world, rank, clocks, peaks)
    if "dropin" in wanted and rank == 0 and world == 1:
        records["dropin_reference_shape"] = dropin_reference_shape(dev)
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None if (world > 1 or args.no_cpu_baseline) else cpu_baseline()
    L, S = args.layers, args.seq
    score_kernel = "score_umma_kernel" if args.path == "tcgen05" else "score_pair_kernel"
    ph = h["phases"]
    copy_ms = ph["compact"]
    moves = h["parts"]["moves"]
    line = {
        "metric": METRIC, "value": round(h["value"], 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(h["ms"], 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V with U(0.5,2) channel scales)",
        "config": {"workload": "BASELINE config 2: Qwen3-8B-shaped paged cache, 1 session per GPU",
                   "layers": L, "q_heads": CFG2["HQ"], "kv_heads": CFG2["HKV"], "head_dim": CFG2["D"],
                   "block_size": CFG2["BS"], "tokens": S, "action_tokens": CFG2["A"], "budget": CFG2["BUDGET"],
                   "sinks": CFG2["P"], "decay": CFG2["DECAY"], "top_p": CFG2["TOP_P"], "kept": h["kept"],
                   "moved_rows": h["n_moved"], "l2": "cache 4.8 GB > L2; restored from a device snapshot between steps",
                   "scoring_path": args.path, "sessions_per_gpu": 1},
        "parity": h["parity"],
        "evict_latency_ms": round(h["ms"], 4), "eager_ms_per_step": round(h["eager_ms"], 4),
        "graph_ms_min_median_max": h["graph_ms_min_median_max"],
        "step_timing": "median over the timed steps of a CUDA graph replay of EvictionPipeline.step (graph_step); "
                       "phases_ms: medians of an eager run of the same step with events between its phases",
        "phases_ms": ph, "phases_ms_min_median_max": h["phase_spread"], "algorithmic_bytes": h["nbytes"], "bytes_breakdown": h["parts"], "score_flops": h["flops"],
        "roofline": {"bound": "tensor", "kernel": score_kernel, "achieved": round(h["ach"], 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(h["ach"] / peaks["bf16_tflops"], 4),
                     "frac_of_sustained_peak": round(h["ach"] / peaks["bf16_tflops_sustained"], 4),
                     "traffic": committed_traffic(score_kernel, "config2") if (L, S) == (CFG2["L"], CFG2["S"]) else None,
                     "traffic_source": "profiles/traffic.txt (ncu dram bytes of a 4-layer capture scaled x9; the "
                                       "one-CTA kernel: 2-layer capture scaled x18)",
                     "peak_source": peak_kind, "sm_mhz_median": clk.get("sm_mhz"),
                     "note": "peak = burst cuBLAS bf16; the step runs under sw_power_cap, see clocks"},
        "roofline_compaction": {"bound": "hbm", "achieved": round(moves / (copy_ms * 1e-3) / 1e9, 1),
                                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                "frac": round(moves / (copy_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)},
        "step_roofline_ms": round(max(h["nbytes"] / (peaks["hbm_gbs"] * 1e9),
                                      h["flops"] / (peaks["bf16_tflops"] * 1e12)) * 1e3, 4),
        "e2e": h["e2e"], "gpu_launches": LAUNCHES_PER_STEP * args.steps, "clocks": clk,
        "device_status": h["status"], "cpu_baseline": cpu,
        "region_lse": h.get("region_lse"), "decode_attention": h.get("decode_attention"),
        "kv_gather": h.get("kv_gather"), **records,
    }
    print(json.dumps(line))


def region_lse_measure(torch, pipe, snap, q, lse, args, dev):
    """The action region's causal lse from the cache on the tensor cores (EvictionPipeline.region_lse,
    two launches), timed apart from the step: the reference takes lse from its attention backend
    and does not time it.  Also its largest difference from the set-up's torch fp32 lse."""
    from actkv_open_b200 import _native as N
    pipe.restore(snap)                       # the step's input cache (region_lse does not modify it)
    out = pipe.region_lse(q)
    torch.cuda.synchronize(dev)
    err = float((out - lse).abs().max())
    for _ in range(args.warmup):
        pipe.region_lse(q)
    times = []
    for _ in range(args.steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        pipe.region_lse(q)
        e.record()
        torch.cuda.synchronize(dev)
        times.append(s.elapsed_time(e))
    ms = statistics.mean(times)
    c = pipe.cache
    L, sum_a, hq, d = q.shape
    S = int(c.seq_used[0].item())
    flops = 2 * L * sum_a * hq * d * S
    peaks, _ = measured_peaks()
    return {"ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "frac": round(flops / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
            "max_abs_err_vs_torch_fp32": err, "status": N.read_device_status(dev),
            "traffic": committed_traffic("lse_umma_kernel", "config2") if (L, S) == (CFG2["L"], CFG2["S"]) else None,
            "kernels": ["lse_umma_kernel", "lse_combine_kernel"], "timed_in_step": False}


def decode_measure(torch, pipe, q, args, dev):
    """Paged decode attention with its lse (lse_attn.paged_decode_attention, flash decoding on CUDA
    cores) for the session's last action query, one layer: an HBM-bound read of the layer's K and V
    (not part of the timed step: the reference's attention backend, which the eviction consumes)."""
    from actkv_open_b200 import _native as N
    from actkv_open_b200.kernels.lse_attn import decode_workspace_bytes, paged_decode_attention
    c = pipe.cache
    S = int(c.seq_used[0].item())
    L = c.n_layers
    qd = q[:, -1:].contiguous()                                    # [L, 1, Hq, D]: the last action token
    bt, seq = c.block_table[:1], c.seq_used[:1]
    out = torch.empty(1, qd.shape[2], qd.shape[3], device=dev)
    lse = torch.empty(1, qd.shape[2], device=dev)
    ws = N.workspace(decode_workspace_bytes(1, qd.shape[2], c.n_kv_heads, c.head_dim, c.max_tokens), dev)
    # every layer once (each layer's K and V, 134 MB at config 2, are not the previous call's, so
    # they come from HBM), replayed from a CUDA graph: one call's host set-up is longer than its
    # kernels, so timing single eager calls would time the host
    def all_layers():
        for l in range(L):
            paged_decode_attention(qd[l], c.kv[l], bt, seq, out=out, lse=lse, workspace=ws)
    all_layers()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        all_layers()
    for _ in range(max(3, args.warmup)):
        g.replay()
    torch.cuda.synchronize(dev)
    times = []
    for i in range(max(5, args.steps)):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize(dev)
        times.append(s.elapsed_time(e) / L)
    ms = statistics.median(times)
    nbytes = 2 * S * c.n_kv_heads * c.head_dim * c.kv.element_size()
    peaks, _ = measured_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"ms": round(ms, 4), "bytes": nbytes, "achieved_gbs": round(gbs, 1), "peak_gbs": peaks["hbm_gbs"],
            "frac": round(gbs / peaks["hbm_gbs"], 4), "tokens": S, "status": N.read_device_status(dev),
            "kernels": ["decode_tc_kernel", "decode_combine_kernel"], "timed_in_step": False,
            "note": "per layer: the mean over a CUDA-graph replay of all layers, one query token per session"}


def kv_gather_measure(torch, pipe, dev, reps: int = 5):
    """What HBM serves the paged cache at in the two read patterns (C actkv_measure_kv_gather over
    the whole [L][2][NB][BS][Hkv][D] cache, larger than L2): one head per CTA, as the scoring and
    decode kernels read it (BS pieces of D elements per block, a token row apart), and whole
    blocks.  Median of `reps` launches each, CUDA events on the launching stream."""
    from actkv_open_b200 import _native as N
    c = pipe.cache
    es = c.kv.element_size()
    head_bytes = c.head_dim * es
    row_bytes = c.n_kv_heads * head_bytes
    n_blocks = c.kv.numel() * es // (c.block_size * row_bytes)
    sink = torch.zeros(1, dtype=torch.int64, device=dev)
    lib = N.load()
    out = {"bytes": int(n_blocks * c.block_size * row_bytes)}
    for mode, key in ((0, "one_head_per_cta_gbs"), (1, "whole_rows_gbs")):
        def run():
            N.check(lib.actkv_measure_kv_gather(c.kv.data_ptr(), n_blocks, c.block_size, row_bytes, head_bytes, mode,
                                                sink.data_ptr(), N.stream_ptr(dev)), "measure_kv_gather")
        run()
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(reps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            torch.cuda.synchronize(dev)
            times.append(s.elapsed_time(e))
        out[key] = round(out["bytes"] / (statistics.median(times) * 1e-3) / 1e9, 1)
    out["ratio"] = round(out["whole_rows_gbs"] / out["one_head_per_cta_gbs"], 3)
    out["note"] = ("reads only; one head per CTA = BS pieces of head_dim elements per block, a 2 KB token row "
                   "apart at config 2, the pattern of every K-streaming kernel here")
    return out


def e2e_measure(torch, pipe, snap, q, lse, args, dev, world, nbytes):
    """Same step through the public API (EvictionPipeline.step_host) with the step's inputs (action
    queries and their lse) in pinned host memory -- step_host copies them layer group by layer group
    and scores each group as it lands -- and its results (perm, lengths, tables, free-stack top)
    copied back, all inside the timed region.  (Replaying this from a CUDA graph measured slower,
    2.11 against 1.72 ms on config 2, so it runs eagerly.)"""
    import torch.distributed as dist
    c = pipe.cache
    q_h = q.cpu().pin_memory()
    lse_h = lse.cpu().pin_memory()
    R, W = c.n_sessions, c.max_tokens
    perm_h = torch.empty(R, W, dtype=torch.int64).pin_memory()
    seq_h = torch.empty(R, dtype=torch.int32).pin_memory()
    bt_h = torch.empty(R, c.max_blocks, dtype=torch.int32).pin_memory()
    top_h = torch.empty(1, dtype=torch.int32).pin_memory()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for i in range(args.warmup + args.steps):
        pipe.restore(snap)
        torch.cuda.synchronize(dev)
        s.record()
        pipe.step_host(q_h, lse_h)
        perm_h.copy_(pipe.perm[:R], non_blocking=True)
        seq_h.copy_(c.seq_used[:R], non_blocking=True)
        bt_h.copy_(c.block_table[:R], non_blocking=True)
        top_h.copy_(c.free_top, non_blocking=True)
        e.record()
        torch.cuda.synchronize(dev)
        if i >= args.warmup:
            times.append(s.elapsed_time(e))
    ms = statistics.median(times)
    ms_mean = statistics.mean(times)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    h2d = q.numel() * q.element_size() + lse.numel() * 4
    d2h = perm_h.numel() * 8 + seq_h.numel() * 4 + bt_h.numel() * 4 + 4
    # this host's plain pinned -> device copy of the same input bytes, for reading the number above
    q_d, lse_d = torch.empty_like(q), torch.empty_like(lse)
    copy_ms = []
    for _ in range(5):
        s.record()
        q_d.copy_(q_h, non_blocking=True)
        lse_d.copy_(lse_h, non_blocking=True)
        e.record()
        torch.cuda.synchronize(dev)
        copy_ms.append(s.elapsed_time(e))
    cm = statistics.median(copy_ms)
    return {"value": round(world * nbytes / (ms * 1e-3) / 1e9, 2), "unit": UNIT, "ms_per_step": round(ms, 4),
            "ms_per_step_is": "median of the timed steps", "ms_per_step_mean": round(ms_mean, 4),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "step_ms_min_median_max": [round(min(times), 4), round(statistics.median(times), 4), round(max(times), 4)],
            "h2d_copy_alone_ms": round(cm, 4), "h2d_copy_alone_gbs": round(h2d / (cm * 1e-3) / 1e9, 1),
            "api": "actkv_open_b200.engine.EvictionPipeline.step_host"}


# --------------------------------------------------------------------------------------- CPU side
def cpu_threads() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, 32))


class CpuLayer:
    """One layer of the config-2 session for the CPU oracle (the reference's torch path restated in
    numpy): fp32 K/V with the channel scales, scattered blocks, 128 N(0,1) action queries and their
    exact causal lse (computed untimed)."""

    def __init__(self, seed: int = 0):
        import numpy as np
        c = CFG2
        S, HQ, HKV, D, BS, A = c["S"], c["HQ"], c["HKV"], c["D"], c["BS"], c["A"]
        G = HQ // HKV
        rng = np.random.default_rng(seed)
        nb = S // BS
        scale = rng.random((HKV, D), dtype=np.float32) * 1.5 + 0.5
        self.kv = rng.standard_normal((2, nb, BS, HKV, D), dtype=np.float32) * scale
        self.perm = rng.permutation(nb)
        self.q = rng.standard_normal((A, HQ, D), dtype=np.float32)
        free = list(self.perm)
        self.table = [free.pop() for _ in range(nb)]
        self.free = free
        bt = np.asarray(self.table, np.int64)
        pos = np.arange(S)
        k = self.kv[0].reshape(nb * BS, HKV, D)[bt[pos // BS] * BS + pos % BS]            # [S, HKV, D]
        self.lse = np.empty((A, HQ), np.float32)
        see = S - A + np.arange(A)
        for h in range(HKV):
            qh = self.q[:, h * G:(h + 1) * G].reshape(A * G, D).astype(np.float64)
            logits = (qh @ k[:, h].T.astype(np.float64)) * D ** -0.5                     # [A*G, S]
            logits[pos[None, :] > np.repeat(see, G)[:, None]] = -np.inf
            m = logits.max(1, keepdims=True)
            self.lse[:, h * G:(h + 1) * G] = (m[:, 0] + np.log(np.exp(logits - m).sum(1))).reshape(A, G)

    def run(self, tokens: int, threads: int):
        """Score the last ``tokens`` action tokens with the reference's per-token computation (one
        action_scores call each, run ``threads`` at a time, folded into the running mean in token
        order -- the same floats as the reference's sequential loop), then this layer's ActionLRFU
        update and evict (mask, plan, copies, tables).  Returns (seconds, moved rows)."""
        from concurrent.futures import ThreadPoolExecutor

        import numpy as np
        from threadpoolctl import threadpool_limits

        from oracle import actkv_oracle as O
        c = CFG2
        S, HKV, BS, A = c["S"], c["HKV"], c["BS"], c["A"]
        nb = S // BS
        cache = O.PagedKVCache(nb, BS, HKV, c["D"], 1)
        cache.kv[0] = self.kv                                       # fresh copy: evict mutates it
        cache.free = list(self.free)
        cache.tables[0] = list(self.table)
        cache.seq_used[0] = S
        bt = np.asarray(self.table, np.int64)[None]
        first = A - tokens

        def one(j):                                                 # action token first + j
            jj = first + j
            n = S - A + jj + 1
            out = np.zeros((1, HKV, nb * BS), np.float32)
            O.action_scores(self.q[jj][None], cache.kv[0], bt, [n], self.lse[jj][None], out,
                            np.zeros(1, np.int64))
            return out[0, :, :n]                                    # = p of this token (out was 0)

        t0 = time.perf_counter()
        with threadpool_limits(1):
            if threads > 1:
                with ThreadPoolExecutor(threads) as ex:
                    ps = list(ex.map(one, range(tokens)))
            else:
                ps = [one(j) for j in range(tokens)]
        out = np.zeros((HKV, S), np.float32)
        for j, p in enumerate(ps):                                  # out += (p - out) / (n_seen + 1)
            n = p.shape[1]
            cur = out[:, :n]
            out[:, :n] = cur + (p - cur) / (np.float32(j) + np.float32(1.0))
        pol = O.ActionLRFU(decay=c["DECAY"], top_p=c["TOP_P"])
        pol.reset(1)
        pol.act = out.mean(0, keepdims=True)
        pol.n_act = tokens
        pol.update_scores(S, c["P"])
        perm = cache.evict(0, pol.ks, c["BUDGET"], c["P"])
        sec = time.perf_counter() - t0
        return sec, moved_rows(list(perm), S, BS)


def cpu_baseline(seed: int = 0):
    """The CPU oracle on one of the config-2 session's 36 layers: all 128 action tokens scored, then
    the layer's ActionLRFU update and evict, on every host thread available (up to 32)."""
    threads = cpu_threads()
    lay = CpuLayer(seed)
    sec, n_moved = lay.run(CFG2["A"], threads)
    nbytes, _ = algorithmic_bytes(1, CFG2["S"], n_moved)
    return {"value": round(nbytes / sec / 1e9, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "seconds_per_layer": round(sec, 3), "seconds_per_step_extrapolated": round(sec * LAYERS_CONFIG2, 1),
            "sample": f"config 2, 1 of 36 layers: all 128 action tokens scored with the reference's per-token "
                      f"computation ({threads} threads over tokens, folded in token order), then that layer's "
                      "ActionLRFU update and evict; throughput in the step's algorithmic bytes for one layer "
                      "(linear in the layers)"}


def run_reference(args):
    """The reference's CPU path (the oracle port, on every host thread) on the headline workload:
    each timed step is one full layer of the config-2 session (128 action tokens scored, ActionLRFU,
    evict); warm-up steps score 8 tokens.  ms_per_step is the measured time of that one-layer step;
    the full 36-layer step is 36 times it (extrapolated_ms_per_full_step)."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    threads = cpu_threads()
    lay = CpuLayer(args.seed)
    for _ in range(args.warmup):
        lay.run(8, threads)
    secs, moved = [], 0
    for _ in range(args.steps):
        s, moved = lay.run(CFG2["A"], threads)
        secs.append(s)
    sec = med(secs)
    nbytes, _ = algorithmic_bytes(1, CFG2["S"], moved)
    v = nbytes / sec / 1e9
    sample = (f"config 2, 1 of 36 layers per step: all 128 action tokens scored ({threads} threads over tokens, "
              "folded in token order), ActionLRFU update and evict of that layer")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "BASELINE config 2 (per-step sample: 1 of 36 layers, all 128 action tokens)",
                   "tokens": CFG2["S"], "layers_sampled": 1, "action_tokens": CFG2["A"]},
        "ms_per_step_is": "one layer (the timed sample)", "extrapolation_factor": LAYERS_CONFIG2,
        "extrapolated_ms_per_full_step": round(sec * 1e3 * LAYERS_CONFIG2, 1),
        "step_s_min_median_max": [round(min(secs), 3), round(sec, 3), round(max(secs), 3)],
        "cpu_baseline": {"kind": "port", "cores": threads, "sample": sample, "value": round(v, 4), "unit": UNIT},
        "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def causal_lse(torch, cache, r, q_r, A, scale):
    """Exact causal lse [L, A, Hq] of session r's last A tokens (action token j sees the first
    n - A + j + 1 tokens), gathered from the paged cache with torch: workload set-up, untimed."""
    import torch.nn.functional as F  # noqa: F401
    c = cache
    L, _, hq, d = q_r.shape
    hkv, bs = c.n_kv_heads, c.block_size
    n = int(c.seq_used[r].item())
    bt = c.block_table[r, :math.ceil(n / bs)].long()
    pos = torch.arange(n, device=c.device)
    slots = bt[pos // bs] * bs + pos % bs
    see = n - A + torch.arange(A, device=c.device)
    out = torch.empty(L, A, hq, device=c.device)
    for l in range(L):
        k = c.kv[l, 0].view(-1, hkv, d)[slots].float()                               # [n, Hkv, D]
        qq = q_r[l].float().view(A, hkv, hq // hkv, d)
        logits = torch.einsum("ahgd,nhd->ahgn", qq, k) * scale
        logits.masked_fill_(pos[None, None, None, :] > see[:, None, None, None], float("-inf"))
        out[l] = torch.logsumexp(logits, -1).reshape(A, hq)
    return out



def adversarial_mask(torch, cache, kind: int, W: int):
    """The agent-loop stress masks, in turn: alternating keep/evict, all-keep, sinks only (the
    first P tokens), one kept token per block."""
    R = cache.n_sessions
    pos = torch.arange(W, device=cache.device)[None, :].expand(R, W)
    n = cache.seq_used[:R, None]
    if kind == 0:
        keep = pos % 2 == 0
    elif kind == 1:
        keep = torch.ones_like(pos, dtype=torch.bool)
    elif kind == 2:
        keep = pos < CFG5["P"]
    else:
        keep = pos % cache.block_size == 0
    return (keep & (pos < n)).to(torch.uint8).contiguous()


def run_config5(args):
    """BASELINE config 5 on this rank's 2 sessions: every round appends 1088 tokens per session on
    the device (DevicePagedCache.append), then evicts to the budget through EvictionPipeline.step
    replayed from a CUDA graph (graph_step: score -> ActionLRFU -> keep mask -> compaction), or,
    every 5th round, through
    evict_with_mask with an adversarial mask.  Timed (CUDA events, summed over rounds): the append
    and the eviction; untimed: the synthetic queries and their exact causal lse."""
    import torch
    import torch.distributed as dist

    from actkv_open_b200 import _native as N
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c5 = CFG5
    L, HQ, HKV, D, BS, A, P = c5["L"], c5["HQ"], c5["HKV"], c5["D"], c5["BS"], c5["A"], c5["P"]
    R, NEW, BUDGET = c5["SESSIONS"], c5["NEW"] + c5["A"], c5["BUDGET"]
    # an all-keep adversarial round leaves a session at its full length, and the next round appends
    # on top of it before evicting
    W = math.ceil((BUDGET + P + 2 * NEW) / BS) * BS
    nb = R * (W // BS + 1)
    gen = torch.Generator(device=dev).manual_seed(5000 + args.seed + rank)
    cache = DevicePagedCache(nb, BS, HKV, D, L, R, W, dtype=torch.bfloat16, device=dev)
    pipe = EvictionPipeline(cache, EvictionConfig(decay=c5["DECAY"], top_p=c5["TOP_P"]))
    free = torch.randperm(nb, generator=torch.Generator().manual_seed(args.seed + rank)).tolist()
    pipe.load([[] for _ in range(R)], [0] * R, free, P)
    k_new = torch.randn(L, R * NEW, HKV, D, generator=gen, device=dev).to(torch.bfloat16)
    v_new = torch.randn(L, R * NEW, HKV, D, generator=gen, device=dev).to(torch.bfloat16)
    scale = D ** -0.5
    N.load()
    # every round appends NEW tokens to each session: the offsets live on the device once
    new_off = torch.arange(0, (R + 1) * NEW, NEW, dtype=torch.int32, device=dev)
    q_buf = torch.empty(L, R * A, HQ, D, dtype=torch.bfloat16, device=dev)
    lse_buf = torch.empty(L, R * A, HQ, device=dev)
    clocks = ClockSampler(gpu_smi_id(torch, dev, local)).start()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def loop(rounds: int, timed: bool):
        t_append, t_evict, nbytes, moved_total, adv = 0.0, 0.0, 0, 0, 0
        for rnd in range(rounds):
            torch.cuda.synchronize(dev)
            clocks.active = timed
            s, e = ev(), ev()
            s.record()
            cache.append(k_new, v_new, new_off, max_new=NEW, check=False)
            e.record()
            torch.cuda.synchronize(dev)
            clocks.active = False
            t_append += s.elapsed_time(e)
            lens = cache.seq_used[:R].tolist()
            if (rnd + 1) % c5["ADV_EVERY"] == 0:
                keep = adversarial_mask(torch, cache, adv % 4, W)
                adv += 1
                torch.cuda.synchronize(dev)
                clocks.active = timed
                s.record()
                pipe.evict_with_mask(keep)
                e.record()
            else:
                q = torch.randn(L, R * A, HQ, D, generator=gen, device=dev).to(torch.bfloat16)
                lse = torch.cat([causal_lse(torch, cache, r, q[:, r * A:(r + 1) * A], A, scale) for r in range(R)], 1)
                q_buf.copy_(q)                   # the step's input buffers stay put: one graph serves
                lse_buf.copy_(lse)               # every round (EvictionPipeline.graph_step)
                pipe.set_round([A] * R, [BUDGET] * R)
                torch.cuda.synchronize(dev)
                clocks.active = timed
                s.record()
                pipe.graph_step(q_buf, lse_buf)
                e.record()
            torch.cuda.synchronize(dev)
            clocks.active = False
            t_evict += s.elapsed_time(e)
            kept = pipe.kept[:R].tolist()
            perms = pipe.perm[:R].cpu()
            moved = sum(moved_rows(perms[r, :kept[r]].tolist(), lens[r], BS) for r in range(R))
            moved_total += moved
            scored = (rnd + 1) % c5["ADV_EVERY"] != 0
            nbytes += (2 * L * 2 * R * NEW * HKV * D * 2                          # appended rows, read + write
                       + (sum(lens) * L * HKV * D * 2 if scored else 0)          # K read by the scoring
                       + 2 * moved * 2 * L * HKV * D * 2)                        # moved rows, read + write
        return t_append, t_evict, nbytes, moved_total

    # untimed warm-up rounds (first-call set-up of every kernel and buffer), then a fresh state
    loop(min(args.warmup, args.rounds), False)
    pipe.load([[] for _ in range(R)], [0] * R, free, P)
    if world > 1:
        dist.barrier()
    t_append, t_evict, nbytes, moved_total = loop(args.rounds, True)
    status = N.read_device_status(dev)
    ms = t_append + t_evict
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
        dist.destroy_process_group()
    clk = clocks.stop()
    if rank != 0:
        return
    print(json.dumps({
        "metric": METRIC, "value": round(world * nbytes / (ms * 1e-3) / 1e9, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.rounds, "warmup": min(args.warmup, args.rounds), "ms_per_step": round(ms / args.rounds, 4),
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V and queries)",
        "config": {"workload": "BASELINE config 5: agent loop, 2 sessions per GPU", "rounds": args.rounds,
                   "sessions_per_gpu": R, "layers": L, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                   "block_size": BS, "tokens_per_round": NEW, "action_tokens": A, "budget": BUDGET,
                   "adversarial_every": c5["ADV_EVERY"], "max_tokens": W},
        "round_ms": {"append": round(t_append / args.rounds, 4), "evict": round(t_evict / args.rounds, 4)},
        "rows_moved_total": moved_total, "final_lengths": cache.seq_used[:R].tolist(),
        "gpu_launches_per_round": "append 3; scored rounds +9, adversarial rounds +4",
        "clocks": clk, "device_status": status}))


def main(argv=None):
    args = parse(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config5":
        run_config5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
