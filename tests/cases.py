"""Seeded synthetic inputs shared by the golden-fixture generator, the oracle tests and the GPU
parity tests.  Everything is built on the CPU with torch.Generator so that the same seed gives
the same bytes here and on the GPU box; fixtures store a checksum of what they were made from.

BASELINE config 1 (and the small cases) come from here; the benchmark builds the large configs
itself on the device with the same recipe.
"""
from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass, field

import numpy as np
import torch

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = a.detach().cpu() if isinstance(a, torch.Tensor) else torch.as_tensor(np.asarray(a))
        if a.dtype == torch.bfloat16:
            a = a.view(torch.int16)
        h.update(np.ascontiguousarray(a.numpy()).tobytes())
    return h.hexdigest()


def to_np(t: torch.Tensor) -> np.ndarray:
    """numpy copy; bf16 becomes float32 (exact)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.numpy().copy()


@dataclass
class SessionCase:
    """A paged cache holding R sessions plus each session's causal action region."""
    n_layers: int
    hq: int
    hkv: int
    d: int
    bs: int
    seq_lens: list
    act_lens: list
    dtype: str
    num_blocks: int
    free0: list                   # initial free list (popped from its end)
    kv: torch.Tensor              # [L, 2, NB, BS, Hkv, D] after appending every session
    tables: list                  # per session list of physical blocks
    free: list                    # free list after the sessions were allocated
    q: list = field(default_factory=list)    # per session [L, A, Hq, D] (cache dtype)


def build_sessions(seed, n_layers, hq, hkv, d, bs, seq_lens, act_lens, dtype="float32",
                   extra_blocks=8, channel_scale=False) -> SessionCase:
    """Seeded cache: shuffled free list, K/V ~ N(0,1) (times a per-layer, per-channel scale drawn
    from U(0.5, 2) when ``channel_scale``), action queries ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    tdt = DTYPES[dtype]
    nb = sum(math.ceil(n / bs) for n in seq_lens) + extra_blocks
    free = torch.randperm(nb, generator=g).tolist()
    kv = torch.zeros(n_layers, 2, nb, bs, hkv, d, dtype=tdt)
    flat = kv.view(n_layers, 2, nb * bs, hkv, d)
    scale = (torch.rand(n_layers, 1, hkv, d, generator=g) * 1.5 + 0.5) if channel_scale else None
    pool = list(free)
    tables = []
    qs = []
    for n, a in zip(seq_lens, act_lens):
        k = torch.randn(n_layers, n, hkv, d, generator=g)
        v = torch.randn(n_layers, n, hkv, d, generator=g)
        if scale is not None:
            k, v = k * scale, v * scale
        blocks = [pool.pop() for _ in range(math.ceil(n / bs))]
        tables.append(blocks)
        pos = torch.arange(n)
        slots = torch.tensor(blocks, dtype=torch.long)[pos // bs] * bs + pos % bs
        flat[:, 0, slots] = k.to(tdt)
        flat[:, 1, slots] = v.to(tdt)
        qs.append(torch.randn(n_layers, a, hq, d, generator=g).to(tdt))
    return SessionCase(n_layers, hq, hkv, d, bs, list(seq_lens), list(act_lens), dtype, nb, free,
                       kv, tables, pool, qs)


def block_table_array(tables, min_width=1):
    mb = max([len(t) for t in tables] + [min_width])
    bt = np.zeros((len(tables), mb), np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    return bt


# one fp32 layer, GQA 32/8, D=128, BS=16, 2048 tokens, action region of
# the last 64 tokens, 4 sinks, 30% of the tokens kept, ActionLRFU decay 0.9 / top_p 0.9.
CONFIG1 = dict(seed=2024, n_layers=1, hq=32, hkv=8, d=128, bs=16, seq_lens=[2048], act_lens=[64],
               dtype="float32", extra_blocks=0)
CONFIG1_PROTECTED = 4
CONFIG1_BUDGET = int(0.3 * 2048)
CONFIG1_DECAY = 0.9
CONFIG1_TOP_P = 0.9

# A small bf16, multi-layer, multi-session pipeline case: head_dim 128 so that it runs on the
# tensor-core scoring path, ragged lengths, action regions not a multiple of 4.
PIPE_BF16 = dict(seed=77, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[300, 517],
                 act_lens=[24, 37], dtype="bfloat16", extra_blocks=5, channel_scale=True)
PIPE_BF16_PROTECTED = 4
PIPE_BF16_BUDGETS = [60, 103]
PIPE_BF16_DECAY = 0.9
PIPE_BF16_TOP_P = 0.9
