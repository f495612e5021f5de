"""Helpers for the GPU parity tests (imported without touching CUDA, so collection works anywhere)."""
import numpy as np
import pytest
import torch

import cases


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def assert_device_clean(dev):
    from actkv_open_b200 import _native as N
    torch.cuda.synchronize(dev)
    st = N.read_device_status(dev)
    assert st == 0, f"device status word {st:#x} (1: bad index, 2: timeout, 4: misaligned)"


def gpu_cache(case: cases.SessionCase, dev):
    """actkv_open_b200.paged.PagedKVCache holding the case's sessions."""
    from actkv_open_b200.paged import PagedKVCache
    c = PagedKVCache(case.num_blocks, case.bs, case.hkv, case.d, n_layers=case.n_layers,
                     dtype=cases.DTYPES[case.dtype], device=dev)
    c.kv.copy_(case.kv.to(dev))
    c.free = list(case.free)
    for r, (t, n) in enumerate(zip(case.tables, case.seq_lens)):
        c.tables[r] = list(t)
        c.seq_used[r] = n
    return c


def packed_region(case: cases.SessionCase, lse_list, dev):
    """q [L, sumA, Hq, D], lse [L, sumA, Hq] and act_off [R+1] of every session's action region."""
    q = torch.cat([qq for qq in case.q], dim=1).to(dev).contiguous()
    lse = torch.cat([torch.as_tensor(np.asarray(l, np.float32)) for l in lse_list], dim=1).to(dev).contiguous()
    off = np.concatenate([[0], np.cumsum(case.act_lens)]).astype(np.int32)
    return q, lse, torch.from_numpy(off).to(dev)


def oracle_lse(case: cases.SessionCase):
    """Exact causal lse [L, A, Hq] of every session's action region (CPU oracle)."""
    from oracle import actkv_oracle as O
    kv = cases.to_np(case.kv)
    out = []
    for r, n in enumerate(case.seq_lens):
        q = cases.to_np(case.q[r])
        bt = np.asarray(case.tables[r], np.int64)
        out.append(np.stack([O.causal_region_lse(q[l], kv[l], bt, n) for l in range(case.n_layers)]))
    return out


def oracle_heads(case: cases.SessionCase, lse_list):
    """Per-head region scores [L, Hkv, S] of every session (CPU oracle)."""
    from oracle import actkv_oracle as O
    kv = cases.to_np(case.kv)
    res = []
    for r, n in enumerate(case.seq_lens):
        q = cases.to_np(case.q[r])
        bt = np.asarray(case.tables[r], np.int64)
        res.append(np.stack([O.layer_scores(kv[l], bt, n, q[l], lse_list[r][l]) for l in range(case.n_layers)]))
    return res
