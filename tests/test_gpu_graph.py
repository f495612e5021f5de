"""EvictionPipeline.graph_step (the step replayed from CUDA graphs) against the eager step: four
consecutive rounds with shrinking budgets, so both keep-score buffer parities are captured and
replayed; every round must leave identical device state."""
import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_device_clean, need_gpu

pytestmark = pytest.mark.gpu

CASE = dict(seed=41, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[700, 430], act_lens=[24, 37],
            dtype="bfloat16", extra_blocks=6)
BUDGETS = [[300, 200], [220, 150], [160, 110], [100, 70]]


def _pipes(case, dev):
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    out = []
    for _ in range(2):
        c = DevicePagedCache(case.num_blocks, case.bs, case.hkv, case.d, case.n_layers, 2, max(case.seq_lens),
                             dtype=cases.DTYPES[case.dtype], device=dev)
        c.kv.copy_(case.kv.to(dev))
        p = EvictionPipeline(c, EvictionConfig(decay=0.9, top_p=0.9))
        p.load(case.tables, case.seq_lens, case.free, 4)
        out.append(p)
    return out


def _state(p):
    c = p.cache
    return [t.clone() for t in (p.keep[:2], p.perm[:2], c.block_table[:2], c.seq_used[:2], c.free_top,
                                c.free_list, p.ks[p.cur][:2], p.pin[p.cur][:2], c.kv)]


def test_graph_replay_equals_eager_steps():
    dev = need_gpu()
    case = cases.build_sessions(**CASE)
    eager, graphed = _pipes(case, dev)
    g = torch.Generator(device=dev).manual_seed(7)
    sum_a = sum(case.act_lens)
    q_buf = torch.empty(case.n_layers, sum_a, case.hq, case.d, dtype=torch.bfloat16, device=dev)
    lse_buf = torch.empty(case.n_layers, sum_a, case.hq, device=dev)
    for rnd, budgets in enumerate(BUDGETS):
        q_buf.copy_(torch.randn(q_buf.shape, generator=g, device=dev).to(torch.bfloat16))
        lse_buf.copy_(torch.rand(lse_buf.shape, generator=g, device=dev) * 2 + 7)
        for p in (eager, graphed):
            p.set_round(case.act_lens, budgets)
        eager.step(q_buf, lse_buf)
        graphed.graph_step(q_buf, lse_buf)
        torch.cuda.synchronize()
        assert eager.cur == graphed.cur
        for a, b in zip(_state(eager), _state(graphed)):
            assert torch.equal(a, b), f"round {rnd}"
        assert np.all(eager.cache.seq_used[:2].cpu().numpy() == [min(n, 4 + b) for n, b in
                                                                  zip(eager.cache.seq_used[:2].tolist(), budgets)])
    assert len(graphed._graphs) == 2          # one graph per keep-score buffer parity
    assert_device_clean(dev)


def test_step_host_with_graphed_finish_equals_eager_steps():
    """step_host replays the part of the step after the scoring from CUDA graphs; over four rounds
    it must leave the same device state as eager steps."""
    dev = need_gpu()
    case = cases.build_sessions(**CASE)
    eager, hosted = _pipes(case, dev)
    g = torch.Generator(device=dev).manual_seed(8)
    sum_a = sum(case.act_lens)
    q_h = torch.empty(case.n_layers, sum_a, case.hq, case.d, dtype=torch.bfloat16).pin_memory()
    lse_h = torch.empty(case.n_layers, sum_a, case.hq).pin_memory()
    for rnd, budgets in enumerate(BUDGETS):
        q = torch.randn(q_h.shape, generator=g, device=dev).to(torch.bfloat16)
        lse = torch.rand(lse_h.shape, generator=g, device=dev) * 2 + 7
        q_h.copy_(q)
        lse_h.copy_(lse)
        for p in (eager, hosted):
            p.set_round(case.act_lens, budgets)
        eager.step(q, lse)
        hosted.step_host(q_h, lse_h, layer_groups=2)
        torch.cuda.synchronize()
        assert eager.cur == hosted.cur
        for a, b in zip(_state(eager), _state(hosted)):
            assert torch.equal(a, b), f"round {rnd}"
    assert len(hosted._graphs) == 2
    assert_device_clean(dev)
