"""Causal region lse on the tensor cores (``action_region_lse`` -> C ``actkv_region_lse``) against
the CPU oracle's causal lse (paged_decode_attention per action token, actkv/kernels/lse_attn.py
:42-60) and against the lse the reference itself produced for the bf16 pipeline golden
(tests/golden/pipe_bf16.npz)."""
import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_device_clean, need_gpu, oracle_lse, packed_region

pytestmark = pytest.mark.gpu

# products of bf16/fp16 operands are exact in the fp32 accumulator; the sums differ from the fp64
# oracle only in order and in ex2.approx (relative error ~2^-22 per term)
RTOL, ATOL = 1e-5, 2e-5

LSE_CASES = {
    "bf16_g4_two_sessions": dict(seed=77, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[300, 517],
                                 act_lens=[24, 37], dtype="bfloat16", extra_blocks=5, channel_scale=True),
    # A*G = 800 and 560: several 128-row blocks per head, the last one partly padding
    "bf16_g8_row_blocks": dict(seed=3, n_layers=2, hq=16, hkv=2, d=128, bs=16, seq_lens=[700, 1500],
                               act_lens=[100, 70], dtype="bfloat16", extra_blocks=3),
    "fp16_g2_ragged_bs8": dict(seed=5, n_layers=2, hq=4, hkv=2, d=128, bs=8, seq_lens=[333, 129, 17],
                               act_lens=[200, 64, 3], dtype="float16", extra_blocks=4),
    "bf16_g16": dict(seed=6, n_layers=1, hq=32, hkv=2, d=128, bs=16, seq_lens=[400], act_lens=[40],
                     dtype="bfloat16", extra_blocks=1),
    "bf16_g1_bs32": dict(seed=4, n_layers=1, hq=2, hkv=2, d=128, bs=32, seq_lens=[900], act_lens=[300],
                         dtype="bfloat16", extra_blocks=2),
    # longer than one split (4096 tokens): partials of several splits merged
    "bf16_long_splits": dict(seed=21, n_layers=1, hq=8, hkv=2, d=128, bs=16, seq_lens=[20000, 9000],
                             act_lens=[33, 130], dtype="bfloat16", extra_blocks=2),
    # a session without action tokens and one with a single action token
    "bf16_zero_and_one_action": dict(seed=12, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[300, 650, 200],
                                     act_lens=[24, 0, 1], dtype="bfloat16", extra_blocks=3),
}


def _region_lse(case, dev, **kw):
    from actkv_open_b200.kernels.lse_attn import action_region_lse
    q, _, off = packed_region(case, [np.zeros((case.n_layers, a, case.hq), np.float32) for a in case.act_lens],
                              dev)
    kv = case.kv.to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    return action_region_lse(q, off, kv, bt, seq, **kw), off.cpu().numpy()


@pytest.mark.parametrize("name", list(LSE_CASES))
def test_region_lse_matches_oracle(name):
    dev = need_gpu()
    case = cases.build_sessions(**LSE_CASES[name])
    want = oracle_lse(case)
    got, off = _region_lse(case, dev)
    got = got.cpu().numpy()
    for r, a in enumerate(case.act_lens):
        np.testing.assert_allclose(got[:, off[r]:off[r] + a], want[r], rtol=RTOL, atol=ATOL,
                                   err_msg=f"{name} session {r}")
    assert_device_clean(dev)


def test_region_lse_matches_reference_golden(golden):
    """The reference's paged_decode_attention_ref lse of the bf16 pipeline case, per action token."""
    dev = need_gpu()
    g = golden("pipe_bf16.npz")
    case = cases.build_sessions(**cases.PIPE_BF16)
    assert cases.digest(case.kv) == g["meta"]["kv_sha256_in"]
    got, off = _region_lse(case, dev)
    got = got.cpu().numpy()
    for r, a in enumerate(case.act_lens):
        np.testing.assert_allclose(got[:, off[r]:off[r] + a], g[f"lse_{r}"], rtol=RTOL, atol=ATOL)
    assert_device_clean(dev)


def test_region_lse_feeds_the_scorer_like_the_oracle_lse():
    """Scores computed with the kernel's lse equal scores computed with the oracle's."""
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import action_scores_region
    case = cases.build_sessions(**LSE_CASES["bf16_g8_row_blocks"])
    lse_gpu, _ = _region_lse(case, dev)
    q, lse_cpu, off = packed_region(case, oracle_lse(case), dev)
    kv = case.kv.to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    W = bt.shape[1] * case.bs
    outs = []
    for lse in (lse_gpu, lse_cpu):
        out = torch.zeros(len(case.seq_lens), case.n_layers, case.hkv, W, device=dev)
        action_scores_region(q, lse, off, kv, bt, seq, out, path="tcgen05")
        outs.append(out.cpu().numpy())
    np.testing.assert_allclose(outs[0], outs[1], rtol=1e-4, atol=1e-9)
    assert_device_clean(dev)


def test_region_lse_rejects_what_it_has_no_kernel_for():
    dev = need_gpu()
    spec = dict(LSE_CASES["bf16_g4_two_sessions"])
    with pytest.raises(NotImplementedError):
        _region_lse(cases.build_sessions(**(spec | dict(dtype="float32"))), dev)
    with pytest.raises(NotImplementedError):
        _region_lse(cases.build_sessions(**(spec | dict(bs=4))), dev)


def test_region_lse_rejects_a_small_workspace():
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    case = cases.build_sessions(**LSE_CASES["bf16_g4_two_sessions"])
    q, _, off = packed_region(case, [np.zeros((case.n_layers, a, case.hq), np.float32) for a in case.act_lens], dev)
    kv = case.kv.to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    out = torch.empty(case.n_layers, q.shape[1], case.hq, device=dev)
    ws = torch.empty(16, dtype=torch.uint8, device=dev)
    code = N.load().actkv_region_lse(
        q.data_ptr(), N.dtype_code(q), q.stride(0), q.stride(1), q.stride(2), off.data_ptr(),
        kv.data_ptr(), N.dtype_code(kv), *kv.stride()[:5], bt.data_ptr(), bt.stride(0), seq.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), len(case.seq_lens), case.n_layers, bt.shape[1],
        case.num_blocks, case.bs, case.hq, case.hkv, case.d, q.shape[1], bt.shape[1] * case.bs,
        case.d ** -0.5, ws.data_ptr(), ws.numel(), N.status_word(dev).data_ptr(), N.stream_ptr(dev))
    assert code == -6


def test_pipeline_step_without_lse_computes_it_on_the_device(golden):
    """EvictionPipeline.step(q) with no lse: the same keep masks as the step fed the reference's
    recorded lse (masks equal except at near-ties of the keep scores)."""
    dev = need_gpu()
    from actkv_open_b200.config import EvictionConfig
    from actkv_open_b200.engine import DevicePagedCache, EvictionPipeline
    from conftest import assert_masks_match
    g = golden("pipe_bf16.npz")
    case = cases.build_sessions(**cases.PIPE_BF16)
    R = len(case.seq_lens)
    res = []
    for given in (True, False):
        cache = DevicePagedCache(case.num_blocks, case.bs, case.hkv, case.d, case.n_layers, R, max(case.seq_lens),
                                 dtype=cases.DTYPES[case.dtype], device=dev)
        cache.kv.copy_(case.kv.to(dev))
        pipe = EvictionPipeline(cache, EvictionConfig(decay=cases.PIPE_BF16_DECAY, top_p=cases.PIPE_BF16_TOP_P))
        pipe.load(case.tables, case.seq_lens, case.free, cases.PIPE_BF16_PROTECTED)
        pipe.set_round(case.act_lens, cases.PIPE_BF16_BUDGETS)
        q, lse, _ = packed_region(case, [g[f"lse_{r}"] for r in range(R)], dev)
        pipe.step(q, lse if given else None)
        torch.cuda.synchronize()
        res.append((pipe.keep.cpu().numpy().astype(bool), pipe.ks[1 - pipe.cur].cpu().numpy()))
    for r, n in enumerate(case.seq_lens):
        assert_masks_match(res[1][0][r, :n], res[0][0][r, :n], res[0][1][r, :, :n].mean(0), rtol=1e-3,
                           what=f"session {r}")
        assert res[1][0][r, :n].sum() == min(n, cases.PIPE_BF16_PROTECTED + cases.PIPE_BF16_BUDGETS[r])
    assert_device_clean(dev)
