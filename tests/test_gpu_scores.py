"""GPU parity of LSE-recovery scoring (Algorithm 3) against the reference's golden outputs and the
CPU oracle: the drop-in one-token ``action_scores`` and the fused region kernel on both paths
(CUDA cores, tcgen05 with one CTA per tile, tcgen05 on CTA pairs).  Tolerance: scores within 1e-3 relative (fp32 accumulate), as the
eviction path's contract states; the one-token path is held to the reference's own 1e-4."""
import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_device_clean, need_gpu, oracle_heads, oracle_lse, packed_region

pytestmark = pytest.mark.gpu

RTOL = 1e-3
ATOL = 1e-12


def test_action_scores_matches_reference_golden(golden):
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import action_scores
    g = golden("scores_small.npz")
    for i, (lens, hq, hkv, d, bs) in enumerate(g["meta"]["shapes"]):
        p = f"c{i}_"
        case = cases.build_sessions(100 + i, 1, hq, hkv, d, bs, lens, [3] * len(lens))
        kv = case.kv[0].to(dev)
        bt = torch.from_numpy(g[p + "bt"]).to(dev)
        seq = torch.from_numpy(g[p + "seq"]).to(dev)
        out = torch.zeros(g[p + "out"].shape, device=dev)
        ns = torch.zeros(len(lens), dtype=torch.int32, device=dev)
        for step in range(3):
            q = torch.from_numpy(g[p + "q"][step]).to(dev)
            lse = torch.from_numpy(g[p + "lse"][step]).to(dev)
            action_scores(q, kv, bt, seq, lse, out, ns)
        torch.testing.assert_close(out.cpu(), torch.from_numpy(g[p + "out"]), rtol=1e-4, atol=1e-6)
        assert ns.cpu().tolist() == g[p + "n_seen"].tolist()
    assert_device_clean(dev)


def test_recovered_scores_are_probabilities():
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import action_scores, paged_decode_attention_ref
    from gpu_util import gpu_cache
    case = cases.build_sessions(7, 1, 1, 1, 16, 16, [50], [1])
    c = gpu_cache(case, dev)
    bt, seq = c.block_table([0]), c.seq_tensor([0])
    q = torch.randn(1, 1, 16, generator=torch.Generator().manual_seed(1)).to(dev)
    _, lse = paged_decode_attention_ref(q, c.kv[0], bt, seq)
    out = torch.zeros(1, 1, bt.shape[1] * 16, device=dev)
    action_scores(q, c.kv[0], bt, seq, lse, out, torch.zeros(1, dtype=torch.int32, device=dev))
    assert abs(float(out[0, 0, :50].sum()) - 1.0) < 1e-4
    assert float(out[0, 0, 50:].abs().sum()) == 0.0
    assert_device_clean(dev)


def test_action_scores_rejects_a_buffer_narrower_than_the_cache():
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import action_scores
    kv = torch.zeros(2, 4, 16, 2, 16, device=dev)
    bt = torch.tensor([[0, 1, 2]], dtype=torch.int32, device=dev)
    seq = torch.tensor([40], dtype=torch.int32, device=dev)
    with pytest.raises(ValueError, match="wide"):
        action_scores(torch.zeros(1, 4, 16, device=dev), kv, bt, seq, torch.zeros(1, 4, device=dev),
                      torch.zeros(1, 2, 16, device=dev), torch.zeros(1, dtype=torch.int32, device=dev))


REGION_CASES = {
    # name: (build_sessions kwargs, paths)
    "bf16_g4_two_sessions": (dict(seed=77, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[300, 517],
                                  act_lens=[24, 37], dtype="bfloat16", extra_blocks=5, channel_scale=True),
                             ("simt", "tcgen05", "pair")),
    "bf16_g8_streamed_q": (dict(seed=3, n_layers=2, hq=16, hkv=2, d=128, bs=16, seq_lens=[700, 1500],
                                act_lens=[100, 70], dtype="bfloat16", extra_blocks=3), ("simt", "tcgen05", "pair")),
    "bf16_g1_resident_two_chunks": (dict(seed=4, n_layers=1, hq=2, hkv=2, d=128, bs=16, seq_lens=[900],
                                         act_lens=[300], dtype="bfloat16", extra_blocks=2), ("simt", "tcgen05", "pair")),
    "fp16_g2_ragged": (dict(seed=5, n_layers=2, hq=4, hkv=2, d=128, bs=16, seq_lens=[333, 129, 17],
                            act_lens=[200, 64, 3], dtype="float16", extra_blocks=4), ("simt", "tcgen05", "pair")),
    "bf16_g16_streamed": (dict(seed=6, n_layers=1, hq=32, hkv=2, d=128, bs=16, seq_lens=[400],
                               act_lens=[40], dtype="bfloat16", extra_blocks=1), ("simt", "tcgen05", "pair")),
    "bf16_bs8": (dict(seed=8, n_layers=1, hq=8, hkv=2, d=128, bs=8, seq_lens=[250, 64],
                      act_lens=[20, 9], dtype="bfloat16", extra_blocks=3), ("simt", "tcgen05", "pair")),
    "fp32_d64_g3": (dict(seed=9, n_layers=2, hq=6, hkv=2, d=64, bs=16, seq_lens=[210, 50],
                         act_lens=[11, 5], dtype="float32", extra_blocks=2), ("simt",)),
    # a session without action tokens between two with: its units have nothing to fold
    "bf16_zero_action_session": (dict(seed=12, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[300, 650, 200],
                                      act_lens=[24, 0, 37], dtype="bfloat16", extra_blocks=3),
                                 ("simt", "tcgen05", "pair")),
    # regions wider than the CTA-pair kernel's four query slots (A*G = 2400: ten chunks in three
    # groups; 1040: five chunks in two) folded over blocks of consecutive tiles, next to a resident
    # region and one without action tokens in the same call (each width class on its own launch)
    "bf16_g8_pair_wide_groups": (dict(seed=16, n_layers=3, hq=16, hkv=2, d=128, bs=16,
                                      seq_lens=[5000, 1900, 700, 300], act_lens=[300, 130, 0, 20],
                                      dtype="bfloat16", extra_blocks=4), ("tcgen05", "pair")),
    # one region of each width class in one call (A*G = 160, 800, 1120, 0): the CTA-pair kernel
    # scores each class on its own launch (two query slots, four slots, the block path)
    "bf16_g8_three_width_classes": (dict(seed=17, n_layers=2, hq=16, hkv=2, d=128, bs=16,
                                         seq_lens=[900, 1300, 1700, 400], act_lens=[20, 100, 140, 0],
                                         dtype="bfloat16", extra_blocks=4), ("tcgen05", "pair")),
    # more units than CTAs: a wide region (4 query chunks) folded over blocks of consecutive tiles
    # that CTA boundaries cut, next to a one-chunk session and one without action tokens in the
    # same launch
    "bf16_g8_wide_blocks_mixed": (dict(seed=14, n_layers=4, hq=16, hkv=2, d=128, bs=16,
                                       seq_lens=[4000, 2500, 1100], act_lens=[100, 30, 0], dtype="bfloat16",
                                       extra_blocks=4), ("simt", "tcgen05", "pair")),
}


def _region_on_gpu(case, lse_list, dev, path, out_init=None, n_seen=None):
    from actkv_open_b200.kernels.lse_attn import action_scores_region
    q, lse, off = packed_region(case, lse_list, dev)
    kv = case.kv.to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    W = bt.shape[1] * case.bs
    out = torch.zeros(len(case.seq_lens), case.n_layers, case.hkv, W, device=dev) if out_init is None else out_init
    action_scores_region(q, lse, off, kv, bt, seq, out, path=path, n_seen=n_seen)
    return out


@pytest.mark.parametrize("name", list(REGION_CASES))
def test_region_scores_match_oracle(name):
    dev = need_gpu()
    spec, paths = REGION_CASES[name]
    case = cases.build_sessions(**spec)
    lse = oracle_lse(case)
    want = oracle_heads(case, lse)
    for path in paths:
        out = _region_on_gpu(case, lse, dev, path).cpu().numpy()
        for r, n in enumerate(case.seq_lens):
            np.testing.assert_allclose(out[r, :, :, :n], want[r], rtol=RTOL, atol=ATOL,
                                       err_msg=f"{name} path={path} session {r}")
            assert not out[r, :, :, n:].any(), "tokens past seq_used must stay untouched"
    assert_device_clean(dev)


def test_region_matches_reference_pipeline_golden(golden):
    """The region kernel reproduces the reference's per-token action_scores loop (golden heads)."""
    dev = need_gpu()
    g = golden("pipe_bf16.npz")
    case = cases.build_sessions(**cases.PIPE_BF16)
    lse = [g[f"lse_{r}"] for r in range(len(case.seq_lens))]
    for path in ("tcgen05", "pair", "simt"):
        out = _region_on_gpu(case, lse, dev, path).cpu().numpy()
        for r, n in enumerate(case.seq_lens):
            np.testing.assert_allclose(out[r, :, :, :n], g[f"heads_{r}"], rtol=RTOL, atol=ATOL)
    assert_device_clean(dev)


def test_region_equals_sequential_single_token_calls():
    """Fusing the region is the same as the reference's one-token-per-call sequence, run on GPU."""
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import action_scores
    spec = dict(seed=21, n_layers=1, hq=8, hkv=2, d=128, bs=16, seq_lens=[260], act_lens=[33],
                dtype="bfloat16", extra_blocks=1)
    case = cases.build_sessions(**spec)
    lse = oracle_lse(case)
    fused = _region_on_gpu(case, lse, dev, "tcgen05")[0, 0]
    kv = case.kv[0].to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    out = torch.zeros(1, 2, bt.shape[1] * 16, device=dev)
    ns = torch.zeros(1, dtype=torch.int32, device=dev)
    n, a = 260, 33
    for j in range(a):
        seq = torch.tensor([n - a + j + 1], dtype=torch.int32, device=dev)
        action_scores(case.q[0][0, j][None].to(dev), kv, bt, seq,
                      torch.from_numpy(lse[0][0, j][None]).to(dev), out, ns)
    torch.testing.assert_close(fused, out[0], rtol=RTOL, atol=1e-9)
    assert int(ns.item()) == a
    assert_device_clean(dev)


@pytest.mark.parametrize("path", ["simt", "tcgen05", "pair"])
def test_region_continues_a_running_mean(path):
    """With n_seen the region folds into an existing running mean, as further one-token calls would."""
    dev = need_gpu()
    from oracle import actkv_oracle as O
    spec = dict(seed=31, n_layers=1, hq=8, hkv=2, d=128, bs=16, seq_lens=[200], act_lens=[24],
                dtype="bfloat16", extra_blocks=1)
    case = cases.build_sessions(**spec)
    lse = oracle_lse(case)
    W = 13 * 16
    prior = np.random.default_rng(0).random((2, W)).astype(np.float32) * 1e-2
    prior[:, 200:] = 0
    want = O.action_scores_region(cases.to_np(case.q[0][0]), cases.to_np(case.kv[0]),
                                  np.asarray(case.tables[0]), 200, lse[0][0], out_row=prior, n_seen0=5)
    out0 = torch.from_numpy(prior).view(1, 1, 2, W).to(dev).contiguous()
    ns = torch.tensor([5], dtype=torch.int32, device=dev)
    got = _region_on_gpu(case, lse, dev, path, out_init=out0, n_seen=ns)
    np.testing.assert_allclose(got[0, 0].cpu().numpy(), want, rtol=RTOL, atol=1e-9)
    assert int(ns.item()) == 5 + 24
    assert_device_clean(dev)


@pytest.mark.parametrize("path", ["simt", "tcgen05", "pair"])
def test_region_without_action_tokens_writes_a_zero_mean(path):
    """A session with an empty action region gets the mean of nothing (0, from a zeroed output, as
    fresh scores are defined) on every token it holds; tokens past seq_used stay untouched."""
    dev = need_gpu()
    spec, _ = REGION_CASES["bf16_zero_action_session"]
    case = cases.build_sessions(**spec)
    lse = oracle_lse(case)
    want = oracle_heads(case, lse)
    W = cases.block_table_array(case.tables).shape[1] * case.bs
    out = torch.full((len(case.seq_lens), case.n_layers, case.hkv, W), 7.0, device=dev)
    got = _region_on_gpu(case, lse, dev, path, out_init=out).cpu().numpy()
    for r, n in enumerate(case.seq_lens):
        np.testing.assert_allclose(got[r, :, :, :n], want[r], rtol=RTOL, atol=ATOL, err_msg=f"session {r}")
        assert (got[r, :, :, n:] == 7.0).all()
    assert (got[1, :, :, :case.seq_lens[1]] == 0).all()
    assert_device_clean(dev)




def test_pair_path_needs_its_workspace():
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import action_scores_region
    case = cases.build_sessions(**REGION_CASES["bf16_g4_two_sessions"][0])
    lse = oracle_lse(case)
    q, lse_t, off = packed_region(case, lse, dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    out = torch.zeros(2, case.n_layers, case.hkv, bt.shape[1] * case.bs, device=dev)
    small = torch.empty(16, dtype=torch.uint8, device=dev)
    with pytest.raises(RuntimeError, match="workspace"):
        action_scores_region(q, lse_t, off, case.kv.to(dev), bt, seq, out, path="pair", workspace=small)
