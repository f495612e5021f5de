"""Paged decode attention with its lse on the GPU (paged_decode_attention -> C
actkv_decode_attention) against the (out, lse) the reference's paged_decode_attention_ref
produced (tests/golden/decode.npz) and the CPU oracle; PagedKVCache.decode_attention uses it."""
import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_device_clean, need_gpu
from oracle import actkv_oracle as O

pytestmark = pytest.mark.gpu

# fp32 sums of products of the cache's values in a different order, ex2.approx per term
RTOL, ATOL = 1e-5, 2e-5


def _run(case, dev, **kw):
    from actkv_open_b200.kernels.lse_attn import paged_decode_attention
    q = torch.cat([qq[0] for qq in case.q], 0).to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    return paged_decode_attention(q, case.kv[0].to(dev), bt, seq, **kw)


def test_decode_attention_matches_reference_golden(golden):
    dev = need_gpu()
    g = golden("decode.npz")
    for c, spec in enumerate(g["meta"]["cases"]):
        case = cases.build_sessions(**spec)
        assert cases.digest(case.kv) == str(g[f"kv_sha_{c}"])
        out, lse = _run(case, dev)
        np.testing.assert_allclose(lse.cpu().numpy(), g[f"lse_{c}"], rtol=RTOL, atol=ATOL, err_msg=f"case {c} lse")
        np.testing.assert_allclose(out.cpu().numpy(), g[f"out_{c}"], rtol=1e-4, atol=ATOL, err_msg=f"case {c} out")
    assert_device_clean(dev)


@pytest.mark.parametrize("spec", [
    dict(seed=61, n_layers=1, hq=16, hkv=2, d=128, bs=16, seq_lens=[33000, 5, 700], act_lens=[1, 1, 1],
         dtype="bfloat16", extra_blocks=3),
    dict(seed=62, n_layers=1, hq=4, hkv=2, d=64, bs=32, seq_lens=[129, 1000], act_lens=[1, 1],
         dtype="float16", extra_blocks=2),
    dict(seed=65, n_layers=1, hq=4, hkv=2, d=128, bs=16, seq_lens=[3000, 17, 250], act_lens=[1, 1, 1],
         dtype="float32", extra_blocks=2),
    # 40 sessions x 8 KV heads (bf16, head_dim 128: the tensor-core kernel, one CTA per SM): more
    # (session, head) pairs than one wave of CTAs, so one split each (asserted in the test)
    dict(seed=67, n_layers=1, hq=8, hkv=8, d=128, bs=16,
         seq_lens=[int(x) for x in np.random.default_rng(67).integers(1, 400, 40)], act_lens=[1] * 40,
         dtype="bfloat16", extra_blocks=4),
    # config 2's head layout (32 query heads over 8 KV heads), partial last tiles
    dict(seed=68, n_layers=1, hq=32, hkv=8, d=128, bs=16, seq_lens=[5000, 9, 130], act_lens=[1, 1, 1],
         dtype="bfloat16", extra_blocks=3),
    # block size 8 (16 paged blocks per 128-token tile), fp16
    dict(seed=69, n_layers=1, hq=16, hkv=4, d=128, bs=8, seq_lens=[777, 32, 1], act_lens=[1, 1, 1],
         dtype="float16", extra_blocks=3),
    # 64 query heads (G = 8 over 8 KV heads), and a single KV head
    dict(seed=70, n_layers=1, hq=64, hkv=8, d=128, bs=16, seq_lens=[1500, 40], act_lens=[1, 1],
         dtype="bfloat16", extra_blocks=2),
    dict(seed=71, n_layers=1, hq=4, hkv=1, d=128, bs=16, seq_lens=[600, 3], act_lens=[1, 1],
         dtype="bfloat16", extra_blocks=2),
])
def test_decode_attention_matches_the_oracle(spec):
    """Long sessions (many token splits) next to very short ones; G = 8, 2 and 2 with fp32 rows of
    D = 128; many short sessions with G = 1 (one split per session and head); config 2's head layout;
    block size 8; G = 8 over 8 KV heads; one KV head.  bf16 / fp16 with head_dim 128 run the
    tensor-core kernel, fp32 and head_dim 64 the CUDA-core kernel."""
    dev = need_gpu()
    case = cases.build_sessions(**spec)
    if len(case.seq_lens) == 40:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        assert len(case.seq_lens) * case.hkv > sms, "the case must overflow one wave of one-CTA-per-SM splits"
    q = torch.cat([qq[0] for qq in case.q], 0)
    want_o, want_l = O.paged_decode_attention(q.float().numpy(), cases.to_np(case.kv)[0],
                                              cases.block_table_array(case.tables).astype(np.int64), case.seq_lens)
    out, lse = _run(case, dev)
    np.testing.assert_allclose(lse.cpu().numpy(), want_l, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(out.cpu().numpy(), want_o, rtol=1e-4, atol=ATOL)
    assert_device_clean(dev)


def test_paged_cache_decode_attention_uses_the_kernel():
    dev = need_gpu()
    from actkv_open_b200.paged import PagedKVCache
    case = cases.build_sessions(seed=63, n_layers=2, hq=8, hkv=2, d=128, bs=16, seq_lens=[90, 300],
                                act_lens=[1, 1], dtype="bfloat16", extra_blocks=2)
    c = PagedKVCache(case.num_blocks, case.bs, case.hkv, case.d, n_layers=2, dtype=torch.bfloat16, device=dev)
    c.kv.copy_(case.kv.to(dev))
    c.free = list(case.free)
    for r, (t, n) in enumerate(zip(case.tables, case.seq_lens)):
        c.tables[r] = list(t)
        c.seq_used[r] = n
    q = torch.cat([qq[1] for qq in case.q], 0).to(dev)       # layer 1's query of each session
    out, lse = c.decode_attention([0, 1], q, layer=1)
    want_o, want_l = O.paged_decode_attention(q.float().cpu().numpy(), cases.to_np(case.kv)[1],
                                              cases.block_table_array(case.tables).astype(np.int64), case.seq_lens)
    np.testing.assert_allclose(lse.cpu().numpy(), want_l, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(out.cpu().numpy(), want_o, rtol=1e-4, atol=ATOL)
    with pytest.raises(NotImplementedError):             # G = 16 has no kernel
        case16 = cases.build_sessions(seed=64, n_layers=1, hq=32, hkv=2, d=128, bs=16, seq_lens=[50], act_lens=[1],
                                      dtype="bfloat16", extra_blocks=1)
        _run(case16, dev)
    assert_device_clean(dev)


def test_decode_attention_rejects_rows_off_the_vector_alignment():
    """Each lane reads its slice of a K / V row as one vector: a cache view starting one element
    past an aligned address is refused, not read with misaligned loads."""
    dev = need_gpu()
    from actkv_open_b200.kernels.lse_attn import paged_decode_attention
    case = cases.build_sessions(seed=66, n_layers=1, hq=8, hkv=2, d=128, bs=16, seq_lens=[100], act_lens=[1],
                                dtype="bfloat16", extra_blocks=1)
    kv = case.kv[0].to(dev)
    flat = torch.empty(kv.numel() + 8, dtype=kv.dtype, device=dev)
    shifted = flat[1:1 + kv.numel()].view(kv.shape)
    shifted.copy_(kv)
    q = case.q[0][0].to(dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    seq = torch.tensor(case.seq_lens, dtype=torch.int32, device=dev)
    with pytest.raises(NotImplementedError, match="aligned"):
        paged_decode_attention(q, shifted, bt, seq)
    out, lse = paged_decode_attention(q, kv, bt, seq)
    assert torch.isfinite(lse).all()
    assert_device_clean(dev)
