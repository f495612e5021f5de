"""Failure detection on the GPU without a fault: a kernel whose bounded mbarrier wait (the helper
every TMA / MMA / epilogue role of the tcgen05 kernels uses) is never satisfied gives up after
~2^31 cycles, reports ACTKV_DEV_TIMEOUT in the status word and returns; the context then runs
the scoring kernel normally."""
import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_device_clean, need_gpu, oracle_heads, oracle_lse, packed_region

pytestmark = pytest.mark.gpu


def test_a_stalled_wait_reports_a_timeout_and_the_context_stays_usable():
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    from actkv_open_b200.kernels.lse_attn import action_scores_region
    assert_device_clean(dev)
    waited = torch.zeros(1, dtype=torch.int64, device=dev)
    N.check(N.load().actkv_selftest_bounded_wait(N.status_word(dev).data_ptr(), waited.data_ptr(),
                                                 N.stream_ptr(dev)), "selftest")
    torch.cuda.synchronize(dev)
    assert int(waited.item()) >= 1 << 31                    # it waited its whole bound, then gave up
    assert N.read_device_status(dev) & N.DEV_TIMEOUT         # reported, and the word is reset here
    # the same context scores correctly afterwards
    case = cases.build_sessions(seed=77, n_layers=1, hq=8, hkv=2, d=128, bs=16, seq_lens=[300],
                                act_lens=[24], dtype="bfloat16", extra_blocks=2)
    lse = oracle_lse(case)
    q, lse_d, off = packed_region(case, lse, dev)
    bt = torch.from_numpy(cases.block_table_array(case.tables)).to(dev)
    out = torch.zeros(1, 1, case.hkv, bt.shape[1] * case.bs, device=dev)
    action_scores_region(q, lse_d, off, case.kv.to(dev), bt, torch.tensor([300], dtype=torch.int32, device=dev),
                         out, path="tcgen05")
    np.testing.assert_allclose(out.cpu().numpy()[0, :, :, :300], oracle_heads(case, lse)[0], rtol=2e-3, atol=1e-6)
    assert_device_clean(dev)


def test_kv_gather_measurement_reads_the_cache_in_both_patterns():
    """actkv_measure_kv_gather (a timing aid): both read patterns run on a paged cache, leave it and
    the status word untouched, and reject sizes it cannot sweep."""
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    kv = torch.randn(2, 2, 64, 16, 8, 128, device=dev).to(torch.bfloat16)
    before = kv.clone()
    sink = torch.zeros(1, dtype=torch.int64, device=dev)
    lib = N.load()
    n_blocks, row_bytes, head_bytes = 2 * 2 * 64, 8 * 128 * 2, 128 * 2
    for mode in (0, 1):
        N.check(lib.actkv_measure_kv_gather(kv.data_ptr(), n_blocks, 16, row_bytes, head_bytes, mode,
                                            sink.data_ptr(), N.stream_ptr(dev)), "measure_kv_gather")
    torch.cuda.synchronize(dev)
    assert torch.equal(kv, before)
    assert lib.actkv_measure_kv_gather(kv.data_ptr(), n_blocks, 16, row_bytes, 100, 0, sink.data_ptr(),
                                       N.stream_ptr(dev)) != 0
    assert_device_clean(dev)
