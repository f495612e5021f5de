"""The allocation-free keep-mask entry point, actkv_keep_mask_static, called through the C ABI.

It exists for callers that cannot allocate device memory (a host runtime without its own device
allocator, a serving engine whose pool is fully carved up, a plugin whose host forbids cudaMalloc
while serving): its scratch is a static array inside the library instead of a caller workspace.
Here it must give the same keep masks and kept counts as actkv_keep_mask (selection is exact, so
the comparison is bit for bit) on two different calls in a row, and refuse a batch larger than its
static scratch.  This file is collected last so a stop-at-first-failure run has already run every
other test; it also passes on its own in a fresh process."""
import numpy as np
import pytest
import torch

from gpu_util import assert_device_clean, need_gpu

pytestmark = pytest.mark.gpu


def _call(lib, N, fn_name, scores, pinned, seq, budget, n_lead, n_red, reduce, keep, kept, dev, ws=None):
    R, W = keep.shape
    args = [scores.data_ptr(), None, scores.stride(0), scores.stride(1) if n_lead > 1 else 0,
            scores.stride(-2) if n_red > 1 else 0, n_lead, n_red, reduce,
            pinned.data_ptr(), pinned.stride(0), 2, seq.data_ptr(), budget.data_ptr(), 1,
            keep.data_ptr(), keep.stride(0), kept.data_ptr(), R, W]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    args += [N.status_word(dev).data_ptr(), N.stream_ptr(dev)]
    N.check(getattr(lib, fn_name)(*args), fn_name)


@pytest.mark.parametrize("order", ["static_first", "workspace_first"])
def test_static_scratch_keep_mask_matches_the_workspace_entry_point(order):
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    lib = N.load()
    gen = torch.Generator().manual_seed(7)
    calls = [  # (R, n_lead, n_red, W, reduce): two calls in a row with different shapes
        (3, 4, 8, 5000, N.REDUCE_MEAN),
        (2, 1, 36, 32768, N.REDUCE_MAX),
    ]
    for R, n_lead, n_red, W, reduce in calls:
        scores = torch.rand(R, n_lead, n_red, W, generator=gen).to(dev)
        seq = torch.tensor([W - 17 * r for r in range(R)], dtype=torch.int32, device=dev)
        budget = torch.tensor([W // 5 + r for r in range(R)], dtype=torch.int32, device=dev)
        pinned = (torch.rand(R, W, generator=gen) < 0.02).to(torch.uint8).to(dev)
        outs = {}
        names = ["actkv_keep_mask_static", "actkv_keep_mask"]
        if order == "workspace_first":
            names.reverse()
        for name in names:
            keep = torch.full((R, W), 7, dtype=torch.uint8, device=dev)
            kept = torch.full((R,), -1, dtype=torch.int32, device=dev)
            ws = None
            if name == "actkv_keep_mask":
                ws = N.workspace(lib.actkv_keep_mask_workspace_bytes(R, W), dev)
            _call(lib, N, name, scores, pinned, seq, budget, n_lead, n_red, reduce, keep, kept, dev, ws)
            torch.cuda.synchronize(dev)
            outs[name] = (keep.cpu().numpy(), kept.cpu().numpy())
        (k_s, n_s), (k_w, n_w) = outs["actkv_keep_mask_static"], outs["actkv_keep_mask"]
        for r in range(R):
            n = int(seq[r])
            np.testing.assert_array_equal(k_s[r, :n], k_w[r, :n], err_msg=f"R={R} W={W} session {r}")
        np.testing.assert_array_equal(n_s, n_w)
        pin = pinned.cpu().numpy().astype(bool)
        for r in range(R):                     # protected = first 2 tokens or pinned, plus the budget
            n = int(seq[r])
            prot = pin[r, :n] | (np.arange(n) < 2)
            assert n_s[r] == prot.sum() + int(budget[r])
    assert_device_clean(dev)


def test_static_scratch_refuses_a_batch_larger_than_its_array():
    dev = need_gpu()
    from actkv_open_b200 import _native as N
    lib = N.load()
    R, W = 33, 32768                       # 33 * 32768 floats > the 2^20-float static array
    scores = torch.zeros(R, W, device=dev)
    keep = torch.zeros(R, W, dtype=torch.uint8, device=dev)
    seq = torch.full((R,), W, dtype=torch.int32, device=dev)
    code = lib.actkv_keep_mask_static(scores.data_ptr(), None, W, 0, 0, 1, 1, N.REDUCE_MEAN, None, 0, 0,
                                      seq.data_ptr(), seq.data_ptr(), 0, keep.data_ptr(), W, None, R, W,
                                      N.status_word(dev).data_ptr(), N.stream_ptr(dev))
    assert code == -6
    assert "static scratch" in lib.actkv_last_error().decode()
    with pytest.raises(RuntimeError, match="static scratch"):
        N.check(code)
    assert not keep.any()                  # nothing was launched
    assert_device_clean(dev)
