"""Device-resident block allocation (DevicePagedCache.append / release -> C actkv_append /
actkv_release) against the reference's host model (PagedKVCache.append / release,
actkv/paged.py:67-90, restated in the oracle): after every operation of a sequence -- appends that
fill partial blocks, a session starting from empty, a release and the reuse of its blocks, and an
append that runs out of blocks part-way through the batch -- the block tables, lengths, free stack
and cache bytes must be identical."""
import numpy as np
import pytest
import torch

from gpu_util import assert_device_clean, need_gpu

pytestmark = pytest.mark.gpu

L, NB, BS, HKV, D = 2, 40, 16, 2, 64


def _state(cache):
    tables, seq, free = cache.state()
    return tables, seq, free, cache.kv.float().cpu().numpy()


def _check(cache, ref, R, what):
    tables, seq, free, kv = _state(cache)
    for r in range(R):
        assert tables[r] == ref.tables.get(r, []), (what, r)
        assert seq[r] == ref.seq_used.get(r, 0), (what, r)
    assert free == ref.free, what
    np.testing.assert_array_equal(kv, ref.kv, err_msg=what)


def _rows(gen, counts, dtype):
    n = sum(counts)
    k = torch.randn(L, n, HKV, D, generator=gen).to(dtype)
    v = torch.randn(L, n, HKV, D, generator=gen).to(dtype)
    return k, v


def _ref_append(ref, counts, k, v):
    """The reference's per-request loop; stops (raises) at the first request that does not fit."""
    off = 0
    for r, n in enumerate(counts):
        try:
            ref.append(r, k[:, off:off + n].float().numpy(), v[:, off:off + n].float().numpy())
        except Exception as e:                 # OutOfBlocks
            return type(e).__name__
        off += n
    return None


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_append_and_release_match_the_reference_allocator(dtype):
    dev = need_gpu()
    from actkv_open_b200._native import OutOfBlocks
    from actkv_open_b200.engine import DevicePagedCache
    from oracle import actkv_oracle as O
    R, W = 3, 640
    ref = O.PagedKVCache(NB, BS, HKV, D, L)
    cache = DevicePagedCache(NB, BS, HKV, D, L, R, W, dtype=dtype, device=dev)
    cache.set_state([[] for _ in range(R)], [0] * R, list(ref.free))
    gen = torch.Generator().manual_seed(5)
    for counts in ([37, 0, 64], [20, 50, 3], [16, 1, 15]):
        k, v = _rows(gen, counts, dtype)
        assert _ref_append(ref, counts, k, v) is None
        cache.append(k.to(dev), v.to(dev), counts)
        _check(cache, ref, R, f"append {counts}")
    ref.release(1)
    cache.release([1])
    _check(cache, ref, R, "release 1")
    assert not cache.pinned[1].any()
    k, v = _rows(gen, [100, 5, 16], dtype)
    assert _ref_append(ref, [100, 5, 16], k, v) is None
    cache.append(k.to(dev), v.to(dev), [100, 5, 16])
    _check(cache, ref, R, "append after release")
    # session 0 fits, session 1 does not: the reference appends 0 and raises at 1
    free_blocks = len(ref.free)
    counts = [BS * 2, BS * (free_blocks + 1), 4]
    k, v = _rows(gen, counts, dtype)
    assert _ref_append(ref, counts, k, v) == "OutOfBlocks"
    with pytest.raises(OutOfBlocks):
        cache.append(k.to(dev), v.to(dev), counts)
    _check(cache, ref, R, "out of blocks")
    for r in (0, 2):                            # a batched release runs in session order
        ref.release(r)
    cache.release([2, 0])
    _check(cache, ref, R, "release 0 and 2")
    assert_device_clean(dev)


def test_append_with_device_offsets_and_a_new_session():
    """Offsets given as a device tensor (no host involvement) and a fourth session that starts
    empty: same tables / free stack as the reference."""
    dev = need_gpu()
    from actkv_open_b200.engine import DevicePagedCache
    from oracle import actkv_oracle as O
    ref = O.PagedKVCache(NB, BS, HKV, D, L)
    cache = DevicePagedCache(NB, BS, HKV, D, L, 4, 512, dtype=torch.bfloat16, device=dev)
    cache.set_state([[], []], [0, 0], list(ref.free))
    gen = torch.Generator().manual_seed(9)
    counts = [33, 7, 0, 48]
    k, v = _rows(gen, counts, torch.bfloat16)
    assert _ref_append(ref, counts, k, v) is None
    off = torch.tensor(np.concatenate([[0], np.cumsum(counts)]), dtype=torch.int32, device=dev)
    cache.append(k.to(dev), v.to(dev), off, max_new=max(counts), check=False)
    assert cache.n_sessions == 4
    _check(cache, ref, 4, "device offsets")
    assert_device_clean(dev)
