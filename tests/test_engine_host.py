"""Host-side layer grouping of EvictionPipeline.step_host (no GPU): the streamed groups (one
scoring launch, at most 16 groups, the first of one layer) and the grouped launches' growing
groups must partition the layers in order."""
import pytest

from actkv_open_b200.engine import _growing_groups, _stream_groups


def _partition(b, L):
    assert b[0] == 0 and b[-1] == L
    assert all(x < y for x, y in zip(b, b[1:]))


@pytest.mark.parametrize("L", [1, 2, 3, 7, 16, 17, 36, 80, 200])
def test_stream_groups_partition(L):
    b = _stream_groups(L)
    _partition(b, L)
    assert len(b) - 1 <= 16                      # the kernel's limit on layer groups
    assert b[1] == 1                             # the one copy nothing hides is a single layer
    sizes = [y - x for x, y in zip(b[1:], b[2:])]
    if sizes:
        assert max(sizes) - min(sizes) <= 1      # the rest in near-equal groups


@pytest.mark.parametrize("L,n", [(1, 4), (2, 4), (36, 4), (36, 1), (80, 6), (5, 9)])
def test_growing_groups_partition(L, n):
    b = _growing_groups(L, n)
    _partition(b, L)
    assert len(b) - 1 == min(n, L)
    sizes = [y - x for x, y in zip(b, b[1:])]
    assert sizes == sorted(sizes) or L < 2 * n   # growing, up to rounding of tiny cases
