"""The C ABI library loads on a machine without a GPU and exports exactly what the header declares,
with the argument counts the ctypes binding uses (no kernel is launched here)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "actkv_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"ACTKV_API\s+[\w\s\*]+?\b(actkv_\w+)\s*\(([^)]*)\)\s*;", src):
        args = m.group(2).strip()
        n = 0 if args in ("", "void") else args.count(",") + 1
        out[m.group(1)] = n
    return out


def test_header_declares_the_entry_points():
    decl = _declared()
    for name in ("actkv_action_scores", "actkv_score_region", "actkv_lrfu_update", "actkv_keep_mask",
                 "actkv_compact", "actkv_plan_compaction", "actkv_apply_copies", "actkv_permute_tokens"):
        assert name in decl


def test_library_builds_loads_and_exports_every_declared_symbol():
    from actkv_open_b200 import _native as N
    from actkv_open_b200 import build
    build.build()
    lib = ctypes.CDLL(N.lib_path())
    for name in _declared():
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_the_header():
    from actkv_open_b200 import _native as N
    decl = _declared()
    assert set(decl) == set(N.SIGNATURES)
    for name, n in decl.items():
        assert len(N.SIGNATURES[name][1]) == n, name


def test_host_only_queries_work_without_a_gpu():
    from actkv_open_b200 import _native as N
    lib = N.load()
    assert lib.actkv_abi_version() == 2
    assert lib.actkv_keep_mask_workspace_bytes(2, 1000) >= 2 * 1000 * 4
    assert lib.actkv_compact_workspace_bytes(3, 100) >= 3 * 100 * 20
    assert lib.actkv_plan_workspace_bytes(100) >= 400


def test_argument_errors_are_reported_before_any_launch():
    """Host validation: the reference's ValueError / assert cases come back as status codes."""
    from actkv_open_b200 import _native as N
    lib = N.load()
    # out narrower than the block table (lse_attn.py:139-142): ValueError
    code = lib.actkv_action_scores(None, 0, 0, 0, None, 0, 0, 0, 0, 0, None, 0, None, None, 0, None, 0, 0,
                                   16, None, 1, 3, 8, 16, 4, 2, 16, 1.0, None, None)
    assert code == -2
    with pytest.raises(ValueError, match="wide"):
        N.check(code)
    # Hq not a multiple of Hkv: AssertionError, as the reference's assert
    code = lib.actkv_action_scores(None, 0, 0, 0, None, 0, 0, 0, 0, 0, None, 0, None, None, 0, None, 0, 0,
                                   48, None, 1, 3, 8, 16, 5, 2, 16, 1.0, None, None)
    with pytest.raises(AssertionError):
        N.check(code)
    # head_reduce outside {mean, max}: ValueError (paged.py:32-33)
    code = lib.actkv_keep_mask(None, None, 0, 0, 0, 1, 1, 7, None, 0, 0, None, None, 0, None, 0, None, 1, 10,
                               None, 0, None, None)
    with pytest.raises(ValueError):
        N.check(code)
    # workspace too small
    code = lib.actkv_compact(None, 2, 0, 0, 16, 16, None, 0, None, None, 0, 1, 16, None, None, 0, None, 0,
                             None, 1, 100, None, 0, None, None)
    assert code == -1            # free list missing is checked first
    # zero sessions is a no-op that succeeds without touching the device
    assert lib.actkv_apply_copies(None, 4, 0, 0, 16, 10, None, None, 0, None, None) == 0


def test_kernels_refuse_cpu_tensors():
    import torch
    from actkv_open_b200.kernels.lse_attn import action_scores
    q = torch.zeros(1, 2, 16)
    kv = torch.zeros(2, 4, 16, 2, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        action_scores(q, kv, torch.zeros(1, 1, dtype=torch.int32), torch.ones(1, dtype=torch.int32),
                      torch.zeros(1, 2), torch.zeros(1, 2, 16), torch.zeros(1, dtype=torch.int32))
