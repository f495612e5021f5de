"""ctypes binding of the C ABI in include/actkv_b200.h (libactkv_b200.so, built in-tree by
actkv_open_b200/build.py).

Status codes become the exception types the reference raises for the same conditions
(actkv/kernels/lse_attn.py:139-149, actkv/kernels/compaction.py:61,102, actkv/paged.py:32-33).
There is no CPU path: every operation requires CUDA tensors and raises if the library or a GPU is
missing.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_native", "libactkv_b200.so")

F32, F16, BF16 = 0, 1, 2
REDUCE_MEAN, REDUCE_MAX = 0, 1
PATH_AUTO, PATH_SIMT, PATH_TCGEN05, PATH_PAIR = 0, 1, 2, 3
DEV_BAD_INDEX, DEV_TIMEOUT, DEV_MISALIGNED, DEV_OUT_OF_BLOCKS = 1, 2, 4, 8

_DTYPES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

P, I32, I64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
F64 = ctypes.c_double
U32 = ctypes.c_uint32

# name -> (restype, argtypes); must match include/actkv_b200.h
SIGNATURES = {
    "actkv_last_error": (ctypes.c_char_p, []),
    "actkv_abi_version": (I32, []),
    "actkv_action_scores": (I32, [P, I32, I64, I64, P, I32, I64, I64, I64, I64, P, I64, P, P, I64, P, I64,
                                  I64, I64, P, I32, I32, I32, I32, I32, I32, I32, F, P, P]),
    "actkv_score_region": (I32, [P, I32, I64, I64, I64, P, I64, I64, P, P, I32, I64, I64, I64, I64, I64, P,
                                 I64, P, P, P, I64, I64, I64, P, I32, I32, I32, I32, I32, I32, I32, I32, I32,
                                 I32, F, I32, P, SZ, P, P]),
    "actkv_score_region_streamed": (I32, [P, I32, I64, I64, I64, P, I64, I64, P, P, I32, I64, I64, I64, I64, I64,
                                          P, I64, P, P, P, I64, I64, I64, P, I32, I32, I32, I32, I32, I32, I32,
                                          I32, I32, I32, F, I32, P, SZ, P, U32, I32, P, P, P]),
    "actkv_stream_signal": (I32, [P, U32, P]),
    "actkv_stream_copy_groups": (I32, [P, P, SZ, P, I32, I32, P, U32, P]),
    "actkv_score_region_workspace_bytes": (SZ, [I32, I32, I32]),
    "actkv_lrfu_update": (I32, [P, P, I64, I64, I64, I32, I32, P, I64, I64, P, I64, I64, P, I64, I32, P, P,
                                I32, I32, I32, F, F, P, P]),
    "actkv_keep_mask_workspace_bytes": (SZ, [I32, I32]),
    "actkv_keep_mask": (I32, [P, P, I64, I64, I64, I32, I32, I32, P, I64, I32, P, P, I32, P, I64, P, I32, I32,
                              P, SZ, P, P]),
    "actkv_keep_mask_static": (I32, [P, P, I64, I64, I64, I32, I32, I32, P, I64, I32, P, P, I32, P, I64, P, I32,
                                     I32, P, P]),
    "actkv_compact_workspace_bytes": (SZ, [I32, I32]),
    "actkv_compact": (I32, [P, I32, I64, I64, I64, I64, P, I64, P, P, I64, I32, I32, P, P, I64, P, I64, P,
                            I32, I32, P, SZ, P, P]),
    "actkv_plan_workspace_bytes": (SZ, [I32]),
    "actkv_plan_compaction": (I32, [P, I32, P, I32, I32, P, P, P, P, P, SZ, P, P]),
    "actkv_apply_copies": (I32, [P, I32, I64, I64, I64, I64, P, P, I64, P, P]),
    "actkv_permute_tokens": (I32, [P, P, I64, I64, I32, P, P, I64, P, I64, P, I32, I32, P, P]),
    "actkv_add_i32": (I32, [P, P, I32, P]),
    "actkv_blocks_workspace_bytes": (SZ, [I32]),
    "actkv_append": (I32, [P, I32, I64, I64, I64, I64, P, P, I64, I64, P, I32, P, P, I64, I32, I32, P, P, I64,
                           I32, P, SZ, P, P]),
    "actkv_release": (I32, [P, P, P, I64, I32, I32, P, P, I64, P, I64, I32, I32, P, SZ, P, P]),
    "actkv_region_lse_workspace_bytes": (SZ, [I32, I32, I32, I64]),
    "actkv_region_lse": (I32, [P, I32, I64, I64, I64, P, P, I32, I64, I64, I64, I64, I64, P, I64, P, P, I64, I64,
                               I32, I32, I32, I32, I32, I32, I32, I32, I32, I64, F, P, SZ, P, P]),
    "actkv_token_confidence": (I32, [P, I32, I64, I32, I32, I32, P, P, I64, P, P, P]),
    "actkv_budget_update": (I32, [P, I64, P, I32, I32, I32, F64, F64, I32, I32, I32, F64, F64, I32, P, I32, P, P, P,
                                  P, P, P]),
    "actkv_streaming_keep": (I32, [P, I64, I32, I32, I32, I32, P]),
    "actkv_snapkv_workspace_bytes": (SZ, [I32, I32]),
    "actkv_snapkv_select": (I32, [P, I64, I64, P, I64, P, I32, I32, I32, I32, I32, I32, I32, P, I64, P, SZ, P, P]),
    "actkv_snapkv_compact_rows": (I32, [P, P, I64, I64, P, I64, P, I32, I32, P, I64, I32, P, P]),
    "actkv_selftest_bounded_wait": (I32, [P, P, P]),
    "actkv_measure_kv_gather": (I32, [P, I64, I32, I32, I32, I32, P, P]),
    "actkv_decode_workspace_bytes": (SZ, [I32, I32, I32, I32, I64]),
    "actkv_decode_attention": (I32, [P, I32, I64, I64, P, I64, I64, I64, I64, P, I64, P, P, I64, I64, P, I64,
                                     I32, I32, I32, I32, I32, I32, I32, F, P, SZ, P, P]),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _LIB_PATH


def load():
    """Load the native library (building it first if it is missing and nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                from . import build as _build
                _build.build()
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class OutOfBlocks(RuntimeError):
    """The allocator has fewer free blocks than a request needs (actkv/paged.py:19)."""


def check(code: int, what: str = "") -> None:
    if code == 0:
        return
    msg = load().actkv_last_error().decode(errors="replace")
    msg = f"{what}: {msg}" if what else msg
    if code in (-2, -7):                      # out too narrow, bad head_reduce
        raise ValueError(msg)
    if code in (-1, -5):                      # the reference's asserts
        raise AssertionError(msg)
    if code == -3:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise AssertionError(f"unsupported dtype {t.dtype}") from None


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("actkv_open_b200 runs its kernels on CUDA tensors only (no CPU path); "
                               f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_status = {}


def status_word(device) -> torch.Tensor:
    """A per-device int32 that kernels OR ACTKV_DEV_* bits into (never reset implicitly)."""
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    t = _status.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _status[key] = t
    return t


def read_device_status(device=None, reset: bool = True) -> int:
    """Synchronising read of the device status word: 0 when no kernel reported a problem."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    t = status_word(dev)
    v = int(t.item())
    if reset and v:
        t.zero_()
    return v


def workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
