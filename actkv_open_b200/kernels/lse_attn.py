"""Drop-in for ``actkv.kernels.lse_attn`` (actkv/kernels/lse_attn.py): LSE-recovery scoring on a
paged KV cache (ActKV Algorithm 3), on hand-written sm_100a kernels.

Paged attention returns the softmax log-sum-exp per (query, head) but not the attention matrix;
since A_ij = exp(s_ij - LSE_i), a token's attention is recovered by recomputing q.k inside its
paged block.  Layout (vLLM, one layer): kv [2, NB, BS, Hkv, D], block_table [R, MB] int32,
seq_used [R] int32; out [R, Hkv, MB*BS] fp32 running mean over action tokens, n_seen [R] int32.

``action_scores`` keeps the reference's signature and semantics (lse_attn.py:133-163) and runs the
CUDA-core scoring kernel through the C ABI; ``action_scores_region`` (new) folds a whole causal
action region of every layer in one launch and uses the tcgen05 tensor-core kernel for bf16/fp16
caches with head_dim 128.  ``action_region_lse`` (new) produces that region's causal lse from the
paged cache on the tensor cores (what the reference's ``paged_decode_attention_ref`` gives per
action token, lse_attn.py:42-60), and ``paged_decode_attention`` (new) is that decode attention
itself, output and lse, on the GPU.  ``gather_kv``, ``paged_decode_attention_ref`` and ``action_scores_ref``
are the module's torch reference helpers (lse_attn.py:32-78), kept because callers import them
(the LSE producer stand-in and test oracles); the kernels never fall back to them.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from .. import _native as N

HAS_KERNELS = os.path.exists(N.lib_path())
# Kept under the reference's name: True means action_scores runs a compiled GPU kernel rather than
# the torch reference.  Here that kernel is CUDA (sm_100a), not Triton.
HAS_TRITON = HAS_KERNELS


# ----------------------------------------------------------------------------- torch helpers

def gather_kv(kv: torch.Tensor, block_table: torch.Tensor, seq_used: int, row: int):
    """Contiguous K, V [S, Hkv, D] of request ``row`` (what a gather-based approach materialises)."""
    bs = kv.shape[2]
    blocks = block_table[row, : math.ceil(seq_used / bs)].long()
    k = kv[0].index_select(0, blocks).flatten(0, 1)[:seq_used]
    v = kv[1].index_select(0, blocks).flatten(0, 1)[:seq_used]
    return k, v


def paged_decode_attention_ref(q, kv, block_table, seq_used, scale=None):
    """Decode attention over the paged cache in fp32: (out [R, Hq, D], lse [R, Hq]).

    Stands in for the paged attention backend whose LSE by-product the scoring consumes.
    """
    r_n, hq, d = q.shape
    hkv = kv.shape[3]
    g = hq // hkv
    scale = d ** -0.5 if scale is None else scale
    out = torch.empty(r_n, hq, d, dtype=torch.float32, device=q.device)
    lse = torch.empty(r_n, hq, dtype=torch.float32, device=q.device)
    lens = [int(s) for s in seq_used.tolist()]
    for r in range(r_n):
        k, v = gather_kv(kv, block_table, lens[r], r)
        qg = q[r].float().view(hkv, g, d)
        logits = torch.matmul(qg, k.float().permute(1, 2, 0)) * scale        # [Hkv, G, S]
        lse[r] = torch.logsumexp(logits, -1).reshape(hq)
        out[r] = torch.matmul(torch.softmax(logits, -1), v.float().transpose(0, 1)).reshape(hq, d)
    return out, lse


def action_scores_ref(q, kv, block_table, seq_used, lse, out, n_seen, scale=None):
    """torch statement of action_scores (the oracle of the reference's own tests)."""
    r_n, hq, d = q.shape
    hkv = kv.shape[3]
    g = hq // hkv
    scale = d ** -0.5 if scale is None else scale
    lens = [int(s) for s in seq_used.tolist()]
    for r in range(r_n):
        s = lens[r]
        k, _ = gather_kv(kv, block_table, s, r)
        logits = torch.matmul(q[r].float().view(hkv, g, d), k.float().permute(1, 2, 0)) * scale
        p = torch.exp(logits - lse[r].view(hkv, g, 1)).amax(1)               # [Hkv, S]
        n = float(n_seen[r])
        out[r, :, :s] += (p - out[r, :, :s]) / (n + 1.0)
    n_seen += 1
    return out


# ----------------------------------------------------------------------------- CUDA kernels

def action_scores(q, kv, block_table, seq_used, lse, out, n_seen, scale=None):
    """Fold one action query token per request into ``out`` (Algorithm 3). In place; returns ``out``.

    q [R, Hq, D], kv [2, NB, BS, Hkv, D], block_table [R, MB] int32, seq_used [R] int32,
    lse [R, Hq] fp32, out [R, Hkv, MB*BS] fp32, n_seen [R] int32 (incremented here).
    Raises ValueError when ``out`` is narrower than the block table spans (lse_attn.py:139-142).
    """
    span = block_table.shape[1] * kv.shape[2]
    if out.shape[-1] < span:
        raise ValueError(f"out is {out.shape[-1]} wide but the block table spans {span} slots; "
                         "allocate it as [R, Hkv, max_blocks * block_size]")
    r_n, hq, d = q.shape
    _, nb, bs, hkv, _ = kv.shape
    assert hq % hkv == 0
    assert kv.stride(-1) == 1 and q.stride(-1) == 1
    assert out.stride(-1) == 1 and lse.stride(-1) == 1
    dev = N.require_cuda(q, kv, block_table, seq_used, lse, out, n_seen)
    assert out.dtype == torch.float32 and lse.dtype == torch.float32
    assert block_table.dtype == torch.int32 and seq_used.dtype == torch.int32 and n_seen.dtype == torch.int32
    scale = d ** -0.5 if scale is None else scale
    bt = block_table if block_table.stride(-1) == 1 else block_table.contiguous()
    lib = N.load()
    N.check(lib.actkv_action_scores(
        q.data_ptr(), N.dtype_code(q), q.stride(0), q.stride(1),
        kv.data_ptr(), N.dtype_code(kv), kv.stride(0), kv.stride(1), kv.stride(2), kv.stride(3),
        bt.data_ptr(), bt.stride(0), seq_used.contiguous().data_ptr(),
        lse.data_ptr(), lse.stride(0),
        out.data_ptr(), out.stride(0), out.stride(1), out.shape[-1],
        n_seen.data_ptr(), r_n, bt.shape[1], nb, bs, hq, hkv, d, float(scale),
        N.status_word(dev).data_ptr(), N.stream_ptr(dev)), "action_scores")
    return out


def score_region_workspace_bytes(L: int, sum_a: int, hq: int) -> int:
    """Bytes of the workspace that lets ``action_scores_region`` use the CTA-pair kernel."""
    return int(N.load().actkv_score_region_workspace_bytes(L, sum_a, hq))


def action_scores_region(q, lse, act_off, kv, block_table, seq_used, out, out_off=None, n_seen=None,
                         scale=None, path: str = "auto", max_actions: int | None = None, workspace=None,
                         streamed=None):
    """Fold each session's whole causal action region, for every layer, in one launch.

    q [L, sumA, Hq, D] and lse [L, sumA, Hq] hold the action tokens of all sessions packed along
    dim 1 (session r owns rows act_off[r]:act_off[r+1]); kv is the full cache
    [L, 2, NB, BS, Hkv, D]; out receives (r, l, h, t) at out_off[r] + l*out.stride(-3) +
    h*out.stride(-2) + t (out_off None: out is [R, L, Hkv, W]).  Action token j of a region of A
    tokens sees the first seq_used - A + j + 1 tokens, so the result equals A calls of
    ``action_scores`` from a zeroed ``out`` (or, with ``n_seen``, continues its running mean).
    ``path``: "auto" (tcgen05 when q/kv are bf16/fp16 with head_dim 128: the CTA-pair kernel for
    A*G <= 1024, else the one-CTA kernel), "simt", "tcgen05" (one CTA per tile) or "pair" (CTA
    pairs).  ``workspace``: a uint8 tensor of ``score_region_workspace_bytes`` (the pair kernel's
    lse operand rows); allocated here when None and a tensor-core path may use it.

    ``streamed``: ``(ready, base, bounds)`` -- the queries of layers [bounds[g], bounds[g+1]) are
    still being copied, and the kernel reads them once the int32 device word ``ready`` has reached
    ``base + g + 1`` (``stream_signal`` on the copy stream); one launch scores every group as it
    lands.  CTA-pair path only: NotImplementedError (nothing launched) where it does not apply.
    """
    L, sum_a, hq, d = q.shape
    _, _, nb, bs, hkv, _ = kv.shape
    assert hq % hkv == 0
    assert kv.stride(-1) == 1 and q.stride(-1) == 1 and lse.stride(-1) == 1 and out.stride(-1) == 1
    dev = N.require_cuda(q, lse, act_off, kv, block_table, seq_used, out, out_off, n_seen)
    assert lse.dtype == torch.float32 and out.dtype == torch.float32
    assert act_off.dtype == torch.int32 and seq_used.dtype == torch.int32
    r_n = seq_used.shape[0]
    if max_actions is None:
        max_actions = int((act_off[1:] - act_off[:-1]).max().item()) if r_n else 0
    scale = d ** -0.5 if scale is None else scale
    path_code = {"auto": N.PATH_AUTO, "simt": N.PATH_SIMT, "tcgen05": N.PATH_TCGEN05, "pair": N.PATH_PAIR}[path]
    if workspace is None and path in ("auto", "pair"):
        workspace = N.workspace(score_region_workspace_bytes(L, sum_a, hq), q.device)
    if out_off is None:
        assert out.dim() == 4 and out.shape[0] == r_n and out.shape[1] == L and out.shape[2] == hkv
        o_r, o_l, o_h = out.stride(0), out.stride(1), out.stride(2)
    else:
        assert out_off.dtype == torch.int64
        o_r, o_l, o_h = 0, out.stride(-3), out.stride(-2)
    lib = N.load()
    common = (q.data_ptr(), N.dtype_code(q), q.stride(0), q.stride(1), q.stride(2),
              lse.data_ptr(), lse.stride(0), lse.stride(1), act_off.data_ptr(),
              kv.data_ptr(), N.dtype_code(kv), kv.stride(0), kv.stride(1), kv.stride(2), kv.stride(3), kv.stride(4),
              block_table.data_ptr(), block_table.stride(0), seq_used.data_ptr(),
              out.data_ptr(), N.ptr(out_off), o_r, o_l, o_h, N.ptr(n_seen),
              r_n, L, block_table.shape[1], nb, bs, hq, hkv, d, sum_a, max_actions, float(scale), path_code,
              N.ptr(workspace), 0 if workspace is None else workspace.numel())
    if streamed is None:
        N.check(lib.actkv_score_region(*common, N.status_word(dev).data_ptr(), N.stream_ptr(dev)),
                "action_scores_region")
        return out
    ready, base, bounds = streamed
    assert ready.device == q.device and ready.dtype == torch.int32 and ready.numel() >= 1
    gl = (ctypes.c_int32 * len(bounds))(*bounds)
    N.check(lib.actkv_score_region_streamed(*common, ready.data_ptr(), base & 0xFFFFFFFF, len(bounds) - 1, gl,
                                            N.status_word(dev).data_ptr(), N.stream_ptr(dev)),
            "action_scores_region (streamed)")
    return out


def stream_signal(word, value: int, stream=None) -> None:
    """Stream-ordered write of ``value`` (mod 2^32) into the int32 device word ``word`` on ``stream``
    (default: the current stream), with no kernel launch: the signal ``action_scores_region``'s
    ``streamed`` groups wait for.  NotImplementedError when the driver has no stream memory ops."""
    dev = N.require_cuda(word)
    st = (stream or torch.cuda.current_stream(dev)).cuda_stream
    N.check(N.load().actkv_stream_signal(word.data_ptr(), value & 0xFFFFFFFF, st), "stream_signal")


def region_lse_workspace_bytes(L: int, sum_a: int, hq: int, max_seq: int) -> int:
    return int(N.load().actkv_region_lse_workspace_bytes(L, sum_a, hq, max_seq))


def action_region_lse(q, act_off, kv, block_table, seq_used, scale=None, max_seq: int | None = None,
                      out=None, workspace=None):
    """Causal log-sum-exp of every session's action region, all layers, on the tensor cores.

    q [L, sumA, Hq, D] bf16/fp16 (session r owns rows act_off[r]:act_off[r+1]), kv the full cache
    [L, 2, NB, BS, Hkv, D] of the same dtype, block_table [R, MB] int32, seq_used [R] int32.
    Returns lse [L, sumA, Hq] fp32 (``out`` if given): for action token j of session r,
    log sum_{t <= seq_used[r] - A_r + j} exp(scale * q . k_t), i.e. the lse that
    ``paged_decode_attention_ref`` (lse_attn.py:42-60) returns for that query with
    seq_used = seq_used[r] - A_r + j + 1.  ``max_seq`` bounds every seq_used (default: the block
    table's width); ``workspace`` is a uint8 tensor of ``region_lse_workspace_bytes`` (allocated
    here when None).
    """
    L, sum_a, hq, d = q.shape
    _, _, nb, bs, hkv, _ = kv.shape
    assert hq % hkv == 0
    assert kv.stride(-1) == 1 and q.stride(-1) == 1
    dev = N.require_cuda(q, act_off, kv, block_table, seq_used, out, workspace)
    assert act_off.dtype == torch.int32 and seq_used.dtype == torch.int32 and block_table.dtype == torch.int32
    assert block_table.stride(-1) == 1
    r_n = seq_used.shape[0]
    if max_seq is None:
        max_seq = block_table.shape[1] * bs
    scale = d ** -0.5 if scale is None else scale
    if out is None:
        out = torch.empty(L, sum_a, hq, dtype=torch.float32, device=dev)
    assert out.dtype == torch.float32 and out.stride(-1) == 1 and tuple(out.shape) == (L, sum_a, hq)
    need = region_lse_workspace_bytes(L, sum_a, hq, max_seq)
    if workspace is None or workspace.numel() < need:
        workspace = N.workspace(need, dev)
    lib = N.load()
    N.check(lib.actkv_region_lse(
        q.data_ptr(), N.dtype_code(q), q.stride(0), q.stride(1), q.stride(2), act_off.data_ptr(),
        kv.data_ptr(), N.dtype_code(kv), kv.stride(0), kv.stride(1), kv.stride(2), kv.stride(3), kv.stride(4),
        block_table.data_ptr(), block_table.stride(0), seq_used.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        r_n, L, block_table.shape[1], nb, bs, hq, hkv, d, sum_a, int(max_seq), float(scale),
        workspace.data_ptr(), workspace.numel(), N.status_word(dev).data_ptr(), N.stream_ptr(dev)),
        "action_region_lse")
    return out


def decode_workspace_bytes(R: int, hq: int, hkv: int, d: int, max_seq: int) -> int:
    return int(N.load().actkv_decode_workspace_bytes(R, hq, hkv, d, max_seq))


def paged_decode_attention(q, kv, block_table, seq_used, scale=None, out=None, lse=None, workspace=None):
    """Decode attention over the paged cache with its log-sum-exp, on the GPU (flash decoding):
    (out [R, Hq, D] fp32, lse [R, Hq] fp32), what ``paged_decode_attention_ref`` computes
    (lse_attn.py:42-60) for one query per session.  q [R, Hq, D] and kv [2, NB, BS, Hkv, D] (one
    layer) of one dtype; head_dim 64 or 128, GQA group 1, 2, 4 or 8; the cache's base and strides
    aligned to 16 bytes (else NotImplementedError)."""
    r_n, hq, d = q.shape
    _, nb, bs, hkv, _ = kv.shape
    assert hq % hkv == 0
    assert q.stride(-1) == 1 and kv.stride(-1) == 1 and block_table.stride(-1) == 1
    assert q.dtype == kv.dtype, "q and the cache must share a dtype"
    dev = N.require_cuda(q, kv, block_table, seq_used, out, lse, workspace)
    assert block_table.dtype == torch.int32 and seq_used.dtype == torch.int32
    scale = d ** -0.5 if scale is None else scale
    out = torch.empty(r_n, hq, d, dtype=torch.float32, device=dev) if out is None else out
    lse = torch.empty(r_n, hq, dtype=torch.float32, device=dev) if lse is None else lse
    assert out.stride(-1) == 1 and lse.stride(-1) == 1
    mb = block_table.shape[1]
    need = decode_workspace_bytes(r_n, hq, hkv, d, mb * bs)
    if workspace is None or workspace.numel() < need:
        workspace = N.workspace(need, dev)
    N.check(N.load().actkv_decode_attention(
        q.data_ptr(), N.dtype_code(q), q.stride(0), q.stride(1), kv.data_ptr(), kv.stride(0), kv.stride(1),
        kv.stride(2), kv.stride(3), block_table.data_ptr(), block_table.stride(0), seq_used.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0), r_n, mb, nb, bs, hq, hkv, d,
        float(scale), workspace.data_ptr(), workspace.numel(), N.status_word(dev).data_ptr(), N.stream_ptr(dev)),
        "paged_decode_attention")
    return out, lse
