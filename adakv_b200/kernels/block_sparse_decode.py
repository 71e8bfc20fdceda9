"""Ragged block-sparse flash-decode attention on B200 (sm_100a).

Drop-in for the reference's ``adakv.kernels.block_sparse_decode``
(``adakv/kernels/block_sparse_decode.py:103-135``): same arguments, same
output.  The Triton kernel is replaced by the hand-written CUDA kernel behind
``adakv_attend`` (``include/adakv_b200.h``): split-KV over work items of a few
selected blocks, cp.async-staged gathers, per-item (m, l, o) partials merged by
the last item of each head.  ``HAS_TRITON`` is kept for import compatibility and
is always ``False``: Triton is not used.

Inputs (decode, one query token per sequence):
    q            : [n_q_heads, head_dim]             fp32 / fp16 / bf16, CUDA
    k_cache      : [n_kv_heads, seq_len, head_dim]   same dtype, head_dim contiguous
    v_cache      : [n_kv_heads, seq_len, head_dim]
    block_table  : [n_q_heads, max_sel] int32        selected block ids per head
    sel_lens     : [n_q_heads] int32                 valid entries per row (0 -> zeros)
Output:
    out          : [n_q_heads, head_dim] in q's dtype
Block ids outside ``[0, ceil(seq_len / block_size))`` are skipped by the kernel
and flagged in the workspace status (``adakv_b200._lib.read_status``).
"""
from __future__ import annotations

import torch

from .. import _lib

HAS_TRITON = False


def block_sparse_decode(q, k_cache, v_cache, block_table, sel_lens, block_size, sm_scale=None):
    """Attention of each query head over exactly its listed blocks (see module docstring)."""
    if q.dim() != 2 or k_cache.dim() != 3 or v_cache.dim() != 3:
        raise ValueError("expected q [Hq, D], k_cache / v_cache [Hkv, S, D]")
    out = block_sparse_decode_batched(q.unsqueeze(0), k_cache.unsqueeze(0), v_cache.unsqueeze(0),
                                      block_table, sel_lens, block_size, sm_scale)
    return out[0]


def block_sparse_decode_batched(q, k_cache, v_cache, block_table, sel_lens, block_size,
                                sm_scale=None, seq_lens=None, max_seq_len=None, out=None):
    """Batched form: q [B, Hq, D], caches [B, Hkv, S, D], block_table [B*Hq, W] (or
    [B, Hq, W]), sel_lens [B*Hq]; ``seq_lens`` (int32 CUDA [B], optional) masks each
    sequence's tokens at or past its length."""
    _lib.require_cuda(q, k_cache, v_cache, block_table, sel_lens)
    B, Hq, D = q.shape
    _, Hkv, S, _ = k_cache.shape
    if v_cache.shape != k_cache.shape:
        raise ValueError("k_cache and v_cache shapes differ")
    if block_table.dtype != torch.int32 or sel_lens.dtype != torch.int32:
        raise ValueError("block_table and sel_lens must be int32")
    bt = block_table.reshape(B * Hq, -1)
    if bt.stride(-1) != 1 or (bt.dim() == 2 and bt.stride(0) != bt.shape[1]):
        bt = bt.contiguous()
    sl = sel_lens.reshape(B * Hq).contiguous()
    width = bt.shape[1]
    if width < 1:
        raise ValueError("block_table must have at least one column")
    if seq_lens is not None:
        seq_lens = seq_lens.to(torch.int32).contiguous()
        _lib.require_cuda(seq_lens)
    S_eff = int(max_seq_len) if max_seq_len is not None else S
    sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / (D ** 0.5)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=q.dtype, device=q.device)
    geo = _lib.geometry(B, Hq, Hkv, D, block_size, S_eff, (S_eff + block_size - 1) // block_size,
                        _lib.dtype_code(q))
    L = _lib.lib()
    nbytes = L.adakv_attend_workspace_bytes(geo, width)
    if nbytes == 0:
        _lib.check(_lib.ERR_INVALID)
    ws = _lib.workspace(nbytes, q.device, "attend")
    qv, kv, vv, ov = _lib.view4(q), _lib.view4(k_cache), _lib.view4(v_cache), _lib.view4(out)
    with torch.cuda.device(q.device):
        _lib.check(L.adakv_attend(geo, qv, kv, vv, bt.data_ptr(), width, sl.data_ptr(),
                                  seq_lens.data_ptr() if seq_lens is not None else None,
                                  sm_scale, ov, ws.data_ptr(), ws.numel(),
                                  _lib.stream_ptr(q.device)))
    return out
