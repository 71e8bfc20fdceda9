"""Decode-time operators (mirror of the reference's ``adakv.attention``).

Same names, arguments, return values and error types as
``adakv/attention.py``; every operator runs on the B200 CUDA kernels behind
the C ABI (``include/adakv_b200.h``):

* :class:`AdaKVCache` keeps the float32 per-block centroid table on the GPU
  (``adakv/attention.py:106-146``); ``append_prefill`` builds it with
  ``adakv_centroid_build``, ``append_decode`` appends in place into a
  preallocated cache and refreshes only the touched blocks
  (``adakv_kv_append``) instead of ``torch.cat``-ing the whole cache.
* :func:`plan_selection` (``adakv/attention.py:149-247``) returns
  ``(block_table [Hq, W] int32, sel_lens [Hq] int32)`` without a host sync:
  ``W`` is the largest count the knobs allow (the reference's
  ``max_sel = kph.max().item()`` needs one).  Rows list each head's blocks in
  ascending block order (a set, as every reference consumer treats it).
* :func:`adakv_decode_attention` (``adakv/attention.py:250-268``) runs selection
  and attention back to back on the device (``adakv_decode_step``).

The realised-budget and recall instruments (``adakv/attention.py:24-103``) keep
their API; like the reference they synchronise only while enabled.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from .kernels.block_sparse_decode import block_sparse_decode  # noqa: F401  (re-export)

# --- realised-budget instrumentation -----------------------------------------
_BUDGET_TRACE = None


def reset_budget_trace():
    """Start (or restart) recording the realised mean blocks/head of every step."""
    global _BUDGET_TRACE
    _BUDGET_TRACE = []


def get_budget_trace():
    """Realised mean blocks/head per recorded step since the last reset."""
    return list(_BUDGET_TRACE) if _BUDGET_TRACE is not None else []


def stop_budget_trace():
    """Stop recording (no synchronisation on the decode path afterwards)."""
    global _BUDGET_TRACE
    _BUDGET_TRACE = None


# --- selection-recall instrumentation ------------------------------------------
_RECALL_TARGET = None
_RECALL_HITS = 0
_RECALL_TOTAL = 0


def set_recall_target(block_ids):
    """Record, from now on, whether these block ids are selected by >= 1 head."""
    global _RECALL_TARGET, _RECALL_HITS, _RECALL_TOTAL
    _RECALL_TARGET = {int(b) for b in block_ids}
    _RECALL_HITS = 0
    _RECALL_TOTAL = 0


def get_recall():
    """Fraction of (step, target block) pairs covered by at least one head."""
    return (_RECALL_HITS / _RECALL_TOTAL) if _RECALL_TOTAL else float("nan")


def clear_recall_target():
    global _RECALL_TARGET
    _RECALL_TARGET = None


def _record_recall(block_table, sel_lens, nb):
    global _RECALL_HITS, _RECALL_TOTAL
    width = block_table.shape[-1]
    cols = torch.arange(width, device=block_table.device)
    valid = cols[None, :] < sel_lens.reshape(-1, 1).to(cols.dtype)
    ids = block_table.reshape(-1, width)[valid].long()
    covered = torch.zeros(nb, dtype=torch.bool, device=block_table.device)
    covered[ids.clamp(0, max(nb - 1, 0))] = True
    hits = covered.cpu()
    for b in _RECALL_TARGET:
        if 0 <= b < nb:
            _RECALL_TOTAL += 1
            _RECALL_HITS += int(bool(hits[b]))


def record_selection(block_table, sel_lens, nb):
    """Feed one step's selection to the active instruments (reference API)."""
    if _BUDGET_TRACE is not None:
        _BUDGET_TRACE.append(float(sel_lens.float().mean().item()))
    if _RECALL_TARGET is not None:
        _record_recall(block_table, sel_lens, nb)


def tracing_enabled() -> bool:
    return _BUDGET_TRACE is not None or _RECALL_TARGET is not None


# --- KV cache + centroid table --------------------------------------------------
class AdaKVCache:
    """Full KV cache plus its float32 block-centroid table (no eviction).

    ``k`` / ``v``: ``[n_kv_heads, S, D]``; ``centroid``: ``[n_kv_heads, n_blocks, D]``
    float32.  After the first ``append_decode`` the cache owns a preallocated
    buffer (capacity doubling) and ``k`` / ``v`` are views of it.
    """

    def __init__(self, block_size: int, estimator: str = "centroid"):
        if estimator not in ("centroid", "minmax"):
            raise ValueError(f"unknown estimator: {estimator!r}")
        self.block_size = int(block_size)
        self.estimator = estimator
        self.k = None
        self.v = None
        self.centroid = None
        self.kmin = None
        self.kmax = None
        self._kbuf = None
        self._vbuf = None
        self._cbuf = None
        self._mmbuf = None  # [2, Hkv, cap, D]: minmax estimator's minima / maxima
        self._len = 0

    # geometry of this (batch 1) cache for the C ABI
    def _geometry(self, n_q_heads: int, dtype_code: int):
        Hkv, _, D = self.k.shape
        return _lib.geometry(1, n_q_heads, Hkv, D, self.block_size, self._len,
                             self._cbuf.shape[1], dtype_code)

    @property
    def n_blocks(self) -> int:
        return (self._len + self.block_size - 1) // self.block_size

    def _ensure_centroid_capacity(self, nb: int, device, Hkv: int, D: int):
        if self._cbuf is None or self._cbuf.shape[1] < nb:
            cap = max(nb, 2 * (self._cbuf.shape[1] if self._cbuf is not None else 0), 64)
            buf = torch.empty((Hkv, cap, D), dtype=torch.float32, device=device)
            if self._cbuf is not None:
                buf[:, : self._cbuf.shape[1]] = self._cbuf
            self._cbuf = buf

    def _ensure_minmax_capacity(self, nb: int, device, Hkv: int, D: int):
        if self._mmbuf is None or self._mmbuf.shape[2] < nb:
            cap = self._cbuf.shape[1]
            buf = torch.empty((2, Hkv, cap, D), dtype=torch.float32, device=device)
            if self._mmbuf is not None:
                buf[:, :, : self._mmbuf.shape[2]] = self._mmbuf
            self._mmbuf = buf

    def _minmax_views(self, nb: int):
        self.kmin = self._mmbuf[0, :, :nb]
        self.kmax = self._mmbuf[1, :, :nb]

    def append_prefill(self, k, v):
        """Store prefill KV ``[Hkv, S, D]`` and build the centroid table (and, for
        the minmax estimator, the per-block key minima / maxima)."""
        _lib.require_cuda(k, v)
        if k.shape != v.shape or k.dim() != 3:
            raise ValueError("expected k, v of identical shape [Hkv, S, D]")
        Hkv, S, D = k.shape
        self.k, self.v, self._len = k, v, S
        self._kbuf = self._vbuf = None
        nb = (S + self.block_size - 1) // self.block_size
        self._cbuf = None
        self._ensure_centroid_capacity(nb, k.device, Hkv, D)
        geo = _lib.geometry(1, Hkv, Hkv, D, self.block_size, S, self._cbuf.shape[1],
                            _lib.dtype_code(k))
        with torch.cuda.device(k.device):
            _lib.check(_lib.lib().adakv_centroid_build(geo, _lib.view4(k.unsqueeze(0)), None,
                                                       self._cbuf.data_ptr(),
                                                       _lib.stream_ptr(k.device)))
        self.centroid = self._cbuf[:, :nb]
        if self.estimator == "minmax":
            self._mmbuf = None
            self._ensure_minmax_capacity(nb, k.device, Hkv, D)
            with torch.cuda.device(k.device):
                _lib.check(_lib.lib().adakv_minmax_build(
                    geo, _lib.view4(k.unsqueeze(0)), None, self._mmbuf[0].data_ptr(),
                    self._mmbuf[1].data_ptr(), _lib.stream_ptr(k.device)))
            self._minmax_views(nb)
        return self

    def append_decode(self, k_t, v_t):
        """Append decoded tokens ``[Hkv, n, D]`` in place; refresh touched centroids."""
        _lib.require_cuda(k_t, v_t)
        if self.k is None:
            raise ValueError("append_prefill must be called first")
        Hkv, S, D = self.k.shape
        n = k_t.shape[1]
        if k_t.shape != (Hkv, n, D) or v_t.shape != k_t.shape:
            raise ValueError(f"expected k_t, v_t of shape [{Hkv}, n, {D}]")
        if k_t.dtype != self.k.dtype or v_t.dtype != self.k.dtype:
            raise ValueError("k_t / v_t dtype must match the cache")
        need = S + n
        if self._kbuf is None or self._kbuf.shape[1] < need:
            cap = max(2 * need, need + 256)
            kb = torch.empty((Hkv, cap, D), dtype=self.k.dtype, device=self.k.device)
            vb = torch.empty_like(kb)
            kb[:, :S] = self.k
            vb[:, :S] = self.v
            self._kbuf, self._vbuf = kb, vb
        nb = (need + self.block_size - 1) // self.block_size
        self._ensure_centroid_capacity(nb, self.k.device, Hkv, D)
        self._len = need
        geo = _lib.geometry(1, Hkv, Hkv, D, self.block_size, need, self._cbuf.shape[1],
                            _lib.dtype_code(self.k))
        k_t = k_t if k_t.stride(-1) == 1 else k_t.contiguous()
        v_t = v_t if v_t.stride(-1) == 1 else v_t.contiguous()
        with torch.cuda.device(self.k.device):
            _lib.check(_lib.lib().adakv_kv_append(
                geo, _lib.view4(self._kbuf.unsqueeze(0)), _lib.view4(self._vbuf.unsqueeze(0)),
                _lib.view4(k_t.unsqueeze(0)), _lib.view4(v_t.unsqueeze(0)), n, None,
                self._cbuf.data_ptr(), _lib.stream_ptr(self.k.device)))
        self.k = self._kbuf[:, :need]
        self.v = self._vbuf[:, :need]
        self.centroid = self._cbuf[:, :nb]
        if self.estimator == "minmax":
            self._ensure_minmax_capacity(nb, self.k.device, Hkv, D)
            with torch.cuda.device(self.k.device):
                _lib.check(_lib.lib().adakv_minmax_refresh(
                    geo, _lib.view4(self._kbuf.unsqueeze(0)), n, None, self._mmbuf[0].data_ptr(),
                    self._mmbuf[1].data_ptr(), _lib.stream_ptr(self.k.device)))
            self._minmax_views(nb)
        return self


def _plan_args(q, cache, avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks, temperature,
               estimator, budget_policy, c_min, nucleus_p=0.9):
    if estimator == "minmax":
        if cache.kmin is None or cache.kmax is None:
            raise ValueError("minmax estimator needs AdaKVCache(estimator='minmax')")
    elif estimator != "centroid":
        raise ValueError(f"unknown estimator: {estimator!r}")
    if cache.centroid is None:
        raise ValueError("cache has no centroid table (call append_prefill first)")
    _lib.require_cuda(q)
    if q.dim() != 2:
        raise ValueError("q must be [n_q_heads, head_dim]")
    sp = _lib.select_params(avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks, c_min,
                            temperature, budget_policy, nucleus_p)
    geo = cache._geometry(q.shape[0], _lib.dtype_code(q))
    return geo, sp


def plan_selection(
    q,
    cache: AdaKVCache,
    avg_budget: int,
    k_min: int = 2,
    k_max: int = 64,
    n_sink_blocks: int = 1,
    n_local_blocks: int = 4,
    temperature: float = 1.0,
    estimator: str = "centroid",
    budget_policy: str = "adaptive",
    c_min: int = 1,
    nucleus_p: float = 0.9,
    order: str = "score",
):
    """Score blocks, allocate per-head budgets, select blocks (reference signature).

    Returns ``(block_table [Hq, max_sel] int32, sel_lens [Hq] int32)`` in the
    reference's format (``adakv/attention.py:229-244``): row ``h`` lists its
    ``sel_lens[h]`` blocks in descending order of the sink/local-biased score
    (forced blocks first, in ascending block order; score ties by ascending
    block index), and ``max_sel = sel_lens.max()`` is read back to the host as
    the reference does (``attention.py:242``); entries past ``sel_lens[h]`` are
    unspecified.  ``order="ascending"`` skips the reordering and the host read:
    rows are then in ascending block order and the width is the largest count
    the knobs allow (the C ABI's ``adakv_plan`` layout).
    """
    if order not in ("score", "ascending"):
        raise ValueError(f"unknown order: {order!r}")
    geo, sp = _plan_args(q, cache, avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks,
                         temperature, estimator, budget_policy, c_min, nucleus_p)
    L = _lib.lib()
    width = L.adakv_plan_table_width(geo, sp)
    if width < 1:
        _lib.check(_lib.ERR_INVALID)
    Hq = q.shape[0]
    block_table = torch.empty((Hq, width), dtype=torch.int32, device=q.device)
    sel_lens = torch.empty((Hq,), dtype=torch.int32, device=q.device)
    nbytes = L.adakv_plan_workspace_bytes(geo, sp)
    ws = _lib.workspace(nbytes, q.device)
    q = q if q.stride(-1) == 1 else q.contiguous()
    with torch.cuda.device(q.device):
        if estimator == "minmax":
            # Quest scores (adakv/attention.py:190-198), then the same budget + top-k
            scores = torch.empty((Hq, cache._cbuf.shape[1]), dtype=torch.float32, device=q.device)
            _lib.check(L.adakv_estimate_minmax(geo, _lib.view4(q.unsqueeze(0)),
                                               cache._mmbuf[0].data_ptr(), cache._mmbuf[1].data_ptr(),
                                               None, scores.data_ptr(), scores.stride(0),
                                               _lib.stream_ptr(q.device)))
            _lib.check(L.adakv_select(geo, sp, scores.data_ptr(), scores.stride(0), None,
                                      block_table.data_ptr(), width, sel_lens.data_ptr(),
                                      ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device)))
        else:
            scores = None
            if order == "score":
                scores = torch.empty((Hq, cache._cbuf.shape[1]), dtype=torch.float32,
                                     device=q.device)
            _lib.check(L.adakv_plan(geo, sp, _lib.view4(q.unsqueeze(0)), cache._cbuf.data_ptr(),
                                    None, block_table.data_ptr(), width, sel_lens.data_ptr(),
                                    scores.data_ptr() if scores is not None else None,
                                    ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device)))
        _lib.raise_if_failed(ws)
        if order == "score":
            block_table = _score_order(block_table, sel_lens, scores, cache.n_blocks,
                                       n_sink_blocks, n_local_blocks)
    record_selection(block_table, sel_lens, cache.n_blocks)
    return block_table, sel_lens


def _score_order(block_table, sel_lens, scores, nb, n_sink_blocks, n_local_blocks):
    """Rows of ascending block ids -> the reference's order (``attention.py:229-234``:
    ``+inf`` on sink / local blocks, descending sort), width ``sel_lens.max()``."""
    max_sel = max(int(sel_lens.max().item()), 1)  # host read, as attention.py:242
    ids = block_table[:, :max_sel].long()
    valid = torch.arange(max_sel, device=ids.device)[None, :] < sel_lens[:, None]
    ids = torch.where(valid, ids, torch.zeros_like(ids))
    key = torch.gather(scores[:, :max(nb, 1)], 1, ids.clamp_max(max(nb, 1) - 1)).double()
    sink, local = min(n_sink_blocks, nb), min(n_local_blocks, nb)
    forced = (ids < sink) | (ids >= nb - local)
    key = torch.where(forced, torch.full_like(key, float("inf")), key)
    key = torch.where(valid, key, torch.full_like(key, float("-inf")))
    # rows are ascending, so a stable descending sort breaks ties by ascending block id
    perm = torch.sort(key, dim=1, descending=True, stable=True).indices
    return torch.gather(block_table[:, :max_sel], 1, perm).contiguous()


def adakv_decode_attention(
    q,
    cache: AdaKVCache,
    avg_budget: int,
    k_min: int = 2,
    k_max: int = 64,
    n_sink_blocks: int = 1,
    n_local_blocks: int = 4,
    temperature: float = 1.0,
):
    """One AdaKV decode step: selection then attention, on the device (reference signature)."""
    return _decode(q, cache, avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks, temperature,
                   "centroid", "adaptive", 1, 1.0 / math.sqrt(q.shape[-1]))


def _decode(q, cache, avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks, temperature,
            estimator, budget_policy, c_min, sm_scale):
    geo, sp = _plan_args(q, cache, avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks,
                         temperature, estimator, budget_policy, c_min)
    if q.dtype != cache.k.dtype:
        raise ValueError("q and the KV cache must share one dtype")
    L = _lib.lib()
    width = L.adakv_plan_table_width(geo, sp)
    Hq = q.shape[0]
    block_table = torch.empty((Hq, width), dtype=torch.int32, device=q.device)
    sel_lens = torch.empty((Hq,), dtype=torch.int32, device=q.device)
    out = torch.empty_like(q) if q.stride(-1) == 1 else torch.empty(q.shape, dtype=q.dtype,
                                                                   device=q.device)
    ws = _lib.workspace(L.adakv_plan_workspace_bytes(geo, sp), q.device)
    q = q if q.stride(-1) == 1 else q.contiguous()
    with torch.cuda.device(q.device):
        _lib.check(L.adakv_decode_step(
            geo, sp, _lib.view4(q.unsqueeze(0)), _lib.view4(cache.k.unsqueeze(0)),
            _lib.view4(cache.v.unsqueeze(0)), None, None, 0, cache._cbuf.data_ptr(), None,
            float(sm_scale),
            block_table.data_ptr(), width, sel_lens.data_ptr(), _lib.view4(out.unsqueeze(0)),
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device)))
    _lib.raise_if_failed(ws)
    if tracing_enabled():
        record_selection(block_table, sel_lens, cache.n_blocks)
    return out
