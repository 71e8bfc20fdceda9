"""Batched, preallocated decode state over the C ABI.

:class:`BatchedDecoder` owns everything one attention layer needs for ragged
batched decode: the K/V cache ``[B, Hkv, capacity, D]``, the float32 centroid
table ``[B, Hkv, nb_cap, D]``, per-sequence lengths on the device, the plan
outputs and one workspace.  Every method only enqueues kernels on the current
stream (no allocation, no host synchronisation), so a decode step can be
captured in a CUDA graph after one warm-up call.

The reference runs batch 1 only (``adakv/runtime.py:97``, ``adakv/patch.py:96``);
this is the batched form of the same step used for ragged-batch decode.
"""
from __future__ import annotations

import math

import torch

from . import _lib


def partition_batch(seq_lens, world):
    """Contiguous, context-balanced split of a batch over ``world`` ranks (no
    collective: sequences are independent).  Returns ``[(start, end)]`` per
    rank; boundaries are placed where the running context sum crosses
    ``r / world`` of the total."""
    lens = [int(x) for x in seq_lens]
    total = sum(lens)
    bounds, acc, b = [0], 0, 0
    for r in range(1, world):
        target = total * r / world
        while b < len(lens) and acc + lens[b] / 2 <= target:
            acc += lens[b]
            b += 1
        bounds.append(max(b, bounds[-1]))
    bounds.append(len(lens))
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def stage(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """Copy ``src`` (a page-locked host tensor, ``pin_memory()``, or a CUDA
    tensor) into the CUDA tensor ``dst`` with the library's staging kernel
    (``adakv_stage``), on the current stream of ``dst``'s device.  For a decode
    step's few KB of inputs this is several microseconds faster than a
    copy-engine transfer (``dst.copy_(src, non_blocking=True)``).  Both tensors
    contiguous, of one byte size, 16-byte aligned."""
    if not dst.is_cuda:
        raise ValueError("dst must be a CUDA tensor")
    if not (src.is_cuda or src.is_pinned()):
        raise ValueError("src must be a CUDA tensor or a page-locked host tensor")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("dst and src must be contiguous")
    nbytes = dst.numel() * dst.element_size()
    if src.numel() * src.element_size() != nbytes:
        raise ValueError("dst and src must have the same size in bytes")
    with torch.cuda.device(dst.device):
        _lib.check(_lib.lib().adakv_stage(dst.data_ptr(), src.data_ptr(), nbytes,
                                          _lib.stream_ptr(dst.device)))
    return dst


class BatchedDecoder:
    def __init__(self, batch, n_q_heads, n_kv_heads, head_dim, block_size, capacity, dtype,
                 device="cuda", avg_budget=64, k_min=2, k_max=64, n_sink_blocks=1,
                 n_local_blocks=4, c_min=1, temperature=1.0, budget_policy="adaptive",
                 nucleus_p=0.9):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("BatchedDecoder needs a CUDA device (no CPU fallback)")
        self.B, self.Hq, self.Hkv, self.D = batch, n_q_heads, n_kv_heads, head_dim
        self.bs, self.capacity, self.dtype = block_size, capacity, dtype
        self.nb_cap = (capacity + block_size - 1) // block_size
        self.params = _lib.select_params(avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks,
                                         c_min, temperature, budget_policy, nucleus_p)
        self.k = torch.zeros((batch, n_kv_heads, capacity, head_dim), dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.centroid = torch.zeros((batch, n_kv_heads, self.nb_cap, head_dim), dtype=torch.float32,
                                    device=device)
        self.seq_lens = torch.zeros((batch,), dtype=torch.int32, device=device)
        self.host_seq_lens = [0] * batch
        geo = self.geometry()
        L = _lib.lib()
        self.table_width = L.adakv_plan_table_width(geo, self.params)
        if self.table_width < 1:
            _lib.check(_lib.ERR_INVALID)
        self.block_table = torch.zeros((batch * n_q_heads, self.table_width), dtype=torch.int32,
                                       device=device)
        self.sel_lens = torch.zeros((batch * n_q_heads,), dtype=torch.int32, device=device)
        self.ws_bytes = L.adakv_plan_workspace_bytes(geo, self.params)
        self.workspace = torch.zeros((self.ws_bytes,), dtype=torch.uint8, device=device)
        # kernels write their ADAKV_ST_* bits to this host word too: a failed
        # step raises on the next call without a device synchronisation
        self.sink = _lib.StatusSink(self.workspace)
        self.out = torch.zeros((batch, n_q_heads, head_dim), dtype=dtype, device=device)
        # The per-step C-ABI arguments that never change, built once: a decode
        # step is short enough (tens of microseconds) that rebuilding them
        # would keep the GPU waiting for the host.
        self._geo = geo
        self._kview, self._vview = _lib.view4(self.k), _lib.view4(self.v)
        self._dev_index = (self.device.index if self.device.index is not None
                           else torch.cuda.current_device())

    def geometry(self, max_seq_len=None):
        return _lib.geometry(self.B, self.Hq, self.Hkv, self.D, self.bs,
                             max_seq_len if max_seq_len is not None else self.capacity,
                             self.nb_cap, _lib.TORCH_DTYPES[self.dtype])

    def _stream(self):
        return _lib.stream_ptr(self.device)

    # -- prefill ------------------------------------------------------------------
    def load(self, K, V, seq_lens):
        """Copy prefilled K/V ``[B, Hkv, S, D]`` into the cache and build the centroids."""
        seq_lens = [int(s) for s in seq_lens]
        S = K.shape[2]
        if S > self.capacity or max(seq_lens) > S:
            raise ValueError("prefill longer than the cache capacity")
        self.k[:, :, :S].copy_(K, non_blocking=True)
        self.v[:, :, :S].copy_(V, non_blocking=True)
        self.host_seq_lens = seq_lens
        self.seq_lens.copy_(torch.tensor(seq_lens, dtype=torch.int32), non_blocking=True)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().adakv_centroid_build(
                self.geometry(), _lib.view4(self.k), self.seq_lens.data_ptr(),
                self.centroid.data_ptr(), self._stream()))

    # -- decode -------------------------------------------------------------------
    def append(self, k_new, v_new, advance=True):
        """Append ``[B, Hkv, n, D]`` tokens to every sequence and refresh the touched
        centroids.  With ``advance=False`` the lengths stay put and the last ``n``
        tokens are overwritten (fixed-context benchmarking)."""
        n = k_new.shape[2]
        if advance:
            if max(self.host_seq_lens) + n > self.capacity:
                raise ValueError("cache capacity exceeded")
            self.host_seq_lens = [s + n for s in self.host_seq_lens]
            self.seq_lens.add_(n)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().adakv_kv_append(
                self.geometry(), _lib.view4(self.k), _lib.view4(self.v), _lib.view4(k_new),
                _lib.view4(v_new), n, self.seq_lens.data_ptr(), self.centroid.data_ptr(),
                self._stream()))

    def plan(self, q, scores_out=None):
        """Block selection for ``q`` ``[B, Hq, D]``; fills ``block_table`` / ``sel_lens``."""
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().adakv_plan(
                self.geometry(), self.params, _lib.view4(q), self.centroid.data_ptr(),
                self.seq_lens.data_ptr(), self.block_table.data_ptr(), self.table_width,
                self.sel_lens.data_ptr(),
                scores_out.data_ptr() if scores_out is not None else None,
                self.workspace.data_ptr(), self.ws_bytes, self._stream()))
        return self.block_table, self.sel_lens

    def step(self, q, sm_scale=None, out=None, k_new=None, v_new=None, advance=True):
        """Selection + attention for ``q`` ``[B, Hq, D]``; returns ``[B, Hq, D]``.

        With ``k_new`` / ``v_new`` (``[B, Hkv, n, D]``) the step first appends those
        tokens (fused into the estimator kernel: in-place cache write + centroid
        refresh).  ``advance=False`` overwrites the last ``n`` tokens instead of
        growing the sequences (fixed-context benchmarking).  ``out`` may be a
        page-locked host tensor (``pin_memory()``, mapped into the device's
        address space): the attention kernel then writes the result straight
        into host memory, with no separate device-to-host copy."""
        out = self.out if out is None else out
        if not out.is_cuda and not out.is_pinned():
            raise ValueError("out must be a CUDA tensor or a page-locked host tensor")
        if out.shape != self.out.shape or out.dtype != self.out.dtype:
            raise ValueError(f"out must be {tuple(self.out.shape)} {self.out.dtype}")
        scale = 1.0 / math.sqrt(self.D) if sm_scale is None else float(sm_scale)
        n_new = 0
        kn = vn = None
        if k_new is not None:
            n_new = k_new.shape[2]
            if advance:
                if max(self.host_seq_lens) + n_new > self.capacity:
                    raise ValueError("cache capacity exceeded")
                self.host_seq_lens = [s + n_new for s in self.host_seq_lens]
                self.seq_lens.add_(n_new)
            kn, vn = _lib.view4(k_new), _lib.view4(v_new)
        self.sink.raise_if_set()
        args = (self._geo, self.params, _lib.view4(q), self._kview, self._vview, kn, vn, n_new,
                self.centroid.data_ptr(), self.seq_lens.data_ptr(), scale,
                self.block_table.data_ptr(), self.table_width, self.sel_lens.data_ptr(),
                _lib.view4(out), self.workspace.data_ptr(), self.ws_bytes, self._stream())
        if torch.cuda.current_device() == self._dev_index:
            _lib.check(_lib.lib().adakv_decode_step(*args))
        else:
            with torch.cuda.device(self.device):
                _lib.check(_lib.lib().adakv_decode_step(*args))
        return out

    def graphed(self, n_new=1, advance=True, sm_scale=None):
        """One decode step captured in a CUDA graph over decoder-owned buffers.

        Returns a :class:`GraphedStep`: write the step's query into ``.q``
        (``[B, Hq, D]``) and its ``n_new`` new tokens into ``.k_new`` /
        ``.v_new`` (``[B, Hkv, n_new, D]``) -- all three are views of one
        device buffer, ``.inputs``, so a host staging row can fill them with
        one copy -- then call it; the output is ``.out``.  A replay launches
        the step's three kernels from one graph instead of three host calls,
        which keeps the GPU from waiting on the host between decode steps.
        One step without append runs first (device set-up that cannot be
        captured); it writes only the plan outputs and ``.out``."""
        return GraphedStep(self, n_new, advance, sm_scale)

    def attend(self, q, block_table, sel_lens, sm_scale=None, out=None):
        """Attention over a caller-given table (``adakv_attend``)."""
        from .kernels.block_sparse_decode import block_sparse_decode_batched
        return block_sparse_decode_batched(q, self.k, self.v, block_table, sel_lens, self.bs,
                                           sm_scale, seq_lens=self.seq_lens,
                                           max_seq_len=self.capacity, out=out)

    def status(self) -> int:
        """Synchronise; return and clear the device status bits (ADAKV_ST_*)."""
        bits = _lib.read_status(self.workspace)
        self.sink.clear()
        return bits

    def last_path(self) -> int:
        """2 if the last step ran as the one-kernel step, 1 as the kernel chain."""
        return int(_lib.lib().adakv_last_path(self.workspace.data_ptr()))

    def scores(self, out=None):
        """Block scores ``[B, Hq, nb]`` (float32, q . centroid) of the last step / plan."""
        nb = self.nb_cap
        out = torch.empty((self.B, self.Hq, nb), dtype=torch.float32, device=self.device) \
            if out is None else out
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().adakv_read_scores(self._geo, self.workspace.data_ptr(),
                                                    self.ws_bytes, out.data_ptr(), out.stride(1),
                                                    self._stream()))
        return out

    def selected_sets(self):
        """Host copy of the selection: list over rows (b*Hq + h) of block-id arrays."""
        bt = self.block_table.cpu().numpy()
        sl = self.sel_lens.cpu().numpy()
        return [bt[r, : sl[r]] for r in range(bt.shape[0])]


class GraphedStep:
    """A decode step of a :class:`BatchedDecoder` replayed from a CUDA graph
    (see :meth:`BatchedDecoder.graphed`)."""

    def __init__(self, dec, n_new, advance, sm_scale):
        self.dec, self.n_new, self.advance = dec, int(n_new), bool(advance)
        B, Hq, Hkv, D = dec.B, dec.Hq, dec.Hkv, dec.D
        nq, nk = B * Hq * D, B * Hkv * self.n_new * D
        self.inputs = torch.zeros(nq + 2 * nk, dtype=dec.dtype, device=dec.device)
        self.q = self.inputs[:nq].view(B, Hq, D)
        self.k_new = self.inputs[nq:nq + nk].view(B, Hkv, self.n_new, D)
        self.v_new = self.inputs[nq + nk:].view(B, Hkv, self.n_new, D)
        self.out = dec.out
        with torch.cuda.device(dec.device):
            dec.step(self.q, sm_scale=sm_scale)  # set-up outside the capture (no append)
            self.graph = torch.cuda.CUDAGraph()
            host_lens = list(dec.host_seq_lens)
            with torch.cuda.graph(self.graph):
                dec.step(self.q, sm_scale=sm_scale, k_new=self.k_new, v_new=self.v_new,
                         advance=self.advance)
            # capture records the step (its length increment included) without
            # running it: the host copy of the lengths moves on replay only
            dec.host_seq_lens = host_lens

    def __call__(self):
        """Replay the step on the current stream; returns ``.out``."""
        dec = self.dec
        dec.sink.raise_if_set()
        if self.advance:
            if max(dec.host_seq_lens) + self.n_new > dec.capacity:
                raise ValueError("cache capacity exceeded")
            dec.host_seq_lens = [s + self.n_new for s in dec.host_seq_lens]
        self.graph.replay()
        return self.out
