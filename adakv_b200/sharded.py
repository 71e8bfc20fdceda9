"""Sequence-sharded AdaKV decode: one long sequence split over several GPUs.

The reference decodes one sequence on one device.  For a context too long to
serve from one GPU at the wanted latency (1M tokens), the sequence is split
into contiguous block ranges, one per rank, and each decode step runs as

1. every rank scores the blocks it holds (``adakv_estimate``: q . centroid,
   GQA folded, the scoring of ``adakv/estimator.py:62-74``);
2. the selection (entropy budget and top-k over each head's whole row,
   ``adakv/budget.py:45-86``, ``adakv/selector.py:18-60``), by default from
   exchanged statistics (``StatsSelector``): each rank all-gathers per-head
   softmax statistics plus its shard's sorted top content candidates, then
   one clamp term per head, and every rank derives the same budgets and keeps
   the selected blocks it holds.  No score row leaves its rank.  The nucleus
   policy, which ranks the whole row's probability mass, instead all-gathers
   the score rows and selects on them (``Selector``, ``selection="rows"``);
3. every rank attends over the selected blocks it holds
   (``adakv_attend_partial``) and returns its normalised output and
   log-sum-exp per query head;
4. the ranks all-gather those partials and merge them by log-sum-exp
   (``adakv_combine``).

Shard ``r`` holds blocks ``[r * L, (r + 1) * L)`` with ``L`` a multiple of 32
blocks (whole selection-bitmap words); the last rank holds the tail, so the
sink blocks live on rank 0 and the local window on the last rank.

Collectives go through a small interface: ``TorchGroup`` (``torch.distributed``,
one process per GPU) or the ``emulate_*`` functions (all shards in one
process, for tests on one device).
"""
from __future__ import annotations

import math

import torch

from . import _lib


def shard_blocks(nb: int, world: int) -> int:
    """Blocks per rank (a multiple of 32) for a sequence of ``nb`` blocks."""
    per = -(-nb // world)
    return max(32, -(-per // 32) * 32)


def shard_range(nb: int, world: int, rank: int):
    """``(first block, block count)`` of rank ``rank``'s shard."""
    L = shard_blocks(nb, world)
    lo = min(nb, rank * L)
    return lo, max(0, min(nb, lo + L) - lo)


class ShardCache:
    """One rank's K/V blocks of the sequence and their centroids.

    ``K``, ``V``: ``[Hkv, S_local, D]`` (tokens ``[tok_lo, tok_lo + S_local)`` of
    the sequence; ``tok_lo`` a multiple of ``32 * block_size``)."""

    def __init__(self, K, V, block_lo: int, n_q_heads: int, block_size: int, capacity_blocks=None):
        _lib.require_cuda(K, V)
        if K.shape != V.shape or K.dim() != 3:
            raise ValueError("K and V must be [Hkv, S_local, D] of one shape")
        if block_lo % 32:
            raise ValueError("a shard must start on a multiple of 32 blocks")
        self.Hkv, self.S, self.D = K.shape
        self.Hq, self.bs, self.block_lo = n_q_heads, block_size, block_lo
        self.k, self.v, self.dtype = K, V, K.dtype
        self.nb = -(-self.S // block_size)
        self.cap = max(capacity_blocks or self.nb, self.nb, 1)
        self.centroid = torch.zeros((self.Hkv, self.cap, self.D), dtype=torch.float32,
                                    device=K.device)
        self._ws = {}
        if self.S > 0:
            with torch.cuda.device(K.device):
                _lib.check(_lib.lib().adakv_centroid_build(
                    self._geo(), _lib.view4(K.unsqueeze(0)), None, self.centroid.data_ptr(),
                    _lib.stream_ptr(K.device)))

    def _geo(self):
        return _lib.geometry(1, self.Hq, self.Hkv, self.D, self.bs, max(self.S, 1), self.cap,
                             _lib.TORCH_DTYPES[self.dtype])

    def _workspace(self, nbytes, device, kind):
        """This shard's workspace of ``kind``, allocated on first use and kept
        (a replay of a captured step must find the same buffer)."""
        ws = self._ws.get(kind)
        if ws is None or ws.numel() < nbytes:
            ws = self._ws[kind] = _lib.workspace(nbytes, device, kind)
        return ws

    def local_scores(self, q, out):
        """Scores of this shard's blocks into ``out[:, :nb]`` (``out``: ``[Hq, >= cap]`` fp32)."""
        if self.S == 0:
            return out
        L = _lib.lib()
        geo = self._geo()
        ws = self._workspace(L.adakv_plan_workspace_bytes(geo, _lib.select_params(
            1, 1, 1, 0, 0, 0, 1.0, "fixed")), q.device, "shard-estimate")
        with torch.cuda.device(q.device):
            _lib.check(L.adakv_estimate(geo, _lib.view4(q.unsqueeze(0)), self.centroid.data_ptr(),
                                        None, out.data_ptr(), out.stride(0), ws.data_ptr(),
                                        ws.numel(), _lib.stream_ptr(q.device)))
        return out

    def attend_partial(self, q, block_table, sel_lens, sm_scale, packed=None):
        """``(o [Hq, D] fp32, lse [Hq] fp32)`` over the selected blocks held here.
        With ``packed`` (float32, ``Hq * (D + 1)`` elements) both are views of it,
        o first, so one collective can carry them."""
        n = self.Hq * self.D
        if packed is None:
            packed = torch.empty(n + self.Hq, dtype=torch.float32, device=q.device)
        o = packed[:n].view(self.Hq, self.D)
        lse = packed[n:n + self.Hq]
        if self.S == 0:  # (otherwise the kernel writes every row, empty ones as 0 and -inf)
            o.zero_()
            lse.fill_(-math.inf)
            return o, lse
        L = _lib.lib()
        geo = self._geo()
        width = block_table.shape[1]
        ws = self._workspace(L.adakv_attend_workspace_bytes(geo, width), q.device, "shard-attend")
        with torch.cuda.device(q.device):
            _lib.check(L.adakv_attend_partial(
                geo, _lib.view4(q.unsqueeze(0)), _lib.view4(self.k.unsqueeze(0)),
                _lib.view4(self.v.unsqueeze(0)), block_table.data_ptr(), width,
                sel_lens.data_ptr(), self.block_lo, None, float(sm_scale), o.data_ptr(),
                lse.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr(q.device)))
        return o, lse


class Selector:
    """Budget + top-k over the full score rows of one sequence (every rank runs it)."""

    def __init__(self, S_total, n_q_heads, n_kv_heads, head_dim, block_size, dtype, device,
                 avg_budget=64, k_min=2, k_max=64, n_sink_blocks=1, n_local_blocks=4, c_min=1,
                 temperature=1.0, budget_policy="adaptive", nucleus_p=0.9):
        self.nb = -(-S_total // block_size)
        self.geo = _lib.geometry(1, n_q_heads, n_kv_heads, head_dim, block_size, S_total, self.nb,
                                 _lib.TORCH_DTYPES[dtype])
        self.params = _lib.select_params(avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks,
                                         c_min, temperature, budget_policy, nucleus_p)
        L = _lib.lib()
        self.width = L.adakv_plan_table_width(self.geo, self.params)
        if self.width < 1:
            _lib.check(_lib.ERR_INVALID)
        self.table = torch.zeros((n_q_heads, self.width), dtype=torch.int32, device=device)
        self.sel_lens = torch.zeros((n_q_heads,), dtype=torch.int32, device=device)
        self.ws = torch.zeros((L.adakv_plan_workspace_bytes(self.geo, self.params),),
                              dtype=torch.uint8, device=device)

    def select(self, scores):
        """``scores``: ``[Hq, >= nb]`` fp32 rows in block order -> (table, sel_lens)."""
        with torch.cuda.device(scores.device):
            _lib.check(_lib.lib().adakv_select(
                self.geo, self.params, scores.data_ptr(), scores.stride(0), None,
                self.table.data_ptr(), self.width, self.sel_lens.data_ptr(), self.ws.data_ptr(),
                self.ws.numel(), _lib.stream_ptr(scores.device)))
        return self.table, self.sel_lens


class StatsSelector:
    """One rank's part of the selection from exchanged statistics
    (``adakv_shard_prep`` / ``adakv_shard_clamp`` / ``adakv_shard_finish``).

    ``prep`` writes this rank's record (per head: softmax statistics and the
    shard's top content candidates, sorted); once every rank's records are
    gathered, ``clamp`` gives this shard's clamp terms of the entropy
    (adaptive policy); once those are gathered too, ``finish`` writes this
    rank's block table: the selected blocks it holds, as global ids."""

    def __init__(self, S_total, n_q_heads, n_kv_heads, head_dim, block_size, dtype, device,
                 block_lo, n_local, avg_budget=64, k_min=2, k_max=64, n_sink_blocks=1,
                 n_local_blocks=4, c_min=1, temperature=1.0, budget_policy="adaptive",
                 nucleus_p=0.9):
        self.nb = -(-S_total // block_size)
        if block_lo < 0 or n_local < 0 or block_lo + n_local > self.nb:
            raise ValueError("the shard's blocks must lie inside the sequence")
        self.geo = _lib.geometry(1, n_q_heads, n_kv_heads, head_dim, block_size, S_total, self.nb,
                                 _lib.TORCH_DTYPES[dtype])
        self.params = _lib.select_params(avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks,
                                         c_min, temperature, budget_policy, nucleus_p)
        L = _lib.lib()
        self.record_bytes = L.adakv_shard_record_bytes(self.geo, self.params)
        if self.record_bytes == 0:
            raise ValueError("the statistics exchange does not apply here (batch 1 and the fixed "
                             "or adaptive policy only): "
                             + L.adakv_last_error().decode(errors="replace"))
        self.width = L.adakv_plan_table_width(self.geo, self.params)
        self.adaptive = budget_policy == "adaptive"
        self.block_lo, self.n_local, self.Hq = block_lo, n_local, n_q_heads
        self.record = torch.zeros((self.record_bytes,), dtype=torch.uint8, device=device)
        self.cc = torch.zeros((n_q_heads,), dtype=torch.float64, device=device)
        self.table = torch.zeros((n_q_heads, self.width), dtype=torch.int32, device=device)
        self.sel_lens = torch.zeros((n_q_heads,), dtype=torch.int32, device=device)
        self.status = torch.zeros((4,), dtype=torch.int32, device=device)

    @staticmethod
    def applies(budget_policy="adaptive", batch=1):
        return batch == 1 and budget_policy in ("fixed", "adaptive")

    def prep(self, scores):
        """``scores``: this shard's rows ``[Hq, >= n_local]`` fp32 -> the record (uint8)."""
        with torch.cuda.device(self.record.device):
            _lib.check(_lib.lib().adakv_shard_prep(
                self.geo, self.params, scores.data_ptr(), scores.stride(0), self.block_lo,
                self.n_local, self.record.data_ptr(), _lib.stream_ptr(self.record.device)))
        return self.record

    def clamp(self, scores, records):
        """``records``: ``[world, record_bytes]`` uint8 in rank order -> ``cc [Hq]`` fp64."""
        records = records.contiguous()
        with torch.cuda.device(self.record.device):
            _lib.check(_lib.lib().adakv_shard_clamp(
                self.geo, self.params, scores.data_ptr(), scores.stride(0), self.block_lo,
                self.n_local, records.data_ptr(), records.stride(0), records.shape[0],
                self.cc.data_ptr(), _lib.stream_ptr(self.record.device)))
        return self.cc

    def finish(self, records, ccs, rank):
        """Every rank's records and clamp terms (``[world, Hq]`` fp64, or None
        for the fixed policy) -> this rank's ``(table, sel_lens)``."""
        records = records.contiguous()
        cc_ptr = None
        if ccs is not None:
            ccs = ccs.contiguous()
            cc_ptr = ccs.data_ptr()
        with torch.cuda.device(self.record.device):
            _lib.check(_lib.lib().adakv_shard_finish(
                self.geo, self.params, records.data_ptr(), records.stride(0), cc_ptr,
                records.shape[0], rank, self.block_lo, self.n_local, self.table.data_ptr(),
                self.width, self.sel_lens.data_ptr(), self.status.data_ptr(),
                _lib.stream_ptr(self.record.device)))
        return self.table, self.sel_lens


def combine(parts, lse, dtype, out=None):
    """Log-sum-exp merge: ``parts [N, Hq, D]`` fp32, ``lse [N, Hq]`` -> ``[Hq, D]``."""
    N, Hq, D = parts.shape
    if out is None:
        out = torch.empty((Hq, D), dtype=dtype, device=parts.device)
    parts = parts.contiguous()
    lse = lse.contiguous()
    with torch.cuda.device(parts.device):
        _lib.check(_lib.lib().adakv_combine(N, 1, Hq, D, _lib.TORCH_DTYPES[dtype], parts.data_ptr(),
                                            lse.data_ptr(), _lib.view4(out.unsqueeze(0)),
                                            _lib.stream_ptr(parts.device)))
    return out


def combine_packed(g, Hq, D, dtype, out=None):
    """Log-sum-exp merge of gathered packed partials ``g [N, Hq * (D + 1)]``
    (each row: o ``[Hq, D]`` then lse ``[Hq]``), read in place."""
    if out is None:
        out = torch.empty((Hq, D), dtype=dtype, device=g.device)
    if g.stride(1) != 1:
        g = g.contiguous()
    with torch.cuda.device(g.device):
        _lib.check(_lib.lib().adakv_combine_packed(g.shape[0], 1, Hq, D, _lib.TORCH_DTYPES[dtype],
                                                   g.data_ptr(), g.stride(0),
                                                   _lib.view4(out.unsqueeze(0)),
                                                   _lib.stream_ptr(g.device)))
    return out


def _concat_scores(gathered, nb, L):
    """``gathered [world, Hq, L]`` (rank r holds blocks [r L, (r + 1) L)) -> ``[Hq, nb]``."""
    world, Hq, _ = gathered.shape
    return gathered.permute(1, 0, 2).reshape(Hq, world * L)[:, :nb].contiguous()


def emulate_step(shards, selector, q, sm_scale=None):
    """One decode step over all shards in one process (no collectives)."""
    L = shards[0].cap
    Hq, D = q.shape
    gathered = torch.zeros((len(shards), Hq, L), dtype=torch.float32, device=q.device)
    for r, sh in enumerate(shards):
        sh.local_scores(q, gathered[r])
    scores = _concat_scores(gathered, selector.nb, L)
    table, sel_lens = selector.select(scores)
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    parts = [sh.attend_partial(q, table, sel_lens, scale) for sh in shards]
    o = torch.stack([p[0] for p in parts])
    lse = torch.stack([p[1] for p in parts])
    return combine(o, lse, q.dtype), table, sel_lens


def emulate_step_stats(shards, selectors, q, sm_scale=None):
    """One decode step over all shards in one process with the statistics
    exchange (``selectors[r]``: shard r's ``StatsSelector``).  Returns the
    output and each rank's ``(table, sel_lens)``."""
    Hq, D = q.shape
    L = shards[0].cap
    world = len(shards)
    scores = torch.zeros((world, Hq, L), dtype=torch.float32, device=q.device)
    recs = []
    for r, (sh, st) in enumerate(zip(shards, selectors)):
        sh.local_scores(q, scores[r])
        recs.append(st.prep(scores[r]).clone())
    records = torch.stack(recs)
    ccs = None
    if selectors[0].adaptive:
        ccs = torch.stack([st.clamp(scores[r], records).clone() for r, st in enumerate(selectors)])
    picks = [tuple(t.clone() for t in st.finish(records, ccs, r)) for r, st in enumerate(selectors)]
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    parts = [sh.attend_partial(q, t, n, scale) for sh, (t, n) in zip(shards, picks)]
    o = torch.stack([p[0] for p in parts])
    lse = torch.stack([p[1] for p in parts])
    return combine(o, lse, q.dtype), picks


class TorchGroup:
    """All-gather over a ``torch.distributed`` process group (NCCL for CUDA tensors)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t, name=None):
        out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        self.dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out


class _DeviceBytes:
    """A device allocation of the library seen by torch (no copy, not owned)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


class PeerGroup:
    """All-gather through peer-mapped memory (``adakv_peer_*``): NVLink stores
    into every rank's buffer and a bounded wait on per-chunk flags, two small
    kernels per call instead of an NCCL collective.

    One buffer per call site (``name``), set up on its first call: a
    ``cudaMalloc``, its IPC handle shared over ``group`` (a collective, so
    every rank makes that first call together, eagerly, before any stream
    capture) and the other ranks' buffers mapped here.  The gathered result
    is a view of this rank's buffer, valid until the next call on the same
    name; every rank must make the same calls in the same order."""

    def __init__(self, group=None, device=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        init = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if init else 1
        self.rank = dist.get_rank(group) if init else 0
        self.device = (torch.device(device) if device is not None
                       else torch.device("cuda", torch.cuda.current_device()))
        self.status = torch.zeros((4,), dtype=torch.int32, device=self.device)
        self._bufs = {}

    def _buffer(self, name, nbytes):
        b = self._bufs.get(name)
        if b is not None:
            if b["slot"] != nbytes:
                raise ValueError(f"peer buffer {name!r} carries {b['slot']} bytes, not {nbytes}")
            return b
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("peer buffers are set up by an eager call before stream capture")
        import ctypes
        L = _lib.lib()
        total = L.adakv_peer_buffer_bytes(self.world, nbytes)
        if total == 0:
            raise ValueError(f"no peer buffer for world {self.world} and {nbytes} bytes per rank")
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        with torch.cuda.device(self.device):
            _lib.check(L.adakv_peer_alloc(total, ctypes.byref(ptr), handle))
            handles = [bytes(handle)]
            if self.world > 1:
                handles = [None] * self.world
                self.dist.all_gather_object(handles, bytes(handle), group=self.group)
            ptrs, opened = [], []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(ptr.value)
                    continue
                q = ctypes.c_void_p()
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r])
                _lib.check(L.adakv_peer_open(hb, ctypes.byref(q)))
                ptrs.append(q.value)
                opened.append(q.value)
        dsts = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        view = torch.as_tensor(_DeviceBytes(ptr.value, self.world * nbytes), device=self.device)
        b = {"slot": nbytes, "local": ptr.value, "dsts": dsts, "opened": opened,
             "view": view.view(self.world, nbytes)}
        self._bufs[name] = b
        return b

    def all_gather(self, t, name=None):
        t = t.contiguous()
        nbytes = t.numel() * t.element_size()
        if nbytes % 16 or t.data_ptr() % 16:
            raise ValueError("peer all-gather payloads are 16-byte multiples, 16-byte aligned")
        b = self._buffer(name or f"bytes{nbytes}", nbytes)
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().adakv_peer_exchange(
                t.data_ptr(), nbytes, b["dsts"].data_ptr(), self.world, self.rank, nbytes,
                b["local"], self.status.data_ptr(), _lib.stream_ptr(self.device)))
        return b["view"].view(t.dtype).view((self.world,) + tuple(t.shape))

    def timed_out(self):
        """True when a wait gave up (ADAKV_ST_WAIT_TIMEOUT); synchronises."""
        return bool(int(self.status[0].item()) & _lib.ST_WAIT_TIMEOUT)

    def close(self):
        """Unmap the other ranks' buffers, then free this rank's (a barrier
        between, so no rank frees memory another still maps)."""
        L = _lib.lib()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for b in self._bufs.values():
                for q in b["opened"]:
                    _lib.check(L.adakv_peer_close(q))
            if self.world > 1:
                self.dist.barrier(group=self.group)
            for b in self._bufs.values():
                b["view"] = None
                _lib.check(L.adakv_peer_free(b["local"]))
        self._bufs = {}


class ShardedDecoder:
    """This rank's part of a sequence-sharded decode step.

    ``K_local``/``V_local``: ``[Hkv, S_local, D]``, the tokens of this rank's
    block range ``shard_range(ceil(S_total / bs), world, rank)``.
    ``selection``: ``"stats"`` (exchange statistics and candidates; fixed and
    adaptive policies), ``"rows"`` (all-gather the score rows; any policy) or
    ``"auto"`` (stats where it applies)."""

    def __init__(self, K_local, V_local, S_total, n_q_heads, block_size, comm, selection="auto",
                 **select_kw):
        self.comm = comm
        self.nb = -(-S_total // block_size)
        self.L = shard_blocks(self.nb, comm.world)
        lo, n = shard_range(self.nb, comm.world, comm.rank)
        if n != -(-K_local.shape[1] // block_size) and K_local.shape[1] > 0:
            raise ValueError("local K/V do not cover this rank's block range")
        self.shard = ShardCache(K_local, V_local, lo, n_q_heads, block_size, capacity_blocks=self.L)
        Hkv, _, D = K_local.shape
        policy = select_kw.get("budget_policy", "adaptive")
        if selection not in ("auto", "stats", "rows"):
            raise ValueError(f"unknown selection exchange {selection!r}")
        use_stats = selection == "stats" or (selection == "auto" and StatsSelector.applies(policy))
        self.stats_sel = self.selector = None
        if use_stats:
            self.stats_sel = StatsSelector(S_total, n_q_heads, Hkv, D, block_size, K_local.dtype,
                                           K_local.device, lo, n, **select_kw)
        else:
            self.selector = Selector(S_total, n_q_heads, Hkv, D, block_size, K_local.dtype,
                                     K_local.device, **select_kw)
        self.scores = torch.zeros((n_q_heads, self.L), dtype=torch.float32, device=K_local.device)

    def select(self):
        """This rank's ``(block table, sel_lens)`` from the current scores."""
        if self.stats_sel is not None:
            s = self.stats_sel
            recs = self.comm.all_gather(s.prep(self.scores), name="records")  # [world, bytes]
            ccs = (self.comm.all_gather(s.clamp(self.scores, recs), name="clamp")
                   if s.adaptive else None)
            return s.finish(recs, ccs, self.comm.rank)
        gathered = self.comm.all_gather(self.scores)                  # [world, Hq, L]
        return self.selector.select(_concat_scores(gathered, self.nb, self.L))

    def step(self, q, sm_scale=None):
        """``q [Hq, D]`` (identical on every rank) -> ``out [Hq, D]`` on every rank."""
        Hq, D = q.shape
        self.shard.local_scores(q, self.scores)
        table, sel_lens = self.select()
        scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
        packed = torch.empty(Hq * D + Hq, dtype=torch.float32, device=q.device)
        self.shard.attend_partial(q, table, sel_lens, scale, packed=packed)
        g = self.comm.all_gather(packed, name="parts")   # [world, Hq * (D + 1)]: (o, lse) per rank
        return combine_packed(g, Hq, D, q.dtype)
