"""Sequence-sharded decode, host side, as gloo ranks on CPU.

Each rank scores and attends only the blocks of its shard (NumPy oracle
standing in for the GPU kernels); the product's shard layout
(``shard_range``, ``_concat_scores``) plus all-gathers and a log-sum-exp
merge must reproduce the oracle's single-device step exactly (scores,
selection) and to float32 dot-product rounding (output).

The selection from exchanged statistics (``StatsSelector``: per-head
softmax statistics and sorted shard candidates, then clamp terms) is
modelled here in NumPy, float64, step for step as the three shard kernels
compute it, and run as 2, 3 and 4 gloo ranks: the union of the ranks' picks
must equal the oracle's selection on the whole rows (up to classified
near-ties)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from adakv_b200.sharded import _concat_scores, shard_blocks, shard_range
from adakv_b200.synth import make_decode_case
from oracle import adakv_oracle as O

Hq, Hkv, D, BS, S = 8, 2, 64, 16, 1500 * 16 + 7  # nb = 1501: a partial tail block


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial(q, K, V, mask, lo, n, scale):
    """(o, lse) of every head over its selected blocks in [lo, lo + n)."""
    Hq_, D_ = q.shape
    g = Hq_ // K.shape[0]
    o = np.zeros((Hq_, D_))
    lse = np.full(Hq_, -np.inf)
    for h in range(Hq_):
        blocks = [b for b in np.nonzero(mask[h])[0] if lo <= b < lo + n]
        if not blocks:
            continue
        tok = (np.array(blocks)[:, None] * BS + np.arange(BS)[None, :]).ravel()
        tok = tok[tok < K.shape[1]]
        a = (K[h // g, tok].astype(np.float64) @ q[h].astype(np.float64)) * scale
        m = a.max()
        w = np.exp(a - m)
        o[h] = w @ V[h // g, tok].astype(np.float64) / w.sum()
        lse[h] = m + np.log(w.sum())
    return o, lse


def _rank(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = make_decode_case(5, 1, Hq, Hkv, D, S, BS, "fp32")
        q, K, V = case.q[0], case.K[0], case.V[0]
        nb = -(-S // BS)
        L = shard_blocks(nb, world)
        lo, n = shard_range(nb, world, rank)
        # 1. this rank's scores (its tokens only), padded to L blocks
        Kl = K[:, lo * BS: min(S, (lo + n) * BS)]
        mine = np.zeros((Hq, L), dtype=np.float32)
        mine[:, :n] = O.block_scores(q, O.build_centroids(Kl, BS))
        gathered = [torch.zeros((Hq, L)) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(mine))
        scores = _concat_scores(torch.stack(gathered), nb, L).numpy()
        full = O.block_scores(q, O.build_centroids(K, BS))
        assert np.array_equal(scores, full)
        # 2. selection on the full rows: what every rank computes
        k = O.allocate_budget(scores, 12, 2, 64, 1, 4, 1)
        mask, _ = O.select_blocks(scores, k, 1, 4, 1)
        # 3. partial attention over this rank's blocks, gathered and merged
        o, lse = _partial(q, K, V, mask, lo, n, 1.0 / np.sqrt(D))
        po = [torch.zeros((Hq, D), dtype=torch.float64) for _ in range(world)]
        pl = [torch.zeros((Hq,), dtype=torch.float64) for _ in range(world)]
        dist.all_gather(po, torch.from_numpy(o))
        dist.all_gather(pl, torch.from_numpy(lse))
        P, Ls = torch.stack(po).numpy(), torch.stack(pl).numpy()
        M = Ls.max(axis=0)
        wts = np.where(np.isfinite(Ls), np.exp(Ls - M), 0.0)
        out = (wts[:, :, None] * P).sum(0) / wts.sum(0)[:, None]
        ref = O.attend_mask(q, K, V, mask, BS)
        q_out.put((rank, float(np.abs(out - ref).max()), int(mask.sum())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_decomposition_two_gloo_ranks(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, f"rank exit codes {codes}"
    res = sorted(q.get(timeout=5) for _ in range(world))
    assert all(err < 1e-6 for _, err, _ in res), res  # oracle dots are float32
    assert len({sel for _, _, sel in res}) == 1  # every rank selected the same blocks


def _np_prep(sc, lo, nb, cap, T, sink=1, local=4):
    """Stage 0 of one shard: (M, Z, A) of z = s / T per head and the top
    ``cap`` content blocks as (score, global id), score desc then id asc."""
    Hq, n = sc.shape
    gi = lo + np.arange(n)
    content = (gi >= sink) & (gi < nb - local)
    z = sc.astype(np.float64) / max(T, 1e-6)
    if n:
        M = z.max(axis=1)
        e = np.exp(z - M[:, None])
        Z, A = e.sum(1), (e * (z - M[:, None])).sum(1)
    else:
        M, Z, A = np.full(Hq, -np.inf), np.zeros(Hq), np.zeros(Hq)
    cands = []
    for h in range(Hq):
        ids, s = gi[content], sc[h, content].astype(np.float64)
        order = np.lexsort((ids, -s))
        take = order[: min(cap, len(ids))]
        cands.append((s[take], ids[take]))
    return M, Z, A, cands


def _merge_mz(recs):
    M = np.max([r[0] for r in recs], axis=0)
    Z = sum(np.where(np.isfinite(r[0]), r[1] * np.exp(r[0] - M), 0.0) for r in recs)
    A = sum(np.where(np.isfinite(r[0]), np.exp(r[0] - M) * (r[2] + r[1] * (r[0] - M)), 0.0)
            for r in recs)
    return M, Z, A


def _np_clamp(sc, T, M, Z):
    """Stage 1: this shard's sum over blocks with p < 1e-9 of
    e (log 1e-9 - (z - M) + log Z), e = exp(z - M)."""
    d = sc.astype(np.float64) / max(T, 1e-6) - M[:, None]
    e = np.exp(d)
    win = e / Z[:, None] < 1e-9
    return np.where(win, e * (np.log(1e-9) - d + np.log(Z)[:, None]), 0.0).sum(1)


def _np_finish(recs, ccs, me, lo, n, nb, kw):
    """Stage 2: budgets from the merged statistics, then this rank's picks
    (its forced blocks and its candidates whose merged position is < Kc)."""
    Hq = len(recs[0][3])
    M, Z, A = _merge_mz(recs)
    H = np.log(Z) - A / Z - sum(ccs) / Z
    w = H / np.log(max(nb, 2)) + 1e-6
    lo_b, hi_b, target = O.budget_bounds(nb, kw["avg"], kw["k_min"], kw["k_max"], 1, 4, 1)
    extra = max(target - lo_b, 0.0) * Hq * w / max(float(w.sum()), 1e-9)
    k = np.clip(np.round(lo_b + extra), lo_b, hi_b).astype(np.int64)
    kh = O.selection_counts(k, nb, 1, 4, 1)
    n_forced = min(1 + 4, nb)
    picks = []
    for h in range(Hq):
        kc = int(kh[h]) - n_forced
        s_me, id_me = recs[me][3][h]
        mine = [b for b in range(lo, lo + n) if b < 1 or b >= nb - 4]
        for j in range(len(id_me)):
            rank = j
            for r, rec in enumerate(recs):
                if r != me:
                    s_r, id_r = rec[3][h]
                    rank += int(np.sum((s_r > s_me[j]) | ((s_r == s_me[j]) & (id_r < id_me[j]))))
            if rank < kc:
                mine.append(int(id_me[j]))
        picks.append(mine)
    return picks


def _stats_rank(rank, world, port, q_out, kw):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = make_decode_case(5, 1, Hq, Hkv, D, S, BS, "fp32")
        q, K = case.q[0], case.K[0]
        nb = -(-S // BS)
        lo, n = shard_range(nb, world, rank)
        sc = O.block_scores(q, O.build_centroids(K[:, lo * BS: min(S, (lo + n) * BS)], BS))
        cap = min(kw["k_max"], nb) - 5
        rec = _np_prep(sc, lo, nb, cap, kw["T"])
        recs = [None] * world
        dist.all_gather_object(recs, rec)
        M, Z, _ = _merge_mz(recs)
        ccs = [None] * world
        dist.all_gather_object(ccs, _np_clamp(sc, kw["T"], M, Z))
        picks = _np_finish(recs, ccs, rank, lo, n, nb, kw)
        allp = [None] * world
        dist.all_gather_object(allp, picks)
        if rank == 0:
            full = O.block_scores(q, O.build_centroids(K, BS))
            k, raw = O.allocate_budget(full, kw["avg"], kw["k_min"], kw["k_max"], 1, 4, 1,
                                       kw["T"], return_raw=True)
            mask, _ = O.select_blocks(full, k, 1, 4, 1)
            sets = [np.array(sorted(sum((p[h] for p in allp), []))) for h in range(Hq)]
            n_exact, n_b, n_s, fails = O.compare_selection(full, k, raw, mask, sets, 1, 4, 1)
            q_out.put((n_exact, n_b, n_s, len(fails)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T", [(2, 1.0), (3, 0.7), (4, 1.0)])
def test_stats_exchange_decomposition_gloo_ranks(world, T):
    kw = dict(avg=12, k_min=2, k_max=64, T=T)
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_stats_rank, args=(r, world, port, q, kw)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    assert [p.exitcode for p in procs] == [0] * world
    n_exact, n_b, n_s, n_fail = q.get(timeout=5)
    assert n_fail == 0 and n_exact + n_b + n_s == Hq
    assert n_exact >= Hq - 1


def test_shard_ranges_cover_the_sequence_once():
    for nb in (1, 31, 32, 33, 1501, 65536):
        for world in (1, 2, 3, 4, 8):
            L = shard_blocks(nb, world)
            assert L % 32 == 0
            covered = []
            for r in range(world):
                lo, n = shard_range(nb, world, r)
                assert lo % 32 == 0 or n == 0
                covered.extend(range(lo, lo + n))
            assert covered == list(range(nb))


def test_partition_batch_is_contiguous_and_balanced():
    from adakv_b200.batch import partition_batch
    from adakv_b200.synth import ragged_seq_lens
    lens = ragged_seq_lens(0, 64, 8192, 131072)
    for world in (1, 2, 4, 8):
        parts = partition_batch(lens, world)
        assert parts[0][0] == 0 and parts[-1][1] == 64
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        sums = [int(lens[a:b].sum()) for a, b in parts]
        assert max(sums) - min(sums) <= int(lens.max())  # within one sequence of balance
