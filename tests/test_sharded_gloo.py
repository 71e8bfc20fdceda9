"""Sequence-sharded decode, host side, as two gloo ranks on CPU.

Each rank scores and attends only the blocks of its shard (NumPy oracle
standing in for the GPU kernels); the product's shard layout
(``shard_range``, ``_concat_scores``) plus all-gathers and a log-sum-exp
merge must reproduce the oracle's single-device step exactly (scores,
selection) and to float32 dot-product rounding (output)."""
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
