"""Sequence-sharded decode on one GPU (shards emulated in one process):
adakv_estimate / adakv_select / adakv_attend_partial / adakv_combine through
the C ABI must select exactly what the single-GPU step selects and produce
the same output; at the cfg4 shape (1M tokens, 64/8 heads) the selection is
also checked against the oracle's budget and top-k on the GPU scores.  The
selection from exchanged statistics (adakv_shard_prep / _clamp / _finish)
is checked against the oracle's budget + top-k on the same score rows, over
1-8 shards, both policies it serves, ties, heavy tails and clamp-dominated
rows, and end to end against the single-GPU step."""
import numpy as np
import pytest
import torch

from adakv_b200 import _lib
from adakv_b200.batch import BatchedDecoder
from adakv_b200.sharded import (Selector, ShardCache, StatsSelector, emulate_step,
                                emulate_step_stats, shard_blocks, shard_range)
from adakv_b200.synth import make_decode_case
from oracle import adakv_oracle as O

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _shards(K, V, nb, world, Hq, bs):
    L = shard_blocks(nb, world)
    out = []
    for r in range(world):
        lo, n = shard_range(nb, world, r)
        t0, t1 = lo * bs, min(K.shape[1], (lo + n) * bs)
        out.append(ShardCache(K[:, t0:t1], V[:, t0:t1], lo, Hq, bs, capacity_blocks=L))
    return out


def _single(K, V, q, S, Hq, bs, **kw):
    Hkv, _, D = K.shape
    dec = BatchedDecoder(1, Hq, Hkv, D, bs, S, K.dtype, "cuda", **kw)
    dec.load(K[None], V[None], [S])
    scores = torch.zeros((Hq, dec.nb_cap), dtype=torch.float32, device="cuda")
    dec.plan(q[None], scores_out=scores)
    sets = [np.sort(s) for s in dec.selected_sets()]
    out = dec.step(q[None])[0].clone()
    return sets, out, scores


@pytest.mark.parametrize("world", [2, 3, 4])
def test_emulated_shards_match_single_gpu(world):
    _need_cuda()
    Hq, Hkv, D, bs, S = 32, 8, 128, 16, 65536 + 7 * 16 + 5
    kw = dict(avg_budget=64, k_min=2, k_max=512)
    case = make_decode_case(31, 1, Hq, Hkv, D, S, bs, "bf16")
    K = torch.from_numpy(case.K[0]).to("cuda", torch.bfloat16)
    V = torch.from_numpy(case.V[0]).to("cuda", torch.bfloat16)
    q = torch.from_numpy(case.q[0]).to("cuda", torch.bfloat16)
    sets1, out1, _ = _single(K, V, q, S, Hq, bs, **kw)
    nb = -(-S // bs)
    shards = _shards(K, V, nb, world, Hq, bs)
    sel = Selector(S, Hq, Hkv, D, bs, torch.bfloat16, "cuda", **kw)
    out, table, sel_lens = emulate_step(shards, sel, q)
    torch.cuda.synchronize()
    bt, sl = table.cpu().numpy(), sel_lens.cpu().numpy()
    for h in range(Hq):
        assert np.array_equal(np.sort(bt[h, : sl[h]]), sets1[h]), f"head {h}"
    err = (out.float() - out1.float()).abs().max().item()
    assert err < BF16_TOL, f"max abs err vs single GPU {err:.3e}"
    # against the oracle at this size too: the selection (up to classified
    # near-ties) and the output over the selected blocks
    ref = O.decode_step(case.q[0], case.K[0], case.V[0], block_size=bs, **kw)
    sets = [bt[h, : sl[h]] for h in range(Hq)]
    _, _, _, fails = O.compare_selection(ref["scores"], ref["k"], ref["raw"], ref["mask"], sets,
                                         1, 4, 1)
    assert not fails, f"selection differs from the oracle: {fails[:3]}"
    mask = np.zeros_like(ref["mask"])
    for h in range(Hq):
        mask[h, sets[h]] = True
    want = O.attend_mask(case.q[0], case.K[0], case.V[0], mask, bs)
    err_o = np.abs(out.float().cpu().numpy() - want).max()
    assert err_o < BF16_TOL, f"max abs err vs oracle {err_o:.3e}"
    exact = np.all(mask == ref["mask"], axis=1)
    assert np.abs(out.float().cpu().numpy()[exact] - ref["out"][exact]).max() < BF16_TOL


def test_cfg4_shape_1m_tokens_sharded_8_ways():
    """cfg4: one 1,048,576-token sequence, 64 q / 8 KV heads, avg_budget 256."""
    _need_cuda()
    Hq, Hkv, D, bs, S = 64, 8, 128, 16, 1 << 20
    kw = dict(avg_budget=256, k_min=2, k_max=1024)
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn((Hq, D), device="cuda", generator=g)
    K = torch.randn((Hkv, S, D), device="cuda", generator=g)
    V = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    nb = S // bs
    # planted retrieval blocks on even KV heads, recency on odd (the synth recipe)
    qm = q.view(Hkv, Hq // Hkv, D).mean(1)
    qhat = qm / qm.norm(dim=-1, keepdim=True)
    for h in range(Hkv):
        if h % 2 == 0:
            for blk in torch.randint(0, nb, (4,), device="cuda", generator=g).tolist():
                K[h, blk * bs:(blk + 1) * bs] += 3.0 * qhat[h]
        else:
            t = torch.arange(S, device="cuda", dtype=torch.float32)
            K[h] += (0.02 * t / 16.0)[:, None] * qhat[h][None, :]
    K = K.to(torch.bfloat16)
    q = q.to(torch.bfloat16)
    sets1, out1, scores = _single(K, V, q, S, Hq, bs, **kw)
    # selection vs the oracle's budget + top-k on the same (GPU) scores
    sc = scores[:, :nb].cpu().numpy().astype(np.float32)
    k, raw = O.allocate_budget(sc, kw["avg_budget"], kw["k_min"], kw["k_max"], 1, 4, 1,
                               return_raw=True)
    mask, _ = O.select_blocks(sc, k, 1, 4, 1)
    n_exact, n_budget, n_score, failures = O.compare_selection(sc, k, raw, mask, sets1, 1, 4, 1)
    assert not failures, failures[:4]
    assert n_exact + n_budget + n_score == Hq
    # 8 emulated shards select the same blocks and give the same output
    shards = _shards(K, V, nb, 8, Hq, bs)
    sel = Selector(S, Hq, Hkv, D, bs, torch.bfloat16, "cuda", **kw)
    out, table, sel_lens = emulate_step(shards, sel, q)
    torch.cuda.synchronize()
    bt, sl = table.cpu().numpy(), sel_lens.cpu().numpy()
    for h in range(Hq):
        assert np.array_equal(np.sort(bt[h, : sl[h]]), sets1[h]), f"head {h}"
    err = (out.float() - out1.float()).abs().max().item()
    assert err < BF16_TOL, f"max abs err vs single GPU {err:.3e}"
    # attention of a few heads against a float64 evaluation over their blocks
    for h in (0, 17, 63):
        blocks = sets1[h]
        tok = (blocks[:, None] * bs + np.arange(bs)[None, :]).ravel()
        kk = K[h // (Hq // Hkv), torch.from_numpy(tok).cuda()].double()
        vv = V[h // (Hq // Hkv), torch.from_numpy(tok).cuda()].double()
        a = (kk @ q[h].double()) / np.sqrt(D)
        ref = torch.softmax(a, 0) @ vv
        e = (out[h].double() - ref).abs().max().item()
        assert e < BF16_TOL, f"head {h}: {e:.3e}"


def test_2m_tokens_plan_reads_rows_from_l2():
    """2,097,152 tokens, 32/8 heads: each plan CTA's slice (65,536 blocks) is
    above the shared-memory staging limit, so the selection reads the score
    rows from L2 (the non-staged plan kernel).  Selection against the oracle's
    budget + top-k on the GPU scores; a few heads' outputs in float64."""
    _need_cuda()
    Hq, Hkv, D, bs, S = 32, 8, 128, 16, 1 << 21
    kw = dict(avg_budget=64, k_min=2, k_max=512)
    g = torch.Generator(device="cuda").manual_seed(6)
    q = torch.randn((Hq, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    nb = S // bs
    for h in range(0, Hkv, 2):  # planted retrieval blocks
        for blk in torch.randint(0, nb, (4,), device="cuda", generator=g).tolist():
            K[h, blk * bs:(blk + 1) * bs] += 3.0 * q[h * (Hq // Hkv)].float().div(
                q[h * (Hq // Hkv)].float().norm()).to(torch.bfloat16)
    sets, out, scores = _single(K, V, q, S, Hq, bs, **kw)
    sc = scores[:, :nb].cpu().numpy()
    k, raw = O.allocate_budget(sc, kw["avg_budget"], kw["k_min"], kw["k_max"], 1, 4, 1,
                               return_raw=True)
    mask, _ = O.select_blocks(sc, k, 1, 4, 1)
    n_exact, n_budget, n_score, failures = O.compare_selection(sc, k, raw, mask, sets, 1, 4, 1)
    assert not failures, failures[:4]
    for h in (0, 21):
        blocks = sets[h]
        tok = torch.from_numpy((blocks[:, None] * bs + np.arange(bs)[None, :]).ravel()).cuda()
        kk = K[h // (Hq // Hkv), tok].double()
        vv = V[h // (Hq // Hkv), tok].double()
        ref = torch.softmax((kk @ q[h].double()) / np.sqrt(D), 0) @ vv
        assert (out[h].double() - ref).abs().max().item() < BF16_TOL


@pytest.mark.parametrize("case", ["floor_miss", "list_overflow", "normal"])
def test_long_slice_selection_paths(case):
    """Score rows long enough (32,768 blocks per plan CTA) for the bucket
    floor and the per-thread candidate lists, shaped so that each path is
    taken: a thin upper tail that leaves fewer blocks above the normal-fit
    floor than the row picks (radix select), a table width so wide that the
    floor drops to mean - sd and the lists overflow (full scan), and plain
    Gaussian rows (compact selection).  adakv_select against the oracle's
    budget + top-k on the same scores."""
    _need_cuda()
    Hq, Hkv, D, bs, S = 64, 8, 128, 16, 1 << 20
    nb = S // bs
    g = torch.Generator(device="cuda").manual_seed(11)
    sc = torch.randn((Hq, nb), device="cuda", generator=g)
    kw = dict(avg_budget=256, k_min=2, k_max=1024)
    if case == "floor_miss":
        # 1 % of the blocks far above the rest: the fit puts the floor above
        # the bulk, and the planted blocks alone are fewer than the budgets
        kw = dict(avg_budget=1000, k_min=900, k_max=1024)
        idx = torch.randint(0, nb, (Hq, nb // 100), device="cuda", generator=g)
        sc.scatter_(1, idx, 100.0 + torch.rand((Hq, nb // 100), device="cuda", generator=g))
    elif case == "list_overflow":
        kw = dict(avg_budget=12000, k_min=2, k_max=16384)
    sel = Selector(S, Hq, Hkv, D, bs, torch.bfloat16, "cuda", **kw)
    table, sel_lens = sel.select(sc)
    torch.cuda.synchronize()
    bt, sl = table.cpu().numpy(), sel_lens.cpu().numpy()
    sets = [np.sort(bt[h, : sl[h]]) for h in range(Hq)]
    s = sc.cpu().numpy().astype(np.float32)
    k, raw = O.allocate_budget(s, kw["avg_budget"], kw["k_min"], kw["k_max"], 1, 4, 1,
                               return_raw=True)
    mask, _ = O.select_blocks(s, k, 1, 4, 1)
    n_exact, n_budget, n_score, failures = O.compare_selection(s, k, raw, mask, sets, 1, 4, 1)
    assert not failures, failures[:4]
    assert n_exact + n_budget + n_score == Hq


class _OneRank:
    """A communicator of one rank (all-gathers are a leading axis of 1)."""
    world, rank = 1, 0

    def all_gather(self, t, name=None):
        return t.unsqueeze(0)


def test_sharded_decoder_one_rank_equals_single_gpu_step():
    """ShardedDecoder.step with one rank (its packed (o, lse) exchange included)
    gives the single-GPU step's selection and output."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from adakv_b200.batch import BatchedDecoder
    from adakv_b200.sharded import ShardedDecoder
    Hq, Hkv, D, bs, S = 32, 8, 128, 16, 20000 + 5
    kw = dict(avg_budget=64, k_min=2, k_max=512)
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn((Hq, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    sd = ShardedDecoder(K, V, S, Hq, bs, _OneRank(), selection="rows", **kw)
    out = sd.step(q)
    ref_dec = BatchedDecoder(1, Hq, Hkv, D, bs, S, torch.bfloat16, "cuda", **kw)
    ref_dec.load(K[None], V[None], [S])
    ref = ref_dec.step(q[None])[0]
    sets = [sd.selector.table[h, : int(sd.selector.sel_lens[h])].cpu().numpy() for h in range(Hq)]
    for a, b in zip(sets, ref_dec.selected_sets()):
        assert np.array_equal(np.sort(a), np.sort(b))
    assert (out.float() - ref.float()).abs().max().item() < 2e-2


def _stats_select(sc, world, kw, bs=16, Hkv=8, D=128):
    """Selection of score rows ``sc [Hq, nb]`` (cuda fp32) split over
    ``world`` emulated ranks through the statistics exchange; returns each
    head's selected global blocks (the union of the ranks' rows)."""
    Hq, nb = sc.shape
    S = nb * bs
    L = shard_blocks(nb, world)
    sels, rows, recs = [], [], []
    for r in range(world):
        lo, n = shard_range(nb, world, r)
        st = StatsSelector(S, Hq, Hkv, D, bs, torch.bfloat16, "cuda", lo, n, **kw)
        row = torch.zeros((Hq, L), dtype=torch.float32, device="cuda")
        row[:, :n] = sc[:, lo:lo + n]
        sels.append(st)
        rows.append(row)
        recs.append(st.prep(row).clone())
    records = torch.stack(recs)
    ccs = None
    if sels[0].adaptive:
        ccs = torch.stack([st.clamp(rows[r], records).clone() for r, st in enumerate(sels)])
    sets = [[] for _ in range(Hq)]
    for r, st in enumerate(sels):
        t, n = st.finish(records, ccs, r)
        t, n = t.cpu().numpy(), n.cpu().numpy()
        lo, cnt = shard_range(nb, world, r)
        assert int(st.status.cpu()[0]) == 0
        for h in range(Hq):
            ids = t[h, : n[h]]
            assert ((ids >= lo) & (ids < lo + cnt)).all(), f"rank {r} head {h}: foreign ids"
            sets[h].extend(ids.tolist())
    out = []
    for h in range(Hq):
        a = np.array(sorted(sets[h]), dtype=np.int64)
        assert len(np.unique(a)) == len(a), f"head {h}: a block selected twice"
        out.append(a)
    return out


def _oracle_check(sc, sets, kw):
    s = sc.cpu().numpy().astype(np.float32)
    k, raw = O.allocate_budget(s, kw["avg_budget"], kw["k_min"], kw["k_max"], 1, 4, 1,
                               kw.get("temperature", 1.0), kw.get("budget_policy", "adaptive"),
                               return_raw=True)
    mask, _ = O.select_blocks(s, k, 1, 4, 1)
    n_exact, n_budget, n_score, failures = O.compare_selection(s, k, raw, mask, sets, 1, 4, 1)
    assert not failures, failures[:4]
    assert n_exact + n_budget + n_score == s.shape[0]
    return n_exact, mask


@pytest.mark.parametrize("world,policy,temperature", [
    (1, "adaptive", 1.0), (2, "adaptive", 1.0), (4, "adaptive", 0.5), (8, "adaptive", 1.0),
    (3, "fixed", 1.0), (8, "fixed", 1.0)])
def test_stats_exchange_selection_matches_oracle(world, policy, temperature):
    """cfg4-sized rows (64 heads x 65,536 blocks, avg_budget 256, k_max
    1024): the union of the ranks' selections against the oracle's budget +
    top-k on the same rows.  One rank holds 65,536 blocks, more than a
    prep CTA stages in shared memory: the rows are read from L2 there."""
    _need_cuda()
    Hq, nb = 64, 65536
    g = torch.Generator(device="cuda").manual_seed(17 + world)
    sc = torch.randn((Hq, nb), device="cuda", generator=g) * 2.0
    kw = dict(avg_budget=256, k_min=2, k_max=1024, budget_policy=policy, temperature=temperature)
    sets = _stats_select(sc, world, kw)
    n_exact, _ = _oracle_check(sc, sets, kw)
    assert n_exact >= Hq - 2


@pytest.mark.parametrize("kind", ["all_equal", "coarse", "heavy_tail", "clamp_window", "tiny"])
def test_stats_exchange_edge_rows(kind):
    """Rows that take the other paths of the shard candidate search: every
    score equal (the exact threshold, ties to the lowest blocks), scores on
    a coarse grid (many ties at the threshold), 1 % of the blocks far above
    the rest (the normal-fit guess misses; bisection), a wide score range
    (most blocks under p = 1e-9, the clamp term decides the budgets), and a
    sequence shorter than one shard per rank."""
    _need_cuda()
    Hq = 32
    g = torch.Generator(device="cuda").manual_seed(23)
    nb, world = 20000, 4
    kw = dict(avg_budget=64, k_min=2, k_max=512)
    if kind == "all_equal":
        sc = torch.zeros((Hq, nb), device="cuda")
    elif kind == "coarse":
        sc = torch.round(torch.randn((Hq, nb), device="cuda", generator=g) * 2.0) / 2.0
    elif kind == "heavy_tail":
        sc = torch.randn((Hq, nb), device="cuda", generator=g)
        idx = torch.randint(0, nb, (Hq, nb // 100), device="cuda", generator=g)
        sc.scatter_(1, idx, 100.0 + torch.rand((Hq, nb // 100), device="cuda", generator=g))
        kw = dict(avg_budget=300, k_min=250, k_max=512)
    elif kind == "clamp_window":
        sc = torch.randn((Hq, nb), device="cuda", generator=g) * 12.0
    else:
        nb, world = 70, 3
        sc = torch.randn((Hq, nb), device="cuda", generator=g)
        kw = dict(avg_budget=8, k_min=2, k_max=64)
    sets = _stats_select(sc, world, kw)
    n_exact, mask = _oracle_check(sc, sets, kw)
    if kind in ("all_equal", "coarse"):
        # exact ties resolve to the lowest blocks, as the oracle's stable order does
        for h in range(Hq):
            assert np.array_equal(sets[h], np.nonzero(mask[h])[0]), f"head {h}"


@pytest.mark.parametrize("world", [2, 3, 4])
def test_stats_exchange_step_matches_single_gpu(world):
    """The whole sharded step with the statistics exchange (emulated ranks)
    against the single-GPU step and the oracle, 64K tokens, 32/8 heads."""
    _need_cuda()
    Hq, Hkv, D, bs, S = 32, 8, 128, 16, 65536 + 7 * 16 + 5
    kw = dict(avg_budget=64, k_min=2, k_max=512)
    case = make_decode_case(31, 1, Hq, Hkv, D, S, bs, "bf16")
    K = torch.from_numpy(case.K[0]).to("cuda", torch.bfloat16)
    V = torch.from_numpy(case.V[0]).to("cuda", torch.bfloat16)
    q = torch.from_numpy(case.q[0]).to("cuda", torch.bfloat16)
    sets1, out1, _ = _single(K, V, q, S, Hq, bs, **kw)
    nb = -(-S // bs)
    shards = _shards(K, V, nb, world, Hq, bs)
    sels = [StatsSelector(S, Hq, Hkv, D, bs, torch.bfloat16, "cuda", sh.block_lo, sh.nb, **kw)
            for sh in shards]
    out, picks = emulate_step_stats(shards, sels, q)
    torch.cuda.synchronize()
    sets = []
    for h in range(Hq):
        ids = np.concatenate([t[h, : int(n[h])].cpu().numpy() for t, n in picks])
        sets.append(np.sort(ids))
    ref = O.decode_step(case.q[0], case.K[0], case.V[0], block_size=bs, **kw)
    _, _, _, fails = O.compare_selection(ref["scores"], ref["k"], ref["raw"], ref["mask"], sets,
                                         1, 4, 1)
    assert not fails, f"selection differs from the oracle: {fails[:3]}"
    same = [np.array_equal(a, b) for a, b in zip(sets, sets1)]
    assert sum(same) >= Hq - 1, "differs from the single-GPU selection beyond a near-tie"
    rows = np.array(same)
    err = (out.float() - out1.float()).abs().max(dim=-1).values.cpu().numpy()
    assert err[rows].max() < BF16_TOL, f"max abs err vs single GPU {err[rows].max():.3e}"
    mask = np.zeros_like(ref["mask"])
    for h in range(Hq):
        mask[h, sets[h]] = True
    want = O.attend_mask(case.q[0], case.K[0], case.V[0], mask, bs)
    assert np.abs(out.float().cpu().numpy() - want).max() < BF16_TOL


def test_sharded_decoder_one_rank_stats_exchange():
    """ShardedDecoder (default: statistics exchange) with one rank, twice:
    the same output both times and the single-GPU step's selection."""
    _need_cuda()
    from adakv_b200.sharded import ShardedDecoder
    Hq, Hkv, D, bs, S = 32, 8, 128, 16, 20000 + 5
    kw = dict(avg_budget=64, k_min=2, k_max=512)
    g = torch.Generator(device="cuda").manual_seed(11)
    q = torch.randn((Hq, D), device="cuda", generator=g).to(torch.bfloat16)
    K = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    sd = ShardedDecoder(K, V, S, Hq, bs, _OneRank(), **kw)
    assert sd.stats_sel is not None
    out = sd.step(q)
    out2 = sd.step(q)
    assert torch.equal(out, out2)
    sets1, out1, _ = _single(K, V, q, S, Hq, bs, **kw)
    st = sd.stats_sel
    sets = [np.sort(st.table[h, : int(st.sel_lens[h])].cpu().numpy()) for h in range(Hq)]
    same = [np.array_equal(a, b) for a, b in zip(sets, sets1)]
    assert sum(same) >= Hq - 1
    err = (out.float() - out1.float()).abs().max(dim=-1).values.cpu().numpy()
    assert err[np.array(same)].max() < BF16_TOL


def test_peer_group_one_rank_gathers_and_matches_the_decoder():
    """PeerGroup with one rank (no process group): the exchange kernels copy
    the payload into the rank's own slot, twice in a row with different
    payloads, and ShardedDecoder over it equals the plain one-rank path."""
    _need_cuda()
    from adakv_b200.sharded import PeerGroup, ShardedDecoder
    pg = PeerGroup()
    try:
        for k in range(2):
            x = torch.arange(1024, dtype=torch.float32, device="cuda") * (k + 1)
            y = pg.all_gather(x, name="t")
            torch.cuda.synchronize()
            assert y.shape == (1, 1024) and torch.equal(y[0], x)
        assert not pg.timed_out()
        Hq, Hkv, D, bs, S = 32, 8, 128, 16, 20000 + 5
        kw = dict(avg_budget=64, k_min=2, k_max=512)
        g = torch.Generator(device="cuda").manual_seed(11)
        q = torch.randn((Hq, D), device="cuda", generator=g).to(torch.bfloat16)
        K = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
        V = torch.randn((Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
        a = ShardedDecoder(K, V, S, Hq, bs, pg, **kw).step(q)
        b = ShardedDecoder(K, V, S, Hq, bs, _OneRank(), **kw).step(q)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
        assert not pg.timed_out()
    finally:
        pg.close()
