"""CUDA path vs the NumPy oracle on identical seeded inputs (needs a B200).

Bars (from the task's parity contract):
* centroid tables: bit-exact (same float32 token-order sums and division);
* block selection: identical block sets per head, except documented near-ties
  (score gap < 1e-6 relative; budget rounding within 1e-4 of a .5 boundary);
* attention outputs: 1e-3 abs for fp32 inputs, 2e-2 abs for bf16 inputs.
Everything calls the C ABI (through the package's ctypes binding).
"""
from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from adakv_b200 import _lib  # noqa: E402
from adakv_b200.batch import BatchedDecoder  # noqa: E402
from adakv_b200.synth import make_decode_case, ragged_seq_lens  # noqa: E402
from oracle import adakv_oracle as O  # noqa: E402

TOL = {"fp32": 1e-3, "bf16": 2e-2, "fp16": 2e-2}
TORCH = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")


def _decoder(case, Hq, Hkv, D, avg=8, k_min=2, k_max=64, sink=1, local=4, c_min=1, T=1.0,
             policy="adaptive", capacity=None):
    B = case.q.shape[0]
    cap = capacity or int(case.seq_lens.max())
    dec = BatchedDecoder(B, Hq, Hkv, D, case.block_size, cap, TORCH[case.dtype], "cuda",
                         avg_budget=avg, k_min=k_min, k_max=k_max, n_sink_blocks=sink,
                         n_local_blocks=local, c_min=c_min, temperature=T, budget_policy=policy)
    dt = TORCH[case.dtype]
    K = torch.from_numpy(case.K).to("cuda", dt)
    V = torch.from_numpy(case.V).to("cuda", dt)
    dec.load(K, V, case.seq_lens)
    q = torch.from_numpy(case.q).to("cuda", dt)
    return dec, q


def _oracle_seq(case, b, **kw):
    S = int(case.seq_lens[b])
    return O.decode_step(case.q[b], case.K[b, :, :S], case.V[b, :, :S],
                         block_size=case.block_size, **kw)


def _check_selection(res, sets, kw, label):
    n_exact, n_budget, n_score, fails = O.compare_selection(
        res["scores"], res["k"], res["raw"], res["mask"], sets, kw["n_sink_blocks"],
        kw["n_local_blocks"], kw["c_min"])
    assert not fails, f"{label}: selection mismatch {fails[:3]}"
    return n_exact, n_budget, n_score


# ---------------------------------------------------------------------------
# (a) centroids
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,D,bs,S", [("fp32", 128, 16, 4096), ("bf16", 128, 16, 4001),
                                          ("fp16", 64, 32, 1000), ("bf16", 64, 16, 17)])
def test_centroid_build_bit_exact(dtype, D, bs, S):
    _need_cuda()
    case = make_decode_case(21, 2, 8, 2, D, [S, max(S - 37, 1)], bs, dtype)
    dec, _ = _decoder(case, 8, 2, D)
    got = dec.centroid.cpu().numpy()
    for b in range(2):
        Sb = int(case.seq_lens[b])
        ref = O.build_centroids(case.K[b, :, :Sb], bs)
        np.testing.assert_array_equal(got[b, :, : ref.shape[1]], ref)


def test_append_refresh_bit_exact():
    _need_cuda()
    D, bs, S0 = 128, 16, 100
    case = make_decode_case(22, 2, 8, 4, D, S0, bs, "bf16")
    dec, _ = _decoder(case, 8, 4, D, capacity=S0 + 80)
    rng = np.random.default_rng(5)
    K = case.K.copy()
    V = case.V.copy()
    for step in range(40):
        n = 1 if step % 5 else 3
        kn = rng.standard_normal((2, 4, n, D)).astype(np.float32)
        vn = rng.standard_normal((2, 4, n, D)).astype(np.float32)
        kt = torch.from_numpy(kn).to("cuda", torch.bfloat16)
        vt = torch.from_numpy(vn).to("cuda", torch.bfloat16)
        dec.append(kt, vt)
        K = np.concatenate([K, kt.float().cpu().numpy()], axis=2)
        V = np.concatenate([V, vt.float().cpu().numpy()], axis=2)
    S = dec.host_seq_lens[0]
    assert S == K.shape[2]
    got_c = dec.centroid.cpu().numpy()
    for b in range(2):
        ref = O.build_centroids(K[b], bs)
        np.testing.assert_array_equal(got_c[b, :, : ref.shape[1]], ref)
    np.testing.assert_array_equal(dec.k[:, :, :S].float().cpu().numpy(), K)
    np.testing.assert_array_equal(dec.v[:, :, :S].float().cpu().numpy(), V)
    assert dec.status() == 0


# ---------------------------------------------------------------------------
# (b)(c) estimator + budget + selection
# ---------------------------------------------------------------------------
PLAN_CASES = [
    # (seed, Hq, Hkv, D, S, bs, dtype, kw)
    (0, 32, 8, 128, 4096, 16, "fp32", dict(avg_budget=8, k_min=2, k_max=64)),
    (1, 8, 2, 128, 4001, 16, "fp32", dict(avg_budget=12, k_min=2, k_max=64)),
    (3, 12, 2, 64, 320, 16, "fp32", dict(avg_budget=8, k_min=2, k_max=256, n_local_blocks=2)),
    (4, 4, 4, 64, 8192, 32, "fp32", dict(avg_budget=16, k_min=2, k_max=64)),
    (6, 8, 2, 64, 10, 16, "fp32", dict(avg_budget=8, k_min=2, k_max=64)),
    (7, 8, 2, 64, 20, 16, "fp32", dict(avg_budget=8, k_min=2, k_max=64)),
    (8, 8, 2, 64, 100, 16, "fp32", dict(avg_budget=5, k_min=2, k_max=64)),
    (9, 32, 8, 128, 8192, 16, "bf16", dict(avg_budget=64, k_min=2, k_max=512)),
    (10, 16, 4, 128, 2048, 16, "fp32", dict(avg_budget=16, k_min=2, k_max=128, temperature=0.5)),
    (11, 32, 8, 128, 4096, 16, "fp32", dict(avg_budget=32, k_min=2, k_max=16)),
    (12, 32, 8, 128, 32768, 16, "bf16", dict(avg_budget=64, k_min=2, k_max=512)),
    (13, 64, 8, 128, 16384, 16, "bf16", dict(avg_budget=64, k_min=2, k_max=512)),
    (14, 16, 4, 128, 4096, 16, "fp16", dict(avg_budget=24, k_min=2, k_max=64,
                                             budget_policy="fixed")),
]


def _full_kw(kw):
    k = dict(n_sink_blocks=1, n_local_blocks=4, c_min=1, temperature=1.0, budget_policy="adaptive")
    k.update(kw)
    return k


@pytest.mark.parametrize("seed,Hq,Hkv,D,S,bs,dtype,kw", PLAN_CASES)
def test_plan_matches_oracle(seed, Hq, Hkv, D, S, bs, dtype, kw):
    _need_cuda()
    kw = _full_kw(kw)
    case = make_decode_case(seed, 1, Hq, Hkv, D, S, bs, dtype)
    dec, q = _decoder(case, Hq, Hkv, D, avg=kw["avg_budget"], k_min=kw["k_min"], k_max=kw["k_max"],
                      sink=kw["n_sink_blocks"], local=kw["n_local_blocks"], c_min=kw["c_min"],
                      T=kw["temperature"], policy=kw["budget_policy"])
    scores = torch.zeros((1, Hq, dec.nb_cap), dtype=torch.float32, device="cuda")
    dec.plan(q, scores_out=scores)
    res = _oracle_seq(case, 0, avg_budget=kw["avg_budget"], k_min=kw["k_min"], k_max=kw["k_max"],
                      n_sink_blocks=kw["n_sink_blocks"], n_local_blocks=kw["n_local_blocks"],
                      c_min=kw["c_min"], temperature=kw["temperature"],
                      policy=kw["budget_policy"])
    nb = res["scores"].shape[1]
    got = scores[0, :, :nb].cpu().numpy()
    err = np.abs(got.astype(np.float64) - res["scores"])
    scale = np.abs(res["scores"]).max(axis=1, keepdims=True) + 1e-30
    assert (err / scale).max() < 2e-6, f"score rel err {(err / scale).max():.3e}"
    sets = dec.selected_sets()
    n_exact, n_budget, n_score = _check_selection(res, sets, kw, f"seed {seed}")
    assert n_exact + n_budget + n_score == Hq
    assert n_budget + n_score <= max(1, Hq // 16), "too many near-ties"
    for s in sets:
        assert np.all(np.diff(s) > 0), "rows must be ascending and duplicate-free"
    assert dec.status() == 0


def test_plan_batched_ragged():
    _need_cuda()
    lens = [4096, 1000, 2500, 17, 3333]
    Hq, Hkv, D, bs = 16, 4, 128, 16
    case = make_decode_case(30, len(lens), Hq, Hkv, D, lens, bs, "bf16")
    kw = _full_kw(dict(avg_budget=24, k_min=2, k_max=128))
    dec, q = _decoder(case, Hq, Hkv, D, avg=24, k_max=128)
    dec.plan(q)
    sets = dec.selected_sets()
    for b in range(len(lens)):
        res = _oracle_seq(case, b, avg_budget=24, k_min=2, k_max=128)
        _check_selection(res, sets[b * Hq:(b + 1) * Hq], kw, f"seq {b}")
    assert dec.status() == 0


# ---------------------------------------------------------------------------
# (d) attention over a given table
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,D,bs,Hq,Hkv,S", [("fp32", 128, 16, 32, 8, 4096),
                                                 ("bf16", 128, 16, 32, 8, 4096),
                                                 ("fp16", 64, 32, 4, 4, 8192),
                                                 ("bf16", 128, 32, 16, 2, 1000),
                                                 ("fp32", 64, 16, 12, 2, 333)])
def test_attend_table_matches_oracle(dtype, D, bs, Hq, Hkv, S):
    _need_cuda()
    case = make_decode_case(40, 1, Hq, Hkv, D, S, bs, dtype)
    nb = (S + bs - 1) // bs
    rng = np.random.default_rng(41)
    width = min(nb, 37)
    table = np.zeros((Hq, width), dtype=np.int32)
    lens = rng.integers(0, width + 1, size=Hq).astype(np.int32)
    lens[0] = width
    lens[1] = 0                      # empty row -> zeros
    for h in range(Hq):
        table[h] = rng.permutation(nb)[:width]
    perm = rng.permutation(nb - 1)   # row 0 starts with the partial tail block, no duplicates
    table[0] = np.concatenate([[nb - 1], perm[: width - 1]])
    from adakv_b200.kernels.block_sparse_decode import block_sparse_decode
    dt = TORCH[dtype]
    q = torch.from_numpy(case.q[0]).to("cuda", dt)
    K = torch.from_numpy(case.K[0]).to("cuda", dt)
    V = torch.from_numpy(case.V[0]).to("cuda", dt)
    out = block_sparse_decode(q, K, V, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(),
                              bs)
    ref = O.attend_table(case.q[0], case.K[0], case.V[0], table, lens, bs)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err < TOL[dtype], f"max abs err {err:.3e}"
    assert np.all(out[1].float().cpu().numpy() == 0)


def test_attend_strided_views_and_scale():
    _need_cuda()
    Hq, Hkv, D, S, bs = 8, 2, 128, 777, 16
    case = make_decode_case(42, 1, Hq, Hkv, D, S, bs, "bf16")
    big = torch.zeros((Hkv, S + 64, D), dtype=torch.bfloat16, device="cuda")
    big[:, :S] = torch.from_numpy(case.K[0]).to("cuda", torch.bfloat16)
    K = big[:, :S]                               # strided view (stride_h = (S+64)*D)
    V = torch.from_numpy(case.V[0]).to("cuda", torch.bfloat16)
    q = torch.from_numpy(case.q[0]).to("cuda", torch.bfloat16)
    nb = (S + bs - 1) // bs
    table = np.stack([np.arange(nb)[::-1][:12] for _ in range(Hq)]).astype(np.int32)
    lens = np.full(Hq, 12, dtype=np.int32)
    from adakv_b200.kernels.block_sparse_decode import block_sparse_decode
    out = block_sparse_decode(q, K, V, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(),
                              bs, sm_scale=0.05)
    ref = O.attend_table(case.q[0], case.K[0], case.V[0], table, lens, bs, sm_scale=0.05)
    assert np.abs(out.float().cpu().numpy() - ref).max() < TOL["bf16"]


def test_attend_flags_bad_block_ids():
    _need_cuda()
    Hq, Hkv, D, S, bs = 4, 1, 64, 64, 16
    case = make_decode_case(43, 1, Hq, Hkv, D, S, bs, "fp32")
    table = np.array([[0, 1, 2, 3], [0, 9, 1, 2], [3, 2, -1, 0], [1, 1, 1, 1]], dtype=np.int32)
    lens = np.array([4, 4, 4, 1], dtype=np.int32)
    from adakv_b200.kernels.block_sparse_decode import block_sparse_decode
    q = torch.from_numpy(case.q[0]).cuda()
    K = torch.from_numpy(case.K[0]).cuda()
    V = torch.from_numpy(case.V[0]).cuda()
    out = block_sparse_decode(q, K, V, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(),
                              bs)
    torch.cuda.synchronize()
    ws = _lib.workspace(0, q.device, "attend")
    assert _lib.read_status(ws) & _lib.ST_BAD_BLOCK_ID
    # the valid entries are still attended
    good = np.array([[0, 1, 2, 3], [0, 1, 2, 2], [3, 2, 0, 0], [1, 1, 1, 1]], dtype=np.int32)
    glens = np.array([4, 3, 3, 1], dtype=np.int32)
    ref = O.attend_table(case.q[0], case.K[0], case.V[0], good, glens, bs)
    assert np.abs(out.cpu().numpy() - ref).max() < TOL["fp32"]


# ---------------------------------------------------------------------------
# full decode step
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("seed,Hq,Hkv,S,dtype,avg,kmax", [(0, 32, 8, 4096, "fp32", 8, 64),
                                                          (12, 32, 8, 32768, "bf16", 64, 512),
                                                          (15, 64, 8, 8192, "bf16", 64, 512)])
def test_decode_step_matches_oracle(seed, Hq, Hkv, S, dtype, avg, kmax):
    _need_cuda()
    D, bs = 128, 16
    case = make_decode_case(seed, 1, Hq, Hkv, D, S, bs, dtype)
    dec, q = _decoder(case, Hq, Hkv, D, avg=avg, k_max=kmax)
    out = dec.step(q).float().cpu().numpy()[0]
    res = _oracle_seq(case, 0, avg_budget=avg, k_min=2, k_max=kmax)
    kw = _full_kw(dict(avg_budget=avg, k_min=2, k_max=kmax))
    n_exact, n_budget, n_score = _check_selection(res, dec.selected_sets(), kw, "step")
    # compare against the oracle's attention over the GPU's own selection (differs from
    # res["out"] only for near-tie heads) and against res["out"] on exact heads
    sets = dec.selected_sets()
    mask = np.zeros_like(res["mask"])
    for h in range(Hq):
        mask[h, sets[h]] = True
    ref = O.attend_mask(case.q[0], case.K[0], case.V[0], mask, bs)
    err = np.abs(out - ref).max()
    assert err < TOL[dtype], f"max abs err {err:.3e}"
    exact = np.all(mask == res["mask"], axis=1)
    assert np.abs(out[exact] - res["out"][exact]).max() < TOL[dtype]
    assert dec.status() == 0


def test_decode_step_batched_ragged():
    _need_cuda()
    lens = ragged_seq_lens(3, 4, 1000, 9000).tolist()
    Hq, Hkv, D, bs = 32, 8, 128, 16
    case = make_decode_case(31, len(lens), Hq, Hkv, D, lens, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, D, avg=32, k_max=256)
    out = dec.step(q).float().cpu().numpy()
    sets = dec.selected_sets()
    kw = _full_kw(dict(avg_budget=32, k_min=2, k_max=256))
    for b, S in enumerate(lens):
        res = _oracle_seq(case, b, avg_budget=32, k_min=2, k_max=256)
        _check_selection(res, sets[b * Hq:(b + 1) * Hq], kw, f"seq {b}")
        mask = np.zeros_like(res["mask"])
        for h in range(Hq):
            mask[h, sets[b * Hq + h]] = True
        ref = O.attend_mask(case.q[b], case.K[b, :, :S], case.V[b, :, :S], mask, bs)
        assert np.abs(out[b] - ref).max() < TOL["bf16"]
    assert dec.status() == 0


def test_repeated_steps_are_deterministic():
    _need_cuda()
    case = make_decode_case(16, 1, 32, 8, 128, 16384, 16, "bf16")
    dec, q = _decoder(case, 32, 8, 128, avg=64, k_max=512)
    a = dec.step(q).clone()
    sets_a = dec.selected_sets()
    for _ in range(3):
        b = dec.step(q)
    assert torch.equal(a, b)
    for x, y in zip(sets_a, dec.selected_sets()):
        np.testing.assert_array_equal(x, y)


# ---------------------------------------------------------------------------
# reference-facing operator API
# ---------------------------------------------------------------------------
def test_reference_api_shapes_and_semantics():
    _need_cuda()
    from adakv_b200.attention import AdaKVCache, adakv_decode_attention, plan_selection
    from adakv_b200.runtime import adakv_decode_step, update_cache_decode
    Hkv, g, S, D, bs = 4, 2, 512, 64, 16
    Hq = Hkv * g
    case = make_decode_case(50, 1, Hq, Hkv, D, S, bs, "fp32")
    q = torch.from_numpy(case.q[0]).cuda()
    k = torch.from_numpy(case.K[0]).cuda()
    v = torch.from_numpy(case.V[0]).cuda()
    cache = AdaKVCache(block_size=bs).append_prefill(k, v)
    assert cache.centroid.shape == (Hkv, S // bs, D) and cache.centroid.dtype == torch.float32
    bt, sl = plan_selection(q, cache, avg_budget=6, n_sink_blocks=2, n_local_blocks=3)
    assert bt.dtype == torch.int32 and sl.dtype == torch.int32 and sl.shape == (Hq,)
    nb = S // bs
    for h in range(Hq):
        ids = set(bt[h, : int(sl[h])].tolist())
        assert {0, 1, nb - 3, nb - 2, nb - 1} <= ids, "sink + local blocks are forced"
    # the reference's table format (attention.py:229-244): width max_sel, forced
    # blocks first, then descending score
    assert bt.shape[1] == int(sl.max())
    ref_scores = O.block_scores(case.q[0], O.build_centroids(case.K[0], bs))
    for h in range(Hq):
        row = bt[h, : int(sl[h])].tolist()
        assert row[:5] == [0, 1, nb - 3, nb - 2, nb - 1], row[:6]
        sc = ref_scores[h, row[5:]]
        assert np.all(np.diff(sc) <= 1e-6 * max(np.abs(sc).max(), 1e-30)), "not descending"
    bta, sla = plan_selection(q, cache, avg_budget=6, n_sink_blocks=2, n_local_blocks=3,
                              order="ascending")
    assert torch.equal(sla, sl)
    for h in range(Hq):
        assert sorted(bt[h, : int(sl[h])].tolist()) == bta[h, : int(sl[h])].tolist()
    # full budget == dense attention
    out = adakv_decode_attention(q, cache, avg_budget=nb, k_min=nb, k_max=nb)
    dense = O.dense_attention(case.q[0], case.K[0], case.V[0])
    assert np.abs(out.cpu().numpy() - dense).max() < 1e-4
    out4 = adakv_decode_step(q[None, :, None, :], cache, avg_budget=nb, k_min=nb, k_max=nb)
    assert out4.shape == (1, Hq, 1, D)
    # decode loop with in-place appends stays equal to dense
    for _ in range(20):
        kt = torch.randn(Hkv, 1, D, device="cuda")
        vt = torch.randn(Hkv, 1, D, device="cuda")
        update_cache_decode(cache, kt, vt)
        qs = torch.randn(1, Hq, 1, D, device="cuda")
        nbn = cache.centroid.shape[1]
        o = adakv_decode_step(qs, cache, avg_budget=nbn, k_min=nbn, k_max=nbn)
        d = O.dense_attention(qs[0, :, 0].cpu().numpy(), cache.k.cpu().numpy(),
                              cache.v.cpu().numpy())
        assert np.abs(o[0, :, 0].cpu().numpy() - d).max() < 1e-4
    rebuilt = AdaKVCache(block_size=bs).append_prefill(cache.k.contiguous(), cache.v.contiguous())
    assert torch.equal(rebuilt.centroid, cache.centroid)
    with pytest.raises(ValueError):
        plan_selection(q, cache, 8, estimator="bogus")
    with pytest.raises(ValueError):
        plan_selection(q, cache, 8, budget_policy="bogus")


def test_budget_trace_and_recall_instruments():
    _need_cuda()
    from adakv_b200 import attention as A
    case = make_decode_case(51, 1, 12, 2, 64, 320, 16, "fp32")
    q = torch.from_numpy(case.q[0]).cuda()
    cache = A.AdaKVCache(16).append_prefill(torch.from_numpy(case.K[0]).cuda(),
                                            torch.from_numpy(case.V[0]).cuda())
    A.reset_budget_trace()
    A.set_recall_target([0])
    for _ in range(3):
        A.plan_selection(q, cache, 8, n_local_blocks=2, k_max=256)
    tr = A.get_budget_trace()
    r = A.get_recall()
    A.stop_budget_trace()
    A.clear_recall_target()
    assert len(tr) == 3 and all(t > 0 for t in tr)
    assert r == 1.0  # the sink block is always covered


def test_fused_append_step_equals_separate_append():
    """The step with new tokens (append fused into the estimator) must equal a
    stand-alone append followed by a plain step, bit for bit."""
    _need_cuda()
    lens = [5000, 3001]
    case = make_decode_case(60, 2, 32, 8, 128, lens, 16, "bf16")
    dec_a, q = _decoder(case, 32, 8, 128, avg=32, k_max=256, capacity=5100)
    dec_b, _ = _decoder(case, 32, 8, 128, avg=32, k_max=256, capacity=5100)
    gen = torch.Generator(device="cuda").manual_seed(3)
    for step in range(6):
        n = 3 if step == 2 else 1
        kt = torch.randn((2, 8, n, 128), device="cuda", generator=gen).to(torch.bfloat16)
        vt = torch.randn((2, 8, n, 128), device="cuda", generator=gen).to(torch.bfloat16)
        qs = (q.float() + 0.3 * torch.randn(q.shape, device="cuda", generator=gen)).to(torch.bfloat16)
        out_a = dec_a.step(qs, k_new=kt, v_new=vt).clone()
        dec_b.append(kt, vt)
        out_b = dec_b.step(qs).clone()
        assert torch.equal(out_a, out_b), f"step {step}"
        assert torch.equal(dec_a.centroid, dec_b.centroid)
        for x, y in zip(dec_a.selected_sets(), dec_b.selected_sets()):
            np.testing.assert_array_equal(x, y)
    S = dec_a.host_seq_lens
    for b in range(2):
        assert torch.equal(dec_a.k[b, :, :S[b]], dec_b.k[b, :, :S[b]])
        assert torch.equal(dec_a.v[b, :, :S[b]], dec_b.v[b, :, :S[b]])
        ref = O.build_centroids(dec_a.k[b, :, :S[b]].float().cpu().numpy(), 16)
        np.testing.assert_array_equal(dec_a.centroid[b, :, :ref.shape[1]].cpu().numpy(), ref)
    assert dec_a.status() == 0 and dec_b.status() == 0


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_minmax_estimator_matches_oracle(dtype):
    """The minmax (Quest) estimator through AdaKVCache / plan_selection:
    exact min / max tables, scores to float rounding, the oracle's selection up
    to documented near-ties, and the attention output."""
    _need_cuda()
    from adakv_b200.attention import AdaKVCache, plan_selection
    from adakv_b200.kernels.block_sparse_decode import block_sparse_decode
    Hq, Hkv, D, bs, S = 16, 4, 128, 16, 3001
    kw = dict(avg_budget=10, k_min=2, k_max=64, n_sink_blocks=1, n_local_blocks=4)
    case = make_decode_case(90, 1, Hq, Hkv, D, S, bs, dtype)
    dt = TORCH[dtype]
    q = torch.from_numpy(case.q[0]).to("cuda", dt)
    K = torch.from_numpy(case.K[0]).to("cuda", dt)
    V = torch.from_numpy(case.V[0]).to("cuda", dt)
    cache = AdaKVCache(bs, estimator="minmax").append_prefill(K, V)
    kmin, kmax = O.build_minmax(case.K[0], bs)
    assert np.array_equal(cache.kmin.cpu().numpy(), kmin)
    assert np.array_equal(cache.kmax.cpu().numpy(), kmax)
    bt, sl = plan_selection(q, cache, estimator="minmax", **kw)
    torch.cuda.synchronize()
    scores = O.minmax_scores(case.q[0], kmin, kmax)
    k, raw = O.allocate_budget(scores, kw["avg_budget"], kw["k_min"], kw["k_max"], 1, 4, 1,
                               return_raw=True)
    mask, _ = O.select_blocks(scores, k, 1, 4, 1)
    sets = [bt[h, : int(sl[h])].cpu().numpy() for h in range(Hq)]
    _, _, _, failures = O.compare_selection(scores, k, raw, mask, sets, 1, 4, 1)
    assert not failures, failures[:4]
    out = block_sparse_decode(q, cache.k, cache.v, bt, sl, bs)
    ref = O.decode_step(case.q[0], case.K[0], case.V[0], block_size=bs, estimator="minmax", **kw)
    err = np.abs(out.float().cpu().numpy() - ref["out"]).max()
    assert err < TOL[dtype], f"max abs err {err:.3e}"
    # append keeps the tables equal to a rebuild
    kt = torch.from_numpy(case.K[0][:, -3:]).to("cuda", dt)
    cache.append_decode(kt, kt)
    K2 = np.concatenate([case.K[0], case.K[0][:, -3:]], axis=1)
    kmin2, kmax2 = O.build_minmax(K2, bs)
    assert np.array_equal(cache.kmin.cpu().numpy(), kmin2)
    assert np.array_equal(cache.kmax.cpu().numpy(), kmax2)


@pytest.mark.parametrize("Hq,Hkv,D,S,avg,kmax", [(12, 2, 64, 320, 8, 256),
                                                 (32, 8, 128, 8192, 64, 512),
                                                 (32, 8, 128, 65536 + 9, 64, 512)])
def test_nucleus_policy_matches_oracle(Hq, Hkv, D, S, avg, kmax):
    """budget_policy='adaptive_nucleus' (adakv/budget.py:38-41): per-head weight
    = number of blocks, in descending probability order, whose cumulative
    softmax mass stays below nucleus_p, plus one.  The GPU budget and selection
    must equal the oracle's on the GPU's own scores."""
    _need_cuda()
    from adakv_b200.batch import BatchedDecoder
    bs = 16
    case = make_decode_case(55, 1, Hq, Hkv, D, S, bs, "bf16")
    dt = torch.bfloat16
    kw = dict(avg_budget=avg, k_min=2, k_max=kmax, budget_policy="adaptive_nucleus", nucleus_p=0.9)
    dec = BatchedDecoder(1, Hq, Hkv, D, bs, S, dt, "cuda", **kw)
    dec.load(torch.from_numpy(case.K).to("cuda", dt), torch.from_numpy(case.V).to("cuda", dt), [S])
    scores = torch.zeros((Hq, dec.nb_cap), dtype=torch.float32, device="cuda")
    dec.plan(torch.from_numpy(case.q).to("cuda", dt), scores_out=scores)
    sets = dec.selected_sets()
    assert dec.status() == 0
    nb = -(-S // bs)
    sc = scores[:, :nb].cpu().numpy()
    k, raw = O.allocate_budget(sc, avg, 2, kmax, 1, 4, 1, policy="adaptive_nucleus",
                               nucleus_p=0.9, return_raw=True)
    mask, _ = O.select_blocks(sc, k, 1, 4, 1)
    n_exact, n_budget, n_score, failures = O.compare_selection(sc, k, raw, mask, sets, 1, 4, 1)
    assert not failures, failures[:4]
    assert n_exact + n_budget + n_score == Hq
