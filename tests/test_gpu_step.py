"""The one-kernel decode step (``adakv_decode_step`` on the persistent kernel,
``ADAKV_KNOB_STEP_PATH`` = 2) against the NumPy oracle, on identical seeded
inputs (needs a B200); the headline-size cases also run the default
three-kernel chain.

Bars: block scores within 2e-6 relative of the float64 oracle; selected block
sets identical per head except documented near-ties (score gap < 1e-6
relative, or an unrounded budget within 1e-5 of a .5 boundary); attention
outputs within 2e-2 abs (bf16 / fp16 inputs).  The same cases also run the
three-kernel chain (``ADAKV_KNOB_STEP_PATH`` = 1) and compare the two paths.
Every call goes through the C ABI.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from adakv_b200 import _lib  # noqa: E402
from adakv_b200.batch import BatchedDecoder  # noqa: E402
from adakv_b200.synth import make_decode_case, ragged_seq_lens  # noqa: E402
from oracle import adakv_oracle as O  # noqa: E402

TORCH = {"bf16": torch.bfloat16, "fp16": torch.float16}
BUDGET_TOL = 1e-5


@pytest.fixture(autouse=True)
def _need_cuda_and_reset_knobs():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    # the one-kernel step unless a test picks the chain (the library default)
    _lib.debug_knob(_lib.KNOB_STEP_PATH, 2)
    yield
    for knob in (_lib.KNOB_WAIT_NS, _lib.KNOB_FLAGS, _lib.KNOB_STEP_PATH, _lib.KNOB_STEP_CLUSTER):
        _lib.debug_knob(knob, 0)


def _kw(avg, k_max, **extra):
    kw = dict(avg_budget=avg, k_min=2, k_max=k_max, n_sink_blocks=1, n_local_blocks=4, c_min=1,
              temperature=1.0, budget_policy="adaptive")
    kw.update(extra)
    return kw


def _decoder(case, Hq, Hkv, kw, capacity=None):
    B, D = case.q.shape[0], case.q.shape[2]
    cap = capacity or int(case.seq_lens.max())
    dt = TORCH[case.dtype]
    dec = BatchedDecoder(B, Hq, Hkv, D, case.block_size, cap, dt, "cuda",
                         avg_budget=kw["avg_budget"], k_min=kw["k_min"], k_max=kw["k_max"],
                         n_sink_blocks=kw["n_sink_blocks"], n_local_blocks=kw["n_local_blocks"],
                         c_min=kw["c_min"], temperature=kw["temperature"],
                         budget_policy=kw["budget_policy"])
    S = int(case.seq_lens.max())
    dec.load(torch.from_numpy(case.K[:, :, :S]).to("cuda", dt),
             torch.from_numpy(case.V[:, :, :S]).to("cuda", dt), case.seq_lens)
    return dec, torch.from_numpy(case.q).to("cuda", dt)


def _oracle(q, K, V, bs, kw, centroids=None):
    return O.decode_step(q, K, V, block_size=bs, avg_budget=kw["avg_budget"], k_min=kw["k_min"],
                         k_max=kw["k_max"], n_sink_blocks=kw["n_sink_blocks"],
                         n_local_blocks=kw["n_local_blocks"], c_min=kw["c_min"],
                         temperature=kw["temperature"], policy=kw["budget_policy"],
                         centroids=centroids)


def _check_seq(res, sets, scores_gpu, out_gpu, q, K, V, bs, kw, label, tol=2e-2):
    """Scores, selection (up to classified near-ties) and output of one sequence."""
    nb = res["scores"].shape[1]
    got = scores_gpu[:, :nb].astype(np.float64)
    err = np.abs(got - res["scores"])
    scale = np.abs(res["scores"]).max(axis=1, keepdims=True) + 1e-30
    assert (err / scale).max() < 2e-6, f"{label}: score rel err {(err / scale).max():.3e}"
    n_exact, n_budget, n_score, fails = O.compare_selection(
        res["scores"], res["k"], res["raw"], res["mask"], sets, kw["n_sink_blocks"],
        kw["n_local_blocks"], kw["c_min"], budget_tol=BUDGET_TOL)
    assert not fails, f"{label}: selection mismatch {fails[:3]}"
    Hq = len(sets)
    assert n_budget + n_score <= max(1, Hq // 16), f"{label}: too many near-ties"
    for s in sets:
        assert np.all(np.diff(s) > 0), "rows must be ascending and duplicate-free"
    mask = np.zeros_like(res["mask"])
    for h in range(Hq):
        mask[h, sets[h]] = True
    ref = O.attend_mask(q, K, V, mask, bs)
    e = np.abs(out_gpu - ref).max()
    assert e < tol, f"{label}: max abs err {e:.3e} vs attention over the GPU selection"
    exact = np.all(mask == res["mask"], axis=1)
    if exact.any():
        e2 = np.abs(out_gpu[exact] - res["out"][exact]).max()
        assert e2 < tol, f"{label}: max abs err {e2:.3e} vs the oracle step"
    return n_exact


# (seed, Hq, Hkv, S, dtype, avg, k_max, extra)
STEP_CASES = [
    (0, 32, 8, 4096, "bf16", 16, 128, {}),
    (12, 32, 8, 32768, "bf16", 64, 512, {}),
    (18, 32, 8, 65536, "bf16", 64, 512, {}),
    (17, 32, 8, 131072, "bf16", 64, 512, {}),               # the headline configuration
    (19, 64, 8, 16384, "bf16", 64, 512, {}),                # GQA 8 (70B attention shape)
    (20, 16, 4, 8000, "fp16", 24, 128, {}),
    (21, 32, 8, 4096, "bf16", 24, 64, {"budget_policy": "fixed"}),
    (22, 16, 4, 2048, "bf16", 16, 128, {"temperature": 0.5}),
    (23, 8, 2, 100, "bf16", 5, 64, {}),                     # 7 blocks, partial tail
    (24, 8, 2, 20, "bf16", 8, 64, {}),                      # 2 blocks: all selected
    (25, 32, 8, 250007, "bf16", 64, 512, {}),               # long row, odd length
]


@pytest.mark.parametrize("path", [1, 2], ids=["chain", "one_kernel"])
@pytest.mark.parametrize("seed,Hq,Hkv,S,dtype,avg,kmax,extra", STEP_CASES)
def test_step_matches_oracle(seed, Hq, Hkv, S, dtype, avg, kmax, extra, path):
    bs = 16
    kw = _kw(avg, kmax, **extra)
    _lib.debug_knob(_lib.KNOB_STEP_PATH, path)
    case = make_decode_case(seed, 1, Hq, Hkv, 128, S, bs, dtype)
    dec, q = _decoder(case, Hq, Hkv, kw)
    out = dec.step(q).float().cpu().numpy()[0]
    assert dec.last_path() == path
    sc = dec.scores().cpu().numpy()[0]
    res = _oracle(case.q[0], case.K[0], case.V[0], bs, kw)
    _check_seq(res, dec.selected_sets(), sc, out, case.q[0], case.K[0], case.V[0], bs, kw, f"S={S}")
    assert dec.status() == 0


@pytest.mark.parametrize("cluster", [1, 2, 4])
@pytest.mark.parametrize("seed,S", [(26, 131072), (27, 40000), (28, 250007)])
def test_step_cluster_sizes_match_oracle(seed, S, cluster):
    """The selection phase on 1, 2 or 4 CTAs per query head (the cluster merges
    histograms and candidates through distributed shared memory)."""
    bs, Hq, Hkv = 16, 32, 8
    kw = _kw(64, 512)
    _lib.debug_knob(_lib.KNOB_STEP_CLUSTER, cluster)
    case = make_decode_case(seed, 1, Hq, Hkv, 128, S, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, kw)
    out = dec.step(q).float().cpu().numpy()[0]
    assert dec.last_path() == 2
    sc = dec.scores().cpu().numpy()[0]
    res = _oracle(case.q[0], case.K[0], case.V[0], bs, kw)
    _check_seq(res, dec.selected_sets(), sc, out, case.q[0], case.K[0], case.V[0], bs, kw,
               f"S={S} cluster<={cluster}")


def test_step_batched_ragged():
    lens = ragged_seq_lens(5, 3, 3000, 40000).tolist()
    Hq, Hkv, bs = 32, 8, 16
    kw = _kw(48, 256)
    case = make_decode_case(26, len(lens), Hq, Hkv, 128, lens, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, kw)
    out = dec.step(q).float().cpu().numpy()
    sc = dec.scores().cpu().numpy()
    sets = dec.selected_sets()
    for b, S in enumerate(lens):
        res = _oracle(case.q[b], case.K[b, :, :S], case.V[b, :, :S], bs, kw)
        _check_seq(res, sets[b * Hq:(b + 1) * Hq], sc[b], out[b], case.q[b], case.K[b, :, :S],
                   case.V[b, :, :S], bs, kw, f"seq {b}")
    assert dec.status() == 0


@pytest.mark.parametrize("n_new", [1, 3])
def test_step_with_append_matches_oracle(n_new):
    """Tokens appended inside the step (cache write + trailing-centroid refresh in
    the same kernel) across block boundaries; the oracle rebuilds from scratch."""
    Hq, Hkv, bs, S0 = 32, 8, 16, 5000
    kw = _kw(32, 256)
    case = make_decode_case(27, 1, Hq, Hkv, 128, S0, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, kw, capacity=S0 + 64)
    rng = np.random.default_rng(28)
    K, V = case.K[0].copy(), case.V[0].copy()
    for step in range(12):
        kn = torch.from_numpy(rng.standard_normal((1, Hkv, n_new, 128), dtype=np.float32)).to(
            "cuda", torch.bfloat16)
        vn = torch.from_numpy(rng.standard_normal((1, Hkv, n_new, 128), dtype=np.float32)).to(
            "cuda", torch.bfloat16)
        out = dec.step(q, k_new=kn, v_new=vn).float().cpu().numpy()[0]
        K = np.concatenate([K, kn[0].float().cpu().numpy()], axis=1)
        V = np.concatenate([V, vn[0].float().cpu().numpy()], axis=1)
    S = dec.host_seq_lens[0]
    assert S == K.shape[1]
    np.testing.assert_array_equal(dec.k[0, :, :S].float().cpu().numpy(), K)
    np.testing.assert_array_equal(dec.v[0, :, :S].float().cpu().numpy(), V)
    cent = O.build_centroids(K, bs)
    np.testing.assert_array_equal(dec.centroid[0, :, : cent.shape[1]].cpu().numpy(), cent)
    res = _oracle(case.q[0], K, V, bs, kw, centroids=cent)
    sc = dec.scores().cpu().numpy()[0]
    _check_seq(res, dec.selected_sets(), sc, out, case.q[0], K, V, bs, kw, f"append {n_new}")
    assert dec.status() == 0


def test_step_radix_path_on_flat_rows():
    """Rows whose content scores are all equal have no bucket range: the exact
    radix select must take the lowest block indices."""
    Hq, Hkv, bs, S = 8, 2, 16, 4096
    kw = _kw(12, 64)
    case = make_decode_case(29, 1, Hq, Hkv, 128, S, bs, "bf16")
    case.K[:] = 0.0
    dec, q = _decoder(case, Hq, Hkv, kw)
    out = dec.step(q).float().cpu().numpy()[0]
    sc = dec.scores().cpu().numpy()[0]
    res = _oracle(case.q[0], case.K[0], case.V[0], bs, kw)
    _check_seq(res, dec.selected_sets(), sc, out, case.q[0], case.K[0], case.V[0], bs, kw, "flat")


@pytest.mark.parametrize("S", [32768, 131072])
def test_step_equals_three_kernel_chain(S):
    Hq, Hkv, bs = 32, 8, 16
    kw = _kw(64, 512)
    case = make_decode_case(30, 1, Hq, Hkv, 128, S, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, kw)
    out1 = dec.step(q).clone()
    sets1 = dec.selected_sets()
    sc1 = dec.scores().clone()
    _lib.debug_knob(_lib.KNOB_STEP_PATH, 1)
    out3 = dec.step(q).clone()
    sets3 = dec.selected_sets()
    sc3 = dec.scores().clone()
    assert torch.equal(sc1, sc3) or (sc1 - sc3).abs().max().item() <= 2e-6 * sc3.abs().max().item()
    differ = [h for h in range(Hq) if not np.array_equal(sets1[h], sets3[h])]
    assert len(differ) <= 1, f"heads whose selection differs between the paths: {differ}"
    same = [h for h in range(Hq) if h not in differ]
    assert (out1[0, same].float() - out3[0, same].float()).abs().max().item() < 2e-2
    assert dec.status() == 0


def test_step_is_deterministic_and_graph_capturable():
    Hq, Hkv, bs, S = 32, 8, 16, 65536
    kw = _kw(64, 512)
    case = make_decode_case(31, 1, Hq, Hkv, 128, S, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, kw)
    a = dec.step(q).clone()
    sets_a = dec.selected_sets()
    for _ in range(5):
        b = dec.step(q)
    assert torch.equal(a, b)
    g = dec.graphed(n_new=1, advance=False)
    g.q.copy_(q)
    for _ in range(3):
        g()
    torch.cuda.synchronize()
    assert dec.status() == 0
    assert len(dec.selected_sets()) == len(sets_a)


@pytest.mark.parametrize("path", [2, 1])
def test_bounded_wait_runs_out_and_is_reported(path):
    """Query head 0 never publishes its entropy (test knob): the other heads'
    bounded exchange waits run out after 1 ms, the status word records
    ADAKV_ST_WAIT_TIMEOUT, the host-mapped sink makes the next call raise, and
    the device stays usable (a normal step afterwards is clean)."""
    import time
    Hq, Hkv, bs, S = 32, 8, 16, 16384
    kw = _kw(64, 512)
    case = make_decode_case(32, 1, Hq, Hkv, 128, S, bs, "bf16")
    dec, q = _decoder(case, Hq, Hkv, kw)
    dec.step(q)
    assert dec.status() == 0
    _lib.debug_knob(_lib.KNOB_STEP_PATH, path)
    _lib.debug_knob(_lib.KNOB_WAIT_NS, 1_000_000)
    _lib.debug_knob(_lib.KNOB_FLAGS, 1)
    t0 = time.perf_counter()
    dec.step(q)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 0.5, f"the failed step took {elapsed:.3f} s"
    assert dec.sink.bits() & _lib.ST_WAIT_TIMEOUT
    with pytest.raises(RuntimeError, match="timed out"):
        dec.step(q)
    assert dec.status() & _lib.ST_WAIT_TIMEOUT
    _lib.debug_knob(_lib.KNOB_FLAGS, 0)
    _lib.debug_knob(_lib.KNOB_WAIT_NS, 0)
    out = dec.step(q).float().cpu().numpy()[0]
    assert dec.status() == 0
    res = _oracle(case.q[0], case.K[0], case.V[0], bs, kw)
    _check_seq(res, dec.selected_sets(), dec.scores().cpu().numpy()[0], out, case.q[0], case.K[0],
               case.V[0], bs, kw, "after timeout")
