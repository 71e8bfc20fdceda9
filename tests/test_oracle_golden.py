"""Pin the NumPy oracle against golden vectors recorded from the reference.

The fixtures in ``tests/golden/*.npz`` were produced by running the
reference's own ``estimator`` / ``budget`` / ``reference.sparse_attention``
(see ``tests/golden/make_golden.py``).  Here the inputs are regenerated from
the seed and the oracle must reproduce the reference bit-for-bit on the
centroid table, the block scores, the per-head budget and the block mask, and
to 1e-6 on the attention output.  CPU only.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from adakv_b200.synth import make_decode_case
from oracle import adakv_oracle as O
from tests.golden.make_golden import CASES, input_digest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    spec = CASES[name]
    g, a = spec["gen"], dict(spec["alg"])
    gold = _load(name)
    case = make_decode_case(g["seed"], 1, g["Hq"], g["Hkv"], g["D"], g["S"], g["bs"], g["dtype"])
    assert input_digest(case) == str(gold["digest"]), "seeded generator drifted"
    q, K, V = case.q[0], case.K[0], case.V[0]
    nb = int(gold["nb"])

    stride = int(gold.get("centroid_stride", 1))
    if a.pop("estimator", "centroid") == "minmax":
        kmin, kmax = O.build_minmax(K, g["bs"])
        assert str(gold["estimator"]) == "minmax"
        assert np.array_equal(np.stack([kmin, kmax])[..., ::stride, :], gold["centroid"]), \
            "min/max tables differ"
        scores = O.minmax_scores(q, kmin, kmax)
    else:
        cent = O.build_centroids(K, g["bs"])
        assert np.array_equal(cent[:, ::stride], gold["centroid"]), "centroid table differs"
        scores = O.block_scores(q, cent)
    assert scores.dtype == np.float32
    assert np.array_equal(scores, gold["scores"]), "block scores differ"

    temperature = a.pop("temperature", 1.0)
    policy = a.pop("policy")
    k, raw = O.allocate_budget(scores, a["avg_budget"], a["k_min"], a["k_max"],
                               a["n_sink_blocks"], a["n_local_blocks"], a["c_min"],
                               temperature=temperature, policy=policy, return_raw=True)
    assert np.array_equal(k, gold["k"]), f"budget differs: {k} vs {gold['k']}"
    if np.isfinite(gold["raw"]).all():
        assert np.array_equal(raw, gold["raw"])

    mask, counts = O.select_blocks(scores, k, a["n_sink_blocks"], a["n_local_blocks"], a["c_min"])
    gmask = np.unpackbits(gold["mask"], axis=1, count=nb).astype(bool)
    assert np.array_equal(mask, gmask), "block mask differs"
    assert np.array_equal(counts, gold["counts"])

    if "out" in gold:
        out = O.attend_mask(q, K, V, mask, g["bs"])
        np.testing.assert_allclose(out, gold["out"], rtol=0, atol=1e-6)


def test_decode_step_bundles_the_pieces():
    spec = CASES["cfg0_fp32"]
    g, a = spec["gen"], spec["alg"]
    gold = _load("cfg0_fp32")
    case = make_decode_case(g["seed"], 1, g["Hq"], g["Hkv"], g["D"], g["S"], g["bs"], g["dtype"])
    r = O.decode_step(case.q[0], case.K[0], case.V[0], block_size=g["bs"],
                      avg_budget=a["avg_budget"], k_min=a["k_min"], k_max=a["k_max"],
                      n_sink_blocks=a["n_sink_blocks"], n_local_blocks=a["n_local_blocks"],
                      c_min=a["c_min"], policy=a["policy"])
    np.testing.assert_allclose(r["out"], gold["out"], rtol=0, atol=1e-6)
    assert np.array_equal(r["counts"], gold["counts"])


def test_attend_table_matches_mask_form():
    rng = np.random.default_rng(0)
    Hq, Hkv, S, D, bs = 8, 2, 200, 32, 16
    q = rng.standard_normal((Hq, D)).astype(np.float32)
    K = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    V = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    nb = (S + bs - 1) // bs
    table = np.stack([rng.permutation(nb)[:5] for _ in range(Hq)]).astype(np.int32)
    table[0, 0] = nb - 1                      # include the partial tail block
    lens = np.array([5, 4, 3, 5, 1, 2, 5, 5], dtype=np.int32)
    out = O.attend_table(q, K, V, table, lens, bs)
    mask = np.zeros((Hq, nb), dtype=bool)
    for h in range(Hq):
        mask[h, table[h, :lens[h]]] = True
    np.testing.assert_array_equal(out, O.attend_mask(q, K, V, mask, bs))
    # full mask == dense attention
    full = O.attend_mask(q, K, V, np.ones((Hq, nb), dtype=bool), bs)
    np.testing.assert_allclose(full, O.dense_attention(q, K, V), atol=1e-12)


def test_compare_selection_classifies_near_ties():
    scores = np.array([[5.0, 1.0, 3.0, 3.0 + 1e-9, 0.5, 2.0]], dtype=np.float64)
    k = np.array([4])
    mask, _ = O.select_blocks(scores, k, 1, 1, 1)      # forced 0 and 5; content: 2 of {1,2,3,4}
    # oracle picks 3 (higher) and 2; a GPU picking 2 and 3 is exact
    assert O.compare_selection(scores, k, np.array([np.nan]), mask, [[0, 2, 3, 5]], 1, 1, 1)[0] == 1
    mask_tie = mask.copy()
    mask_tie[0, 2] = False
    mask_tie[0, 1] = True   # pretend oracle chose 1 instead of 2: a real failure (gap 2.0)
    res = O.compare_selection(scores, k, np.array([np.nan]), mask_tie, [[0, 2, 3, 5]], 1, 1, 1)
    assert len(res[3]) == 1
    # a swap between 3.0 and 3.0+1e-9 is a score near-tie
    mask2 = np.zeros_like(mask)
    mask2[0, [0, 5, 3, 1]] = True
    s2 = scores.copy()
    s2[0, 1] = 3.0 + 2e-9
    m3, _ = O.select_blocks(s2, k, 1, 1, 1)
    res = O.compare_selection(s2, k, np.array([np.nan]), m3, [[0, 5, 2, 1]], 1, 1, 1)
    assert res[2] == 1 and not res[3]
    # budget near-tie: oracle raw 4.50001 -> 5 ... gpu took 4
    s3 = np.array([[5.0, 1.0, 3.0, 2.5, 0.5, 2.0]])
    m5, _ = O.select_blocks(s3, np.array([5]), 1, 1, 1)
    res = O.compare_selection(s3, np.array([5]), np.array([4.50001]), m5, [[0, 5, 2, 3]], 1, 1, 1)
    assert res[1] == 1 and not res[3]


@pytest.mark.parametrize("name", sorted(__import__("tests.golden.make_golden",
                                                   fromlist=["BASELINE_CASES"]).BASELINE_CASES))
def test_baseline_oracle_matches_reference_golden(name):
    """H2O / SnapKV: importance to 1e-6 relative, retained masks (every budget),
    the frozen decode-time mask and the frozen attention output, against the
    reference's own outputs."""
    import hashlib
    from adakv_b200.synth import make_prefill_case
    from tests.golden.make_golden import BASELINE_CASES
    c = BASELINE_CASES[name]
    gold = _load(name)
    Q, K, V, q = make_prefill_case(c["seed"], c["Hq"], c["Hkv"], c["D"], c["S"])
    h = hashlib.sha256()
    for a in (Q, K, V, q):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(gold["digest"]), "seeded generator drifted"
    g = c["Hq"] // c["Hkv"]
    Kq, Vq = np.repeat(K, g, axis=0), np.repeat(V, g, axis=0)
    h2o = O.h2o_key_importance(Q, Kq)
    snap = O.snapkv_key_importance(Q, Kq, c["window"], c["pool"])
    for got, ref in ((h2o, gold["h2o"]), (snap, gold["snapkv"])):
        assert np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()
    nb = (c["S"] + c["bs"] - 1) // c["bs"]
    for bud in c["budgets"]:
        for kind, imp in (("h2o", h2o), ("snapkv", snap)):
            m = O.retain_blocks(imp, c["bs"], c["S"], bud, c["sink"], c["local"], c["c_min"])
            assert np.array_equal(m, gold[f"mask_{kind}_{bud}"]), f"{kind} budget {bud}"
            dm = O.frozen_decode_mask(m, nb + 2, c["sink"], c["local"])
            assert np.array_equal(dm, gold[f"decode_mask_{kind}_{bud}"])
            out = O.attend_mask(q, K, V, m, c["bs"])
            assert np.abs(out - gold[f"out_{kind}_{bud}"]).max() < 1e-6
