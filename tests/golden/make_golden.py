"""Generate golden vectors by running the reference implementation itself.

Run in a checkout that has the reference project available::

    python tests/golden/make_golden.py --reference <path to the adakv project>

The reference package is imported under the private name ``adakv_ref`` (it is
also called ``adakv``) and its own functions are called on seeded inputs made
by :func:`adakv_b200.synth.make_decode_case`:

* ``estimator.build_block_summaries`` / ``block_scores`` on GQA-expanded keys
  (``adakv/estimator.py:27-74``, ``adakv/reference.py:29-33``);
* ``budget.allocate_budget`` with the floor ``reference.sparse_attention``
  passes (``adakv/reference.py:71-73``), plus its unrounded ``lo + extra``;
* ``reference.sparse_attention(..., return_mask=True)`` for the block mask,
  counts and the attention output (``adakv/reference.py:44-84``);
* the H2O / SnapKV baselines: ``baselines.h2o_key_importance``,
  ``snapkv_key_importance``, ``retain_blocks``, ``frozen_sparse_attention``
  and ``baselines_rt.frozen_decode_block_table`` (``baselines_*.npz``).

Each case is written to ``tests/golden/<name>.npz`` together with a SHA-256
of the generated inputs, so the tests can detect generator drift.  The
fixtures are small (outputs only); the inputs are regenerated from the seed.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from adakv_b200.synth import make_decode_case  # noqa: E402

# name -> generator + algorithm parameters.  Shapes cover the headline
# configuration's CPU case (32/8 heads, D 128, S 4096, avg 8), partial trailing
# blocks, odd GQA groups (6, as the reference's factorial test), block size 32
# with D 64 (the reference kernel test's second shape), tiny block counts,
# a full budget, bf16-rounded inputs, a non-unit temperature and the fixed /
# nucleus policies.
CASES = {
    "cfg0_fp32": dict(gen=dict(seed=0, Hq=32, Hkv=8, D=128, S=4096, bs=16, dtype="fp32"),
                      alg=dict(avg_budget=8, k_min=2, k_max=64, n_sink_blocks=1,
                               n_local_blocks=4, c_min=1, policy="adaptive")),
    "partial_tail": dict(gen=dict(seed=1, Hq=8, Hkv=2, D=128, S=4001, bs=16, dtype="fp32"),
                         alg=dict(avg_budget=12, k_min=2, k_max=64, n_sink_blocks=1,
                                  n_local_blocks=4, c_min=1, policy="adaptive")),
    "partial_tail9": dict(gen=dict(seed=2, Hq=8, Hkv=4, D=64, S=1033, bs=16, dtype="fp32"),
                          alg=dict(avg_budget=10, k_min=2, k_max=64, n_sink_blocks=2,
                                   n_local_blocks=3, c_min=1, policy="adaptive")),
    "gqa6_adaptive": dict(gen=dict(seed=3, Hq=12, Hkv=2, D=64, S=320, bs=16, dtype="fp32"),
                          alg=dict(avg_budget=8, k_min=2, k_max=256, n_sink_blocks=1,
                                   n_local_blocks=2, c_min=1, policy="adaptive")),
    "gqa6_fixed": dict(gen=dict(seed=3, Hq=12, Hkv=2, D=64, S=320, bs=16, dtype="fp32"),
                       alg=dict(avg_budget=8, k_min=2, k_max=256, n_sink_blocks=1,
                                n_local_blocks=2, c_min=1, policy="fixed")),
    "gqa6_nucleus": dict(gen=dict(seed=3, Hq=12, Hkv=2, D=64, S=320, bs=16, dtype="fp32"),
                         alg=dict(avg_budget=8, k_min=2, k_max=256, n_sink_blocks=1,
                                  n_local_blocks=2, c_min=1, policy="adaptive_nucleus")),
    "bs32_d64": dict(gen=dict(seed=4, Hq=4, Hkv=4, D=64, S=8192, bs=32, dtype="fp32"),
                     alg=dict(avg_budget=16, k_min=2, k_max=64, n_sink_blocks=1,
                              n_local_blocks=4, c_min=1, policy="adaptive")),
    "full_budget": dict(gen=dict(seed=5, Hq=8, Hkv=2, D=64, S=512, bs=16, dtype="fp32"),
                        alg=dict(avg_budget=32, k_min=32, k_max=32, n_sink_blocks=1,
                                 n_local_blocks=4, c_min=1, policy="adaptive")),
    "tiny_nb1": dict(gen=dict(seed=6, Hq=8, Hkv=2, D=64, S=10, bs=16, dtype="fp32"),
                     alg=dict(avg_budget=8, k_min=2, k_max=64, n_sink_blocks=1,
                              n_local_blocks=4, c_min=1, policy="adaptive")),
    "tiny_nb2": dict(gen=dict(seed=7, Hq=8, Hkv=2, D=64, S=20, bs=16, dtype="fp32"),
                     alg=dict(avg_budget=8, k_min=2, k_max=64, n_sink_blocks=1,
                              n_local_blocks=4, c_min=1, policy="adaptive")),
    "tiny_nb7": dict(gen=dict(seed=8, Hq=8, Hkv=2, D=64, S=100, bs=16, dtype="fp32"),
                     alg=dict(avg_budget=5, k_min=2, k_max=64, n_sink_blocks=1,
                              n_local_blocks=4, c_min=1, policy="adaptive")),
    "bf16_8k": dict(gen=dict(seed=9, Hq=32, Hkv=8, D=128, S=8192, bs=16, dtype="bf16"),
                    alg=dict(avg_budget=64, k_min=2, k_max=512, n_sink_blocks=1,
                             n_local_blocks=4, c_min=1, policy="adaptive")),
    "temperature": dict(gen=dict(seed=10, Hq=16, Hkv=4, D=128, S=2048, bs=16, dtype="fp32"),
                        alg=dict(avg_budget=16, k_min=2, k_max=128, n_sink_blocks=1,
                                 n_local_blocks=4, c_min=1, policy="adaptive",
                                 temperature=0.5)),
    "minmax_fp32": dict(gen=dict(seed=12, Hq=8, Hkv=2, D=128, S=4001, bs=16, dtype="fp32"),
                        alg=dict(avg_budget=12, k_min=2, k_max=64, n_sink_blocks=1,
                                 n_local_blocks=4, c_min=1, policy="adaptive",
                                 estimator="minmax")),
    "minmax_bf16": dict(gen=dict(seed=13, Hq=32, Hkv=8, D=128, S=8192, bs=16, dtype="bf16"),
                        alg=dict(avg_budget=64, k_min=2, k_max=512, n_sink_blocks=1,
                                 n_local_blocks=4, c_min=1, policy="adaptive",
                                 estimator="minmax")),
    "kmax_cap": dict(gen=dict(seed=11, Hq=32, Hkv=8, D=128, S=4096, bs=16, dtype="fp32"),
                     alg=dict(avg_budget=32, k_min=2, k_max=16, n_sink_blocks=1,
                              n_local_blocks=4, c_min=1, policy="adaptive")),
}


def input_digest(case) -> str:
    h = hashlib.sha256()
    for a in (case.q, case.K, case.V, case.seq_lens):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_reference(path: str):
    pkg_dir = os.path.join(path, "adakv")
    spec = importlib.util.spec_from_file_location(
        "adakv_ref", os.path.join(pkg_dir, "__init__.py"),
        submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["adakv_ref"] = mod
    spec.loader.exec_module(mod)
    import importlib as il
    return (il.import_module("adakv_ref.reference"), il.import_module("adakv_ref.estimator"),
            il.import_module("adakv_ref.budget"))


def run_case(name, spec, ref, est, bud):
    g, a = spec["gen"], dict(spec["alg"])
    case = make_decode_case(g["seed"], 1, g["Hq"], g["Hkv"], g["D"], g["S"], g["bs"], g["dtype"])
    q, K, V = case.q[0], case.K[0], case.V[0]
    Kq, Vq = ref.expand_gqa(K, g["Hq"]), ref.expand_gqa(V, g["Hq"])
    temperature = a.pop("temperature", 1.0)
    policy = a.pop("policy")
    estimator = a.pop("estimator", "centroid")
    nb = (g["S"] + g["bs"] - 1) // g["bs"]
    summ = est.build_block_summaries(Kq, g["bs"], estimator)
    scores = est.block_scores(q, summ)
    floor = min(a["n_sink_blocks"], nb) + min(a["n_local_blocks"], nb) + a["c_min"]
    k = bud.allocate_budget(scores, a["avg_budget"], min(a["k_min"], nb), min(a["k_max"], nb),
                            temperature=temperature, policy=policy, floor=floor)
    raw = np.full((g["Hq"],), np.nan)
    if nb > 1 and policy != "fixed":
        lo = min(max(int(floor), int(min(a["k_min"], nb)), 1), nb)
        hi = min(int(min(a["k_max"], nb)), nb)
        target = float(np.clip(a["avg_budget"], lo, hi))
        w = bud._weights(scores, policy, temperature, 0.9)
        raw = lo + max(target - lo, 0.0) * g["Hq"] * w / max(float(w.sum()), 1e-9)
    out = counts = mask = None
    if temperature == 1.0:
        out, counts, mask = ref.sparse_attention(
            q, Kq, Vq, block_size=g["bs"], avg_budget=a["avg_budget"], k_min=a["k_min"],
            k_max=a["k_max"], n_sink_blocks=a["n_sink_blocks"], n_local_blocks=a["n_local_blocks"],
            c_min=a["c_min"], budget_policy=policy, estimator=estimator, return_mask=True)
    else:  # sparse_attention has no temperature argument; select from the budget directly
        from adakv_ref.selector import select_blocks
        mask, counts = select_blocks(scores, k, a["n_sink_blocks"], a["n_local_blocks"], a["c_min"])
    if estimator == "minmax":  # the per-KV-head tables stacked as [2, Hkv, nb, D]
        table = np.stack([summ["kmin"][:: g["Hq"] // g["Hkv"]], summ["kmax"][:: g["Hq"] // g["Hkv"]]])
    else:
        table = summ["centroid"][:: g["Hq"] // g["Hkv"]]
    rec = dict(digest=np.array(input_digest(case)), scores=scores.astype(np.float32),
               centroid=table.astype(np.float32), estimator=np.array(estimator),
               k=np.asarray(k, dtype=np.int64), raw=np.asarray(raw, dtype=np.float64),
               counts=np.asarray(counts, dtype=np.int64), mask=np.packbits(mask, axis=1),
               nb=np.array(nb))
    if out is not None:
        rec["out"] = np.asarray(out, dtype=np.float64)
    # the centroid table is large for the big cases; keep only a strided sample of rows
    if rec["centroid"].size > 20_000:
        stride = int(np.ceil(rec["centroid"].size / 20_000)) | 1
        rec["centroid"] = rec["centroid"][..., ::stride, :].copy() if estimator == "minmax" \
            else rec["centroid"][:, ::stride].copy()
        rec["centroid_stride"] = np.array(stride)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
    return counts


# H2O / SnapKV eviction baselines (adakv/baselines.py, adakv/baselines_rt.py):
# inputs from adakv_b200.synth.make_prefill_case, keys expanded to the query
# heads for the reference's per-query-head functions.
BASELINE_CASES = {
    "baselines_h6": dict(seed=20, Hq=6, Hkv=6, D=64, S=384, bs=16, sink=1, local=2, c_min=1,
                         budgets=(6, 8, 12), window=32, pool=7),
    "baselines_gqa4": dict(seed=21, Hq=8, Hkv=2, D=128, S=517, bs=16, sink=1, local=4, c_min=1,
                           budgets=(8, 16), window=32, pool=7),
}


def run_baseline_case(name, spec, path):
    from adakv_b200.synth import make_prefill_case
    import importlib as il
    bl = il.import_module("adakv_ref.baselines")
    rt = il.import_module("adakv_ref.baselines_rt")
    import torch
    c = spec
    Q, K, V, q = make_prefill_case(c["seed"], c["Hq"], c["Hkv"], c["D"], c["S"])
    g = c["Hq"] // c["Hkv"]
    Kq, Vq = np.repeat(K, g, axis=0), np.repeat(V, g, axis=0)
    h2o = bl.h2o_key_importance(Q, Kq)
    snap = bl.snapkv_key_importance(Q, Kq, obs_window=c["window"], pool_kernel=c["pool"])
    rec = dict(h2o=h2o, snapkv=snap)
    digest = hashlib.sha256()
    for a in (Q, K, V, q):
        digest.update(np.ascontiguousarray(a).tobytes())
    rec["digest"] = np.array(digest.hexdigest())
    nb = (c["S"] + c["bs"] - 1) // c["bs"]
    for bud in c["budgets"]:
        for kind, imp in (("h2o", h2o), ("snapkv", snap)):
            m = bl.retain_blocks(imp, c["bs"], c["S"], bud, c["sink"], c["local"], c["c_min"])
            rec[f"mask_{kind}_{bud}"] = m
            # the decode-time table two blocks later, and one frozen decode step
            bt, sl = rt.frozen_decode_block_table(torch.from_numpy(m), nb + 2, c["sink"], c["local"])
            dm = np.zeros((c["Hq"], nb + 2), dtype=bool)
            for h in range(c["Hq"]):
                dm[h, bt[h, :int(sl[h])].numpy()] = True
            rec[f"decode_mask_{kind}_{bud}"] = dm
            out, _ = bl.frozen_sparse_attention(q, Kq, Vq, m, c["bs"])
            rec[f"out_{kind}_{bud}"] = np.asarray(out, dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference project")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    ref, est, bud = load_reference(args.reference)
    for name, spec in CASES.items():
        if args.only and name not in args.only:
            continue
        counts = run_case(name, spec, ref, est, bud)
        print(f"{name}: counts mean {np.mean(counts):.2f} min {np.min(counts)} max {np.max(counts)}")
    for name, spec in BASELINE_CASES.items():
        if args.only and name not in args.only:
            continue
        run_baseline_case(name, spec, args.reference)
        print(f"{name}: written")


if __name__ == "__main__":
    main()
