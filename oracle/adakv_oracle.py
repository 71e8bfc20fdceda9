"""CPU oracle for the AdaKV decode hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in NumPy, the reference algorithm of liukefan821/adakv
for one decode step (centroid summaries -> block scores -> entropy budget ->
sink/local-forced top-k selection -> attention over the selected blocks).
It is the checker the CUDA path is compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it; the product path (``adakv_b200``) never
does, and has no CPU fallback.

Parity status: PINNED.  ``tests/golden/make_golden.py`` imported the Python
reference package and recorded its outputs on seeded inputs into
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this module
against those fixtures bit-for-bit (block masks, per-head budgets, scores)
and to 1e-6 on attention outputs.

Every function cites the reference file:line it follows (paths are relative
to the reference project root).  Differences from the reference, all
deliberate and checked by the golden tests:

* GQA is folded (KV-head arrays are never expanded to the query-head count
  for K/V, only the small centroid table is repeated for the score einsum so
  the score arithmetic is the reference's own), which lets the oracle run at
  128K-1M tokens;
* ties in the top-k order are broken by lowest block index (stable sort);
  the reference's ``np.argsort`` default is an unstable quicksort, so exact
  ties are unspecified there and are treated as near-ties by the tests;
* attention is computed over the selected tokens only (identical math to the
  reference's full-row masked softmax, ``reference.py:76-80``, which assigns
  exactly zero weight to unselected tokens).
"""
from __future__ import annotations

import math

import numpy as np

POLICY_FIXED = "fixed"
POLICY_ADAPTIVE = "adaptive"
POLICY_NUCLEUS = "adaptive_nucleus"


# --------------------------------------------------------------------------
# (a) per-block key centroids
# --------------------------------------------------------------------------
def build_centroids(K: np.ndarray, block_size: int) -> np.ndarray:
    """Mean key per block over real tokens only.

    Follows ``adakv/estimator.py:40-48``: ``c[:, b] = keys[:, s:e].mean(axis=1)``
    with ``e = min((b+1)*bs, S)`` so a partial trailing block is averaged over
    its real token count.  NumPy reduces a non-contiguous axis sequentially
    in float32 and divides in float64 before rounding back to float32 (which
    equals a correctly rounded float32 division); this restatement performs
    the same sequential float32 accumulation vectorised over blocks, so the
    result is bit-identical (pinned by the golden tests).

    K: ``[H, S, D]`` float32 -> ``[H, nb, D]`` float32.
    """
    K = np.asarray(K, dtype=np.float32)
    H, S, D = K.shape
    nb = (S + block_size - 1) // block_size
    out = np.empty((H, nb, D), dtype=np.float32)
    n_full = S // block_size
    if n_full:
        blk = K[:, : n_full * block_size].reshape(H, n_full, block_size, D)
        acc = blk[:, :, 0, :].copy()
        for t in range(1, block_size):
            acc += blk[:, :, t, :]
        out[:, :n_full] = acc / np.float32(block_size)
    if nb > n_full:  # partial trailing block
        tail = K[:, n_full * block_size:]
        acc = tail[:, 0, :].copy()
        for t in range(1, tail.shape[1]):
            acc += tail[:, t, :]
        out[:, n_full] = acc / np.float32(tail.shape[1])
    return out


# --------------------------------------------------------------------------
# (b) centroid block estimator
# --------------------------------------------------------------------------
def block_scores(q: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """Unscaled ``q . centroid`` per (query head, block).

    Follows ``adakv/estimator.py:73-74`` (``einsum("hd,hbd->hb")``) with the
    caller-side GQA expansion of ``adakv/reference.py:61-62`` applied to the
    centroid table only (``np.repeat`` over the group, as ``expand_gqa``,
    ``reference.py:29-33``), so the float32 einsum is the reference's own.

    q: ``[Hq, D]`` float32, centroids: ``[Hkv, nb, D]`` float32 -> ``[Hq, nb]``.
    """
    q = np.asarray(q, dtype=np.float32)
    Hq = q.shape[0]
    Hkv = centroids.shape[0]
    assert Hq % Hkv == 0, "n_q_heads must be a multiple of n_kv_heads"
    c = np.repeat(centroids, Hq // Hkv, axis=0)
    return np.einsum("hd,hbd->hb", q, c)


def build_minmax(K: np.ndarray, block_size: int):
    """Per-block per-dimension key minimum and maximum over real tokens (the
    "minmax" (Quest) summaries of ``adakv/estimator.py:50-57``).

    K: ``[H, S, D]`` float32 -> ``(kmin, kmax)``, each ``[H, nb, D]`` float32.
    Minima and maxima are exact, so the result does not depend on order.
    """
    K = np.asarray(K, dtype=np.float32)
    H, S, D = K.shape
    nb = (S + block_size - 1) // block_size
    kmin = np.empty((H, nb, D), dtype=np.float32)
    kmax = np.empty((H, nb, D), dtype=np.float32)
    for b in range(nb):
        s, e = b * block_size, min((b + 1) * block_size, S)
        kmin[:, b] = K[:, s:e].min(axis=1)
        kmax[:, b] = K[:, s:e].max(axis=1)
    return kmin, kmax


def minmax_scores(q: np.ndarray, kmin: np.ndarray, kmax: np.ndarray) -> np.ndarray:
    """Quest upper bound of ``max_{k in block} q . k`` per (query head, block),
    the formula of ``adakv/estimator.py:76-79``:
    ``sum_d max(q_d, 0) kmax_d + min(q_d, 0) kmin_d``, with the summaries
    expanded over the GQA group as the reference's caller does.

    q: ``[Hq, D]``; kmin / kmax: ``[Hkv, nb, D]`` -> ``[Hq, nb]`` float32.
    """
    q = np.asarray(q, dtype=np.float32)
    Hq = q.shape[0]
    g = Hq // kmin.shape[0]
    kmn = np.repeat(kmin, g, axis=0)
    kmx = np.repeat(kmax, g, axis=0)
    qpos = np.clip(q, 0.0, None)[:, None, :]
    qneg = np.clip(q, None, 0.0)[:, None, :]
    return (qpos * kmx + qneg * kmn).sum(-1)


# --------------------------------------------------------------------------
# (c) entropy budget
# --------------------------------------------------------------------------
def budget_weights(scores: np.ndarray, policy: str, temperature: float = 1.0,
                   nucleus_p: float = 0.9) -> np.ndarray:
    """Per-head surplus weights, ``adakv/budget.py:28-42``.

    Entropy policy: ``p = softmax(scores / max(T, 1e-6))`` in float32, then
    ``-(p * log(clip(p, 1e-9))).sum() / log(max(nb, 2)) + 1e-6``; the division
    by the NumPy float64 scalar ``np.log(...)`` promotes the weight to float64
    (NumPy 2 promotion rules), exactly as in the reference.
    """
    nb = scores.shape[1]
    z = scores / max(temperature, 1e-6)
    z = z - z.max(axis=-1, keepdims=True)
    p = np.exp(z)
    p /= p.sum(axis=-1, keepdims=True)
    if policy == POLICY_ADAPTIVE:
        ent = -(p * np.log(np.clip(p, 1e-9, None))).sum(axis=-1) / np.log(max(nb, 2))
        return ent + 1e-6
    if policy == POLICY_NUCLEUS:
        ps = np.sort(p, axis=-1)[:, ::-1]
        cum = np.cumsum(ps, axis=-1)
        return (cum < nucleus_p).sum(axis=-1).astype(np.float64) + 1.0
    raise ValueError(f"unknown budget policy: {policy!r}")


def budget_bounds(nb: int, avg_budget: float, k_min: int, k_max: int,
                  n_sink_blocks: int, n_local_blocks: int, c_min: int):
    """``(lo, hi, target)`` as the reference computes them.

    ``adakv/reference.py:71-73`` passes ``min(k_min, nb)``, ``min(k_max, nb)``
    and ``floor = min(sink, nb) + min(local, nb) + c_min``; then
    ``adakv/budget.py:75-77`` sets ``lo = min(max(floor, k_min, 1), nb)``,
    ``hi = min(k_max, nb)``, ``target = clip(avg_budget, lo, hi)``.
    """
    k_min_c, k_max_c = min(k_min, nb), min(k_max, nb)
    floor = min(n_sink_blocks, nb) + min(n_local_blocks, nb) + c_min
    lo = min(max(int(floor), int(k_min_c), 1), nb)
    hi = min(int(k_max_c), nb)
    target = float(np.clip(avg_budget, lo, hi))
    return lo, hi, target


def allocate_budget(scores: np.ndarray, avg_budget: float, k_min: int, k_max: int,
                    n_sink_blocks: int = 1, n_local_blocks: int = 4, c_min: int = 1,
                    temperature: float = 1.0, policy: str = POLICY_ADAPTIVE,
                    nucleus_p: float = 0.9, return_raw: bool = False):
    """Per-head total block budget, ``adakv/budget.py:45-86``.

    ``k = clip(round_half_even(lo + (target-lo)*H * w / sum(w)), lo, hi)``;
    the fixed policy returns ``round(target)`` for every head
    (``budget.py:79-80``); ``nb <= 1`` returns ``min(max(k_min, 1), nb)``
    (``budget.py:72-73``).  With ``return_raw`` the unrounded
    ``lo + extra`` per head is returned too (for near-tie analysis).
    """
    H, nb = scores.shape
    raw = np.full((H,), np.nan)
    if nb <= 1:
        k = np.full((H,), min(max(min(k_min, nb), 1), nb), dtype=np.int64)
        return (k, raw) if return_raw else k
    lo, hi, target = budget_bounds(nb, avg_budget, k_min, k_max,
                                   n_sink_blocks, n_local_blocks, c_min)
    if policy == POLICY_FIXED:
        k = np.full((H,), int(round(target)), dtype=np.int64)
        return (k, np.full((H,), target)) if return_raw else k
    w = budget_weights(scores, policy, temperature, nucleus_p)
    surplus_total = max(target - lo, 0.0) * H
    extra = surplus_total * w / max(float(w.sum()), 1e-9)
    raw = lo + extra
    k = np.clip(np.round(raw), lo, hi).astype(np.int64)
    return (k, raw) if return_raw else k


# --------------------------------------------------------------------------
# (c) sink/local-forced top-k selection
# --------------------------------------------------------------------------
def selection_counts(k_per_head: np.ndarray, nb: int, n_sink_blocks: int,
                     n_local_blocks: int, c_min: int) -> np.ndarray:
    """Realised per-head selected count, ``adakv/selector.py:47-54``:
    ``min(max(k_h, min(sink + local + c_min, nb)), nb)``."""
    sink, local = min(n_sink_blocks, nb), min(n_local_blocks, nb)
    floor = min(sink + local + c_min, nb)
    return np.minimum(np.maximum(np.asarray(k_per_head, dtype=np.int64), floor), nb)


def select_blocks(scores: np.ndarray, k_per_head: np.ndarray, n_sink_blocks: int = 1,
                  n_local_blocks: int = 4, c_min: int = 1):
    """Boolean block mask and per-head count, ``adakv/selector.py:18-60``.

    Sink blocks ``[0, sink)`` and local blocks ``[nb-local, nb)`` get a
    ``+inf`` bias (float64 copy of the scores, ``selector.py:44-48``); each head
    keeps the first ``k_h'`` entries of the descending order.  Ties are broken
    by lowest block index (stable argsort of the negated keys).
    """
    H, nb = scores.shape
    sink, local = min(n_sink_blocks, nb), min(n_local_blocks, nb)
    biased = scores.astype(np.float64, copy=True)
    if sink:
        biased[:, :sink] = np.inf
    if local:
        biased[:, nb - local:] = np.inf
    order = np.argsort(-biased, axis=1, kind="stable")
    kh = selection_counts(k_per_head, nb, n_sink_blocks, n_local_blocks, c_min)
    mask = np.zeros((H, nb), dtype=bool)
    for h in range(H):
        mask[h, order[h, : kh[h]]] = True
        if sink:
            mask[h, :sink] = True
        if local:
            mask[h, nb - local:] = True
    return mask, mask.sum(axis=1)


# --------------------------------------------------------------------------
# (d) attention over the selected blocks
# --------------------------------------------------------------------------
def attend_mask(q: np.ndarray, K: np.ndarray, V: np.ndarray, mask: np.ndarray,
                block_size: int, sm_scale: float | None = None) -> np.ndarray:
    """Softmax attention of each query head over its selected tokens.

    Same math as ``adakv/reference.py:76-80`` (``q.K / sqrt(D)`` promoted to
    float64, masked full-row softmax, weighted sum of V), evaluated only over
    the selected tokens of the head's KV head.  q: ``[Hq, D]``, K/V:
    ``[Hkv, S, D]`` (not expanded), mask: ``[Hq, nb]`` -> ``[Hq, D]`` float64.
    """
    q = np.asarray(q, dtype=np.float32)
    Hq, D = q.shape
    Hkv, S, _ = K.shape
    g = Hq // Hkv
    scale = (1.0 / np.sqrt(D)) if sm_scale is None else float(sm_scale)
    out = np.zeros((Hq, D), dtype=np.float64)
    for h in range(Hq):
        blocks = np.nonzero(mask[h])[0]
        if blocks.size == 0:
            continue
        tok = (blocks[:, None] * block_size + np.arange(block_size)[None, :]).ravel()
        tok = tok[tok < S]
        kk = np.asarray(K[h // g, tok], dtype=np.float32)
        vv = np.asarray(V[h // g, tok], dtype=np.float32)
        a = (kk @ q[h]).astype(np.float64) * scale
        a -= a.max()
        w = np.exp(a)
        w /= w.sum()
        out[h] = w @ vv.astype(np.float64)
    return out


def attend_table(q, K, V, block_table, sel_lens, block_size, sm_scale=None):
    """Attention over exactly a given block table.

    Semantics of the reference kernel's ground truth
    ``tests/test_kernel_parity.py:25-43`` (``_ref_from_table``): the first
    ``sel_lens[h]`` entries of row ``h`` name the blocks of query head ``h``;
    tokens at or past ``S`` are masked (``kernels/block_sparse_decode.py:81-82``).
    Duplicate entries are counted once.
    """
    Hq = q.shape[0]
    nb = (K.shape[1] + block_size - 1) // block_size
    mask = np.zeros((Hq, nb), dtype=bool)
    for h in range(Hq):
        ids = np.asarray(block_table[h, : int(sel_lens[h])], dtype=np.int64)
        mask[h, ids] = True
    return attend_mask(q, K, V, mask, block_size, sm_scale)


def dense_attention(q, K, V, sm_scale=None):
    """Full attention, ``adakv/reference.py:36-41`` (GQA folded)."""
    nb = K.shape[1]
    mask = np.ones((q.shape[0], nb), dtype=bool)
    return attend_mask(q, K, V, mask, 1, sm_scale)


# --------------------------------------------------------------------------
# one decode step
# --------------------------------------------------------------------------
def decode_step(q, K, V, block_size=16, avg_budget=8, k_min=2, k_max=64,
                n_sink_blocks=1, n_local_blocks=4, c_min=1, temperature=1.0,
                policy=POLICY_ADAPTIVE, nucleus_p=0.9, sm_scale=None,
                centroids=None, estimator="centroid"):
    """One AdaKV decode step for one sequence, ``adakv/reference.py:44-84``.

    q: ``[Hq, D]``; K, V: ``[Hkv, S, D]`` (GQA folded).  ``centroids`` may be
    passed in (maintained incrementally by the caller) to skip the rebuild.
    Returns a dict with ``out [Hq, D]``, ``scores``, ``k`` (budget), ``raw``
    (unrounded budget), ``counts`` (realised) and ``mask``.
    """
    q = np.asarray(q, dtype=np.float32)
    if estimator == "minmax":
        kmin, kmax = build_minmax(K, block_size)
        scores = minmax_scores(q, kmin, kmax)
    elif estimator == "centroid":
        if centroids is None:
            centroids = build_centroids(K, block_size)
        scores = block_scores(q, centroids)
    else:
        raise ValueError(f"unknown estimator: {estimator!r}")
    k, raw = allocate_budget(scores, avg_budget, k_min, k_max, n_sink_blocks,
                             n_local_blocks, c_min, temperature, policy, nucleus_p,
                             return_raw=True)
    mask, counts = select_blocks(scores, k, n_sink_blocks, n_local_blocks, c_min)
    out = attend_mask(q, K, V, mask, block_size, sm_scale)
    return {"out": out, "scores": scores, "k": k, "raw": raw, "counts": counts,
            "mask": mask, "centroids": centroids}


# --------------------------------------------------------------------------
# parity helpers (selection near-ties)
# --------------------------------------------------------------------------
def compare_selection(scores, k_oracle, raw_oracle, mask_oracle, sets_gpu,
                      n_sink_blocks, n_local_blocks, c_min,
                      score_rel_tol=1e-6, budget_tol=1e-5):
    """Classify GPU-vs-oracle selection differences head by head.

    Returns ``(n_exact, n_budget_near_ties, n_score_near_ties, failures)``.
    A head passes when its GPU block set equals the oracle's, or when every
    difference is a documented near-tie:

    * budget near-tie: the counts differ by one and the oracle's unrounded
      budget ``lo + extra`` lies within ``budget_tol`` of a ``.5`` rounding
      boundary (the GPU sums the entropy in a different order: the weights
      agree to about 1e-7 relative, which moves a raw budget of ~64 by well
      under 1e-5);
    * score near-tie: the blocks in the symmetric difference all have
      scores within ``score_rel_tol`` (relative) of each other.
    """
    H, nb = scores.shape
    n_exact = n_budget = n_score = 0
    failures = []
    kh_oracle = selection_counts(k_oracle, nb, n_sink_blocks, n_local_blocks, c_min)
    for h in range(H):
        gset = np.zeros(nb, dtype=bool)
        gset[np.asarray(sets_gpu[h], dtype=np.int64)] = True
        if len(sets_gpu[h]) != int(gset.sum()):
            failures.append((h, "duplicate block ids"))
            continue
        omask = mask_oracle[h]
        kg = int(gset.sum())
        if kg != int(kh_oracle[h]):
            r = raw_oracle[h]
            if abs(kg - int(kh_oracle[h])) == 1 and np.isfinite(r) and \
                    abs((r - math.floor(r)) - 0.5) < budget_tol:
                n_budget += 1
                m2, _ = select_blocks(scores[h:h + 1], np.array([kg]), n_sink_blocks,
                                      n_local_blocks, c_min)
                omask = m2[0]
            else:
                failures.append((h, f"count {kg} != oracle {int(kh_oracle[h])}"))
                continue
        if np.array_equal(gset, omask):
            n_exact += 1
            continue
        a = np.nonzero(gset & ~omask)[0]
        b = np.nonzero(omask & ~gset)[0]
        sa = scores[h, a].astype(np.float64)
        sb = scores[h, b].astype(np.float64)
        scale = np.maximum(np.abs(np.concatenate([sa, sb])).max(), 1e-30)
        gap = max(sa.max() - sb.min(), sb.max() - sa.min())
        if a.size == b.size and gap / scale < score_rel_tol:
            n_score += 1
        else:
            failures.append((h, f"set differs: gpu-only {a[:8].tolist()} "
                                f"oracle-only {b[:8].tolist()} rel gap {gap / scale:.3e}"))
    return n_exact, n_budget, n_score, failures


# --------------------------------------------------------------------------
# (f4) H2O / SnapKV frozen-selection baselines (reference adakv/baselines.py)
# --------------------------------------------------------------------------
def _causal_importance(Q: np.ndarray, K: np.ndarray, q_first: int) -> np.ndarray:
    """Sum over query rows i in [q_first, S) of each row's causal softmax over
    the keys j <= i, in float64 (``baselines.py:69-83``, ``101-116``).
    ``Q, K : [H, S, D]`` (query heads); returns ``[H, S]`` float64."""
    H, S, D = K.shape
    Qw = Q[:, q_first:, :].astype(np.float64)
    logits = np.einsum("hwd,hjd->hwj", Qw, K.astype(np.float64)) / np.sqrt(D)
    pos = np.arange(q_first, S)[:, None]
    logits = np.where(np.arange(S)[None, :] <= pos, logits, -np.inf)
    logits = logits - logits.max(axis=2, keepdims=True)
    e = np.exp(logits)
    return (e / e.sum(axis=2, keepdims=True)).sum(axis=1)


def h2o_key_importance(Q: np.ndarray, K: np.ndarray) -> np.ndarray:
    """H2O's accumulated attention per key over every causal prompt query
    (``baselines.py:69-83``); ``[H, S]`` float32."""
    return _causal_importance(Q, K, 0).astype(np.float32)


def snapkv_key_importance(Q: np.ndarray, K: np.ndarray, obs_window: int = 32,
                          pool_kernel: int = 7) -> np.ndarray:
    """SnapKV: attention from the last ``obs_window`` queries, then a
    same-length max-pool over key positions with edge padding
    (``baselines.py:86-117``); ``[H, S]`` float32."""
    H, S, D = K.shape
    w = int(min(obs_window, S))
    imp = _causal_importance(Q, K, S - w)
    if pool_kernel > 1:
        pad = pool_kernel // 2
        xp = np.concatenate([np.repeat(imp[:, :1], pad, axis=1), imp,
                             np.repeat(imp[:, -1:], pad, axis=1)], axis=1)
        win = np.lib.stride_tricks.sliding_window_view(xp, pool_kernel, axis=1)
        imp = win.max(axis=2)
    return imp.astype(np.float32)


def retain_blocks(importance: np.ndarray, block_size: int, n_real: int, budget: int,
                  n_sink_blocks: int = 1, n_local_blocks: int = 4, c_min: int = 1) -> np.ndarray:
    """Fixed-budget retention: forced sink and local blocks plus the top content
    blocks by summed importance, ``k = min(max(budget, sink + local + c_min), nb)``
    blocks per head (``baselines.py:121-163``); ties to the lowest block index.
    Returns ``[H, nb]`` bool."""
    H = importance.shape[0]
    nb = (n_real + block_size - 1) // block_size
    imp = np.zeros((H, nb * block_size), dtype=np.float64)
    imp[:, :n_real] = importance[:, :n_real]
    blk = imp.reshape(H, nb, block_size).sum(axis=2)
    sink, local = min(n_sink_blocks, nb), min(n_local_blocks, nb)
    biased = blk.copy()
    biased[:, :sink] = np.inf
    if local:
        biased[:, nb - local:] = np.inf
    k = min(max(int(budget), min(sink + local + c_min, nb)), nb)
    order = np.argsort(-biased, axis=1, kind="stable")
    mask = np.zeros((H, nb), dtype=bool)
    np.put_along_axis(mask, order[:, :k], True, axis=1)
    mask[:, :sink] = True
    if local:
        mask[:, nb - local:] = True
    return mask


def frozen_decode_mask(fmask: np.ndarray, nb_now: int, n_sink_blocks: int,
                       n_local_blocks: int) -> np.ndarray:
    """The frozen prefill selection extended to ``nb_now`` blocks: content stays
    as frozen, sink and the current local window are forced
    (``baselines_rt.py:176-205``)."""
    H, nbp = fmask.shape
    m = np.zeros((H, nb_now), dtype=bool)
    m[:, :nbp] = fmask
    m[:, :min(n_sink_blocks, nb_now)] = True
    local = min(n_local_blocks, nb_now)
    if local:
        m[:, nb_now - local:] = True
    return m
