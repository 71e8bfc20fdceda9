"""Seeded synthetic decode inputs with planted retrieval blocks and recency heads.

The reference's headline configurations use seeded Gaussian K/V/q with
structure planted per KV head (the reference's own tests plant a strongly
aligned block, ``tests/test_reference.py:24-32``):

* K, V ~ N(0, 1) ``[B, Hkv, S, D]``; q ~ N(0, 1) ``[B, Hq, D]``;
* for KV head ``h``, ``qhat`` = the normalised mean of its GQA group's queries;
* even KV heads (retrieval): ``planted_scale * qhat`` is added to every key of
  ``n_planted`` blocks drawn uniformly without replacement from ``[0, nb)``;
* odd KV heads (local): ``recency * (t / 16) * qhat`` is added to key ``t``;
* values are cast to the compute dtype after planting.

Draw order (fixed, so a seed names one input): q, then K, then V (float32
ziggurat normals of ``numpy.random.default_rng(seed)``), then for each
sequence ``b`` and each even KV head the planted block ids.  Ragged batches
keep ``[B, Hkv, S_max, D]`` storage; positions at or past ``seq_lens[b]``
hold noise that no kernel may read.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class DecodeCase:
    q: np.ndarray          # [B, Hq, D] float32 (already rounded to `dtype`)
    K: np.ndarray          # [B, Hkv, S_max, D] float32 (already rounded to `dtype`)
    V: np.ndarray          # [B, Hkv, S_max, D] float32 (already rounded to `dtype`)
    seq_lens: np.ndarray   # [B] int32
    planted: list          # per sequence: {kv_head: np.ndarray of block ids}
    dtype: str             # "fp32" | "bf16" | "fp16"
    block_size: int


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (nearest-even) and return float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "fp32":
        return x
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        # round to nearest even on the upper 16 bits; in uint32 arithmetic only
        # NaN patterns can wrap, and those are restored below
        u = x.view(np.uint32)
        r = (u >> np.uint32(16)) & np.uint32(1)
        r += np.uint32(0x7FFF)
        r += u
        r &= np.uint32(0xFFFF0000)
        out = r.view(np.float32)
        nan = np.isnan(x)
        if nan.any():
            out[nan] = np.nan
        return out
    raise ValueError(f"unknown dtype {dtype!r}")


def make_decode_case(seed: int, batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                     seq_lens, block_size: int = 16, dtype: str = "bf16",
                     n_planted: int = 4, planted_scale: float = 3.0,
                     recency: float = 0.02) -> DecodeCase:
    """Generate one seeded decode case (see module docstring for the recipe)."""
    rng = np.random.default_rng(seed)
    if np.isscalar(seq_lens):
        seq_lens = [int(seq_lens)] * batch
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    assert seq_lens.shape == (batch,)
    S_max = int(seq_lens.max())
    g = n_q_heads // n_kv_heads
    q = rng.standard_normal((batch, n_q_heads, head_dim), dtype=np.float32)
    K = rng.standard_normal((batch, n_kv_heads, S_max, head_dim), dtype=np.float32)
    V = rng.standard_normal((batch, n_kv_heads, S_max, head_dim), dtype=np.float32)
    planted = []
    for b in range(batch):
        S = int(seq_lens[b])
        nb = (S + block_size - 1) // block_size
        pb = {}
        for h in range(n_kv_heads):
            qm = q[b, h * g:(h + 1) * g].mean(axis=0)
            qhat = (qm / max(float(np.linalg.norm(qm)), 1e-12)).astype(np.float32)
            if h % 2 == 0:
                ids = np.sort(rng.choice(nb, size=min(n_planted, nb), replace=False))
                pb[h] = ids
                for blk in ids:
                    s, e = blk * block_size, min((blk + 1) * block_size, S)
                    K[b, h, s:e] += np.float32(planted_scale) * qhat
            else:
                t = np.arange(S, dtype=np.float32)
                K[b, h, :S] += (np.float32(recency) * (t / np.float32(16)))[:, None] * qhat[None, :]
        planted.append(pb)
    return DecodeCase(q=round_to_dtype(q, dtype), K=round_to_dtype(K, dtype),
                      V=round_to_dtype(V, dtype), seq_lens=seq_lens, planted=planted,
                      dtype=dtype, block_size=block_size)


def ragged_seq_lens(seed: int, batch: int, lo: int = 8192, hi: int = 131072) -> np.ndarray:
    """Per-sequence contexts drawn uniformly from ``[lo, hi]`` (seeded)."""
    rng = np.random.default_rng(seed + 1_000_003)
    return rng.integers(lo, hi + 1, size=batch).astype(np.int32)


def make_prefill_case(seed: int, Hq: int, Hkv: int, D: int, S: int):
    """Seeded prompt queries and keys for the H2O / SnapKV baselines, as the
    reference's baseline tests draw them (Gaussian, scale 0.5): ``Q [Hq, S, D]``,
    ``K, V [Hkv, S, D]`` and one decode query ``q [Hq, D]``, all float32."""
    rng = np.random.default_rng(seed)
    Q = (rng.standard_normal((Hq, S, D)) * 0.5).astype(np.float32)
    K = (rng.standard_normal((Hkv, S, D)) * 0.5).astype(np.float32)
    V = rng.standard_normal((Hkv, S, D)).astype(np.float32)
    q = (rng.standard_normal((Hq, D)) * 0.5).astype(np.float32)
    return Q, K, V, q
