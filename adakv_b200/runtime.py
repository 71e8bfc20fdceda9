"""Decode-loop glue (mirror of the reference's ``adakv.runtime``).

* :func:`update_cache_decode` (``adakv/runtime.py:43-60``): appends one token's
  K/V in place (no full-cache ``torch.cat``) and recomputes the touched block's
  centroid from its tokens, so it equals a rebuild exactly.
* :func:`adakv_decode_step` (``adakv/runtime.py:85-112``): ``[1, Hq, 1, D]`` in,
  ``[1, Hq, 1, D]`` out, selection + attention on the device.  The reference's
  ``backend`` switch (Triton / torch) is kept for signature compatibility; the
  only backend is the CUDA kernel ("auto" or "cuda"), there is no CPU fallback.
"""
from __future__ import annotations

import math

from .attention import AdaKVCache, _decode


def update_cache_decode(cache: AdaKVCache, k_t, v_t):
    """Append one decoded token's KV ``[Hkv, 1, D]`` and refresh its block centroid."""
    return cache.append_decode(k_t, v_t)


def adakv_decode_step(
    q,
    cache: AdaKVCache,
    avg_budget: int,
    k_min: int = 2,
    k_max: int = 64,
    n_sink_blocks: int = 1,
    n_local_blocks: int = 4,
    temperature: float = 1.0,
    backend: str = "auto",
):
    """One AdaKV decode step. ``q`` ``[1, Hq, 1, D]`` -> ``[1, Hq, 1, D]``."""
    if backend not in ("auto", "cuda"):
        raise ValueError(f"backend {backend!r} is not available: the B200 build runs the CUDA "
                         "kernel only (use the oracle package for CPU reference results)")
    if q.dim() != 4 or q.shape[0] != 1 or q.shape[2] != 1:
        raise ValueError("q must be [1, Hq, 1, D] (batched decode: adakv_b200.batch)")
    qh = q[0, :, 0, :]
    out = _decode(qh, cache, avg_budget, k_min, k_max, n_sink_blocks, n_local_blocks, temperature,
                  "centroid", "adaptive", 1, 1.0 / math.sqrt(q.shape[-1]))
    return out.unsqueeze(0).unsqueeze(2)
