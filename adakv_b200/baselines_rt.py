"""H2O / SnapKV frozen-selection baselines on the device (reference
``adakv/baselines_rt.py``, same function names, arguments and results).

At the prefill call the retained block set of each query head is decided once
from the prompt's (Q, K) and frozen; every later decode step attends to it
(plus the sink blocks and the current local window) through the same
block-sparse attention kernel as AdaKV:

* per-key importance: ``adakv_key_importance``, the causal softmax of the
  last n prompt queries summed per key (n = S: H2O's accumulated attention;
  n = obs_window: SnapKV's observation window), computed per KV head without
  expanding the keys;
* SnapKV's same-length max-pool over key positions (torch ``max_pool1d``,
  ``-inf`` padding, which for a max equals the oracle's edge padding);
* the fixed-budget retention: per-block importance sums, then the library's
  own top-k (``adakv_select`` with the fixed policy: forced sink and local
  blocks, ``k = min(max(budget, sink + local + c_min), nb)`` blocks per head,
  ties to the lower block index).

Tensors follow the reference's layout: ``Q, K : [H, L, D]`` already expanded
to the query heads.  ``key_importance`` takes the unexpanded GQA views
``[B, Hq, L, D]`` / ``[B, Hkv, L, D]`` the patched model holds.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _lib

__all__ = [
    "expand_kv_heads",
    "key_importance",
    "h2o_key_importance_torch",
    "snapkv_key_importance_torch",
    "retain_blocks_torch",
    "h2o_retained_mask_torch",
    "snapkv_retained_mask_torch",
    "mask_to_block_table",
    "frozen_decode_block_table",
]


def expand_kv_heads(x: torch.Tensor, group: int) -> torch.Tensor:
    """``[Hkv, L, D] -> [Hq, L, D]`` by repeating each KV head ``group`` times."""
    return x.repeat_interleave(group, dim=0) if group > 1 else x


def key_importance(q: torch.Tensor, k: torch.Tensor, n_query: int, sm_scale: float | None = None):
    """Per-key importance ``[B * Hq, L]`` float32 from ``q [B, Hq, L, D]`` and
    ``k [B, Hkv, L, D]`` (CUDA, one dtype, head_dim 64 or 128): the last
    ``n_query`` query rows' causal softmax, summed per key."""
    _lib.require_cuda(q, k)
    B, Hq, L, D = q.shape
    Hkv = k.shape[1]
    if k.shape != (B, Hkv, L, D) or q.dtype != k.dtype:
        raise ValueError(f"q {tuple(q.shape)} / k {tuple(k.shape)} must share B, L, D and dtype")
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    n_query = int(min(max(n_query, 1), L))
    scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(D)
    nb = (L + 15) // 16
    geo = _lib.geometry(B, Hq, Hkv, D, 16, L, nb, _lib.TORCH_DTYPES[q.dtype])
    L_ = _lib.lib()
    imp = torch.empty((B * Hq, L), dtype=torch.float32, device=q.device)
    nbytes = L_.adakv_importance_workspace_bytes(geo, n_query)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        _lib.check(L_.adakv_key_importance(geo, _lib.view4(q), _lib.view4(k), n_query, scale,
                                           imp.data_ptr(), L, ws.data_ptr(), nbytes,
                                           _lib.stream_ptr(q.device)))
    return imp


@torch.no_grad()
def h2o_key_importance_torch(Q: torch.Tensor, K: torch.Tensor, chunk: int = 256) -> torch.Tensor:
    """Accumulated attention each key receives over all causal prompt queries
    (reference ``baselines_rt.py:43-62``).  ``Q, K : [H, L, D]``; returns
    ``[H, L]`` float32.  ``chunk`` is accepted for signature compatibility (the
    kernel tiles the queries itself)."""
    return key_importance(Q.unsqueeze(0), K.unsqueeze(0), Q.shape[1])


@torch.no_grad()
def snapkv_key_importance_torch(Q: torch.Tensor, K: torch.Tensor, obs_window: int = 32,
                                pool_kernel: int = 7) -> torch.Tensor:
    """SnapKV importance from the last ``obs_window`` queries with a key-axis
    max-pool (reference ``baselines_rt.py:65-82``).  ``Q, K : [H, L, D]``."""
    imp = key_importance(Q.unsqueeze(0), K.unsqueeze(0), int(min(obs_window, Q.shape[1])))
    return _pool(imp, pool_kernel)


def _pool(imp: torch.Tensor, pool_kernel: int) -> torch.Tensor:
    if pool_kernel <= 1:
        return imp
    return F.max_pool1d(imp.unsqueeze(1), kernel_size=pool_kernel, stride=1,
                        padding=pool_kernel // 2).squeeze(1)


@torch.no_grad()
def retain_blocks_torch(importance: torch.Tensor, block_size: int, n_real: int, budget: int,
                        n_sink_blocks: int = 1, n_local_blocks: int = 4,
                        c_min: int = 1) -> torch.Tensor:
    """Fixed-budget retained-block mask ``[H, nb]`` bool (reference
    ``baselines_rt.py:85-123``): forced sink and local blocks plus the top
    content blocks by summed importance."""
    _lib.require_cuda(importance)
    H = importance.shape[0]
    nb = (n_real + block_size - 1) // block_size
    imp = importance[:, :n_real].float()
    pad = nb * block_size - n_real
    if pad:
        imp = F.pad(imp, (0, pad), value=0.0)
    stride = (nb + 3) // 4 * 4  # 16-byte score rows
    scores = torch.zeros((H, stride), dtype=torch.float32, device=importance.device)
    scores[:, :nb] = imp.reshape(H, nb, block_size).sum(dim=2)
    sink, local = min(n_sink_blocks, nb), min(n_local_blocks, nb)
    k = min(max(int(budget), min(sink + local + c_min, nb)), nb)
    geo = _lib.geometry(1, H, H, 64, block_size, n_real, nb, _lib.TORCH_DTYPES[torch.float32])
    sp = _lib.select_params(k, 1, nb, n_sink_blocks, n_local_blocks, c_min, 1.0, "fixed", 0.9)
    L = _lib.lib()
    width = L.adakv_plan_table_width(geo, sp)
    table = torch.empty((H, width), dtype=torch.int32, device=importance.device)
    lens = torch.empty((H,), dtype=torch.int32, device=importance.device)
    ws = _lib.workspace(L.adakv_plan_workspace_bytes(geo, sp), importance.device)
    _lib.raise_if_failed(ws)
    with torch.cuda.device(importance.device):
        _lib.check(L.adakv_select(geo, sp, scores.data_ptr(), stride, None, table.data_ptr(), width,
                                  lens.data_ptr(), ws.data_ptr(), ws.numel(),
                                  _lib.stream_ptr(importance.device)))
    # entries past sel_lens are unspecified: send them to a spare column
    valid = torch.arange(width, device=importance.device)[None, :] < lens[:, None].long()
    idx = torch.where(valid, table.long(), torch.full_like(table, nb, dtype=torch.long))
    mask = torch.zeros((H, nb + 1), dtype=torch.bool, device=importance.device)
    mask.scatter_(1, idx, True)
    return mask[:, :nb]


def h2o_retained_mask_torch(Q, K, block_size: int = 16, budget: int = 8, n_sink_blocks: int = 1,
                            n_local_blocks: int = 4, c_min: int = 1, chunk: int = 256):
    """Frozen H2O retained-block mask ``[H, nb]`` from the prompt (Q, K)."""
    imp = h2o_key_importance_torch(Q, K, chunk=chunk)
    return retain_blocks_torch(imp, block_size, K.shape[1], budget, n_sink_blocks,
                               n_local_blocks, c_min)


def snapkv_retained_mask_torch(Q, K, block_size: int = 16, budget: int = 8, obs_window: int = 32,
                               pool_kernel: int = 7, n_sink_blocks: int = 1,
                               n_local_blocks: int = 4, c_min: int = 1):
    """Frozen SnapKV retained-block mask ``[H, nb]`` from the prompt (Q, K)."""
    imp = snapkv_key_importance_torch(Q, K, obs_window, pool_kernel)
    return retain_blocks_torch(imp, block_size, K.shape[1], budget, n_sink_blocks,
                               n_local_blocks, c_min)


def mask_to_block_table(mask: torch.Tensor):
    """Equal-count retained mask ``[H, nb]`` -> ``(block_table [H, k] int32,
    sel_lens [H] int32)``, ascending block ids (reference
    ``baselines_rt.py:151-171``)."""
    H, nb = mask.shape
    counts = mask.sum(dim=1)
    k = int(counts.max().item())
    if not bool((counts == k).all()):
        raise ValueError("mask_to_block_table expects an equal count per head")
    table = mask.nonzero(as_tuple=False)[:, 1].view(H, k).to(torch.int32).contiguous()
    return table, counts.to(torch.int32)


@torch.no_grad()
def frozen_decode_block_table(fmask: torch.Tensor, nb_now: int, n_sink_blocks: int,
                              n_local_blocks: int):
    """Decode-step ``(block_table, sel_lens)`` from the frozen prefill mask: the
    frozen content plus the sink blocks and the current local window
    (reference ``baselines_rt.py:174-205``)."""
    H, nbp = fmask.shape
    if nb_now < nbp:
        raise ValueError("decode block count must not shrink below prefill")
    dmask = torch.zeros((H, nb_now), dtype=torch.bool, device=fmask.device)
    dmask[:, :nbp] = fmask
    sink, local = min(n_sink_blocks, nb_now), min(n_local_blocks, nb_now)
    if sink:
        dmask[:, :sink] = True
    if local:
        dmask[:, nb_now - local:] = True
    return mask_to_block_table(dmask)
