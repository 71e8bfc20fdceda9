"""Plug the AdaKV decode path into a HuggingFace model (transformers >= 5).

Mirror of the reference's ``adakv/patch.py`` interface:

    from adakv_b200.patch import install_adakv, enable_adakv, disable_adakv, patch_model
    install_adakv(model); enable_adakv(block_size=16, avg_budget=64)
    # or: patch_model(model, block_size=16, avg_budget=64)
    ... model.generate(...) ...
    disable_adakv()

``adakv_attention_forward`` is registered as the attention implementation
"adakv" (``adakv/patch.py:90-124``).  Prefill (``q_len > 1``) stays dense
through SDPA, as in the reference; single-token decode runs the sparse path on
the device: estimator, entropy budget, top-k and block-sparse attention in
three kernel launches with no host synchronisation.

Differences from the reference, all on the performance side:

* The reference rebuilds every block centroid from the whole key cache on
  every decode step of every layer (``patch.py:110``).  Here each layer keeps
  its float32 centroid table between calls (keyed by the module, like the
  reference's ``_FROZEN``): the prefill pass builds it from the prompt keys,
  and each decode step refreshes only the blocks touched by the tokens
  appended since (``adakv_centroid_refresh``).  The centroids are bit-identical
  to a full rebuild.
* With ``adakv_b200.hf_cache.AdaKVStaticCache`` as the model's cache, the K / V
  live in preallocated per-layer buffers (no per-step concatenation) and the
  cache's own update writes each token and refreshes its block's centroid in
  one launch (the prompt's table is built while the prefill writes the cache);
  this function then uses that table as it stands.
* Batched decode (``B > 1``) without an attention mask (no padding: every
  sequence has the key length) runs the same batched kernels; with a mask it
  goes dense, as the reference does for every ``B != 1`` call (``patch.py:96``).

The H2O / SnapKV eviction baselines (``selection="h2o" | "snapkv"``,
``patch.py:57-87``): the single-sequence prefill call freezes each layer's
retained block set from the prompt's (Q, K) (``adakv_b200.baselines_rt``:
the importance kernel, SnapKV's max-pool, the library's fixed-budget top-k)
and still returns dense attention; each decode step then attends to the frozen
set plus the sink blocks and the current local window through the same
block-sparse attention kernel.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from . import baselines_rt as _brt
from . import hf_cache as _hf_cache
from .attention import record_selection, tracing_enabled

try:
    from transformers import AttentionInterface
except Exception:  # pragma: no cover - older layout
    from transformers.modeling_utils import AttentionInterface
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

# same keys and defaults as the reference's configuration (adakv/patch.py:43-48)
_ADAKV_CFG = dict(enabled=True, block_size=16, avg_budget=16, k_min=2, k_max=64,
                  n_sink_blocks=1, n_local_blocks=4, temperature=1.0,
                  estimator="centroid", budget_policy="adaptive",
                  c_min=1, nucleus_p=0.9,
                  selection="adakv", obs_window=32, pool_kernel=7, h2o_chunk=256)
_SDPA = ALL_ATTENTION_FUNCTIONS["sdpa"]


class _LayerState:
    """Centroid table of one attention layer: ``cbuf [B, Hkv, cap, D]`` float32,
    valid for the first ``n`` tokens of the layer's key cache."""

    __slots__ = ("cbuf", "mm", "n", "bs", "shape", "dtype", "device")

    def __init__(self):
        self.cbuf = None
        self.mm = None  # minmax estimator: [2, B, Hkv, cap, D] key minima / maxima
        self.n = 0
        self.bs = 0
        self.shape = None
        self.dtype = None
        self.device = None


# per-layer state keyed by id(module); cleared by enable_adakv / disable_adakv
_STATE: dict[int, _LayerState] = {}
# per-layer frozen retained-block mask [Hq, nb_prefill] of the eviction
# baselines, keyed by id(module) (the reference's _FROZEN, patch.py:55-58)
_FROZEN: dict[int, torch.Tensor] = {}


def _capture_frozen(module, query, key, cfg, sel):
    """Freeze this layer's retained block set from the prompt (reference
    ``patch.py:60-76``); the prefill output stays dense."""
    L, D = key.shape[2], key.shape[3]
    n_query = L if sel == "h2o" else int(min(cfg["obs_window"], L))
    imp = _brt.key_importance(query, key, n_query, sm_scale=1.0 / math.sqrt(D))
    if sel == "snapkv":
        imp = _brt._pool(imp, int(cfg["pool_kernel"]))
    _FROZEN[id(module)] = _brt.retain_blocks_torch(
        imp, int(cfg["block_size"]), L, int(cfg["avg_budget"]), int(cfg["n_sink_blocks"]),
        int(cfg["n_local_blocks"]), int(cfg["c_min"]))


def _frozen_decode(module, query, key, value, scaling, cfg):
    """One decode step over the layer's frozen set (reference ``patch.py:79-87``,
    then its block-sparse kernel)."""
    B, Hq, _, D = query.shape
    bs = int(cfg["block_size"])
    S = key.shape[2]
    nb_now = (S + bs - 1) // bs
    fmask = _FROZEN.get(id(module))
    if fmask is None:  # prefill not seen: attend to everything
        fmask = torch.ones((Hq, nb_now), dtype=torch.bool, device=query.device)
    bt, sl = _brt.frozen_decode_block_table(fmask, nb_now, int(cfg["n_sink_blocks"]),
                                            int(cfg["n_local_blocks"]))
    if tracing_enabled():
        record_selection(bt, sl, nb_now)
    sm_scale = float(scaling) if scaling is not None else 1.0 / math.sqrt(D)
    out = torch.empty((B, 1, Hq, D), dtype=query.dtype, device=query.device)
    q3 = query[:, :, 0, :]
    if q3.stride(-1) != 1:
        q3 = q3.contiguous()
    geo = _geometry(B, Hq, key.shape[1], D, bs, S, nb_now, query.dtype)
    L = _lib.lib()
    width = bt.shape[1]
    with torch.cuda.device(query.device):
        wa = _lib.workspace(L.adakv_attend_workspace_bytes(geo, width), query.device, "attend")
        _lib.raise_if_failed(wa)
        _lib.check(L.adakv_attend(geo, _lib.view4(q3), _lib.view4(key), _lib.view4(value),
                                  bt.data_ptr(), width, sl.data_ptr(), None, sm_scale,
                                  _lib.view4(out[:, 0]), wa.data_ptr(), wa.numel(),
                                  _lib.stream_ptr(query.device)))
    return out, None


def _geometry(B, Hq, Hkv, D, bs, S, nb_cap, dtype):
    return _lib.geometry(B, Hq, Hkv, D, bs, S, nb_cap, _lib.TORCH_DTYPES[dtype])


def _sync_centroids(module, key, Hq, bs, rebuild, minmax=False):
    """Bring the layer's centroid table (and, for the minmax estimator, its
    key minima / maxima) up to date with ``key [B, Hkv, S, D]``."""
    B, Hkv, S, D = key.shape
    st = _STATE.get(id(module))
    if st is None:
        st = _STATE[id(module)] = _LayerState()
    nb = (S + bs - 1) // bs
    shape = (B, Hkv, D)
    stale = (st.cbuf is None or st.shape != shape or st.bs != bs or st.dtype != key.dtype
             or st.device != key.device or st.n > S)
    rebuild = rebuild or stale
    if stale or st.cbuf.shape[2] < nb:
        cap = max(nb, 64, 0 if stale else 2 * st.cbuf.shape[2])
        buf = torch.empty((B, Hkv, cap, D), dtype=torch.float32, device=key.device)
        if not rebuild:  # capacity growth: keep the valid rows
            buf[:, :, : st.cbuf.shape[2]].copy_(st.cbuf)
        st.cbuf = buf
    st.shape, st.bs, st.dtype, st.device = shape, bs, key.dtype, key.device
    geo = _geometry(B, Hq, Hkv, D, bs, S, st.cbuf.shape[2], key.dtype)
    L = _lib.lib()
    stream = _lib.stream_ptr(key.device)
    full = rebuild or S - st.n > S // 2
    if full:
        _lib.check(L.adakv_centroid_build(geo, _lib.view4(key), None, st.cbuf.data_ptr(), stream))
    elif S > st.n:
        _lib.check(L.adakv_centroid_refresh(geo, _lib.view4(key), S - st.n, None,
                                            st.cbuf.data_ptr(), stream))
    if minmax:
        if st.mm is None or st.mm.shape[1:] != (B, Hkv, st.cbuf.shape[2], D):
            st.mm = torch.empty((2, B, Hkv, st.cbuf.shape[2], D), dtype=torch.float32,
                                device=key.device)
            full = True
        if full:
            _lib.check(L.adakv_minmax_build(geo, _lib.view4(key), None, st.mm[0].data_ptr(),
                                            st.mm[1].data_ptr(), stream))
        elif S > st.n:
            _lib.check(L.adakv_minmax_refresh(geo, _lib.view4(key), S - st.n, None,
                                              st.mm[0].data_ptr(), st.mm[1].data_ptr(), stream))
    st.n = S
    return st


def adakv_attention_forward(module, query, key, value, attention_mask, scaling, dropout=0.0,
                            **kwargs):
    """HF attention function (reference ``adakv/patch.py:90-121``).

    ``query [B, Hq, q_len, D]``, ``key`` / ``value [B, Hkv, S, D]``; returns
    ``(out [B, q_len, Hq, D], None)``."""
    cfg = _ADAKV_CFG
    B, Hq, q_len, D = query.shape
    sel = cfg.get("selection", "adakv")
    if sel not in ("adakv", "h2o", "snapkv"):
        raise ValueError(f"unknown selection: {sel!r}")
    if sel != "adakv":
        if not cfg["enabled"] or B != 1 or not query.is_cuda or D not in (64, 128):
            return _SDPA(module, query, key, value, attention_mask=attention_mask, scaling=scaling,
                         dropout=dropout, **kwargs)
        if q_len > 1:  # prefill: freeze the retained set, return dense attention
            _capture_frozen(module, query, key, cfg, sel)
            return _SDPA(module, query, key, value, attention_mask=attention_mask, scaling=scaling,
                         dropout=dropout, **kwargs)
        _lib.require_cuda(query, key, value)
        return _frozen_decode(module, query, key, value, scaling, cfg)
    sparse = cfg["enabled"] and q_len == 1 and (B == 1 or attention_mask is None)
    ext = None  # a preallocated cache layer whose centroid table is already current
    if cfg["enabled"] and cfg["estimator"] == "centroid" and query.is_cuda:
        ext = _hf_cache.layer_of(key, int(cfg["block_size"]))
    if not sparse:
        if cfg["enabled"] and q_len > 1 and query.is_cuda and D in (64, 128) and ext is None:
            # prompt keys are final for these positions: build the table now
            with torch.cuda.device(query.device):
                _sync_centroids(module, key, Hq, cfg["block_size"], rebuild=True,
                                minmax=cfg["estimator"] == "minmax")
        return _SDPA(module, query, key, value, attention_mask=attention_mask, scaling=scaling,
                     dropout=dropout, **kwargs)

    _lib.require_cuda(query, key, value)
    if cfg["estimator"] not in ("centroid", "minmax"):
        raise ValueError(f"unknown estimator: {cfg['estimator']!r}")
    minmax = cfg["estimator"] == "minmax"
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("query, key and value must share one dtype")
    bs = int(cfg["block_size"])
    _, Hkv, S, _ = key.shape
    sm_scale = float(scaling) if scaling is not None else 1.0 / math.sqrt(D)
    with torch.cuda.device(query.device):
        if ext is not None:
            st, cbuf = None, ext.centroid
        else:
            st = _sync_centroids(module, key, Hq, bs, rebuild=False, minmax=minmax)
            cbuf = st.cbuf
        sp = _lib.select_params(cfg["avg_budget"], cfg["k_min"], cfg["k_max"],
                                cfg["n_sink_blocks"], cfg["n_local_blocks"], cfg["c_min"],
                                cfg["temperature"], cfg["budget_policy"], cfg["nucleus_p"])
        geo = _geometry(B, Hq, Hkv, D, bs, S, cbuf.shape[2], query.dtype)
        L = _lib.lib()
        width = L.adakv_plan_table_width(geo, sp)
        if width < 1:
            _lib.check(_lib.ERR_INVALID)
        block_table = torch.empty((B * Hq, width), dtype=torch.int32, device=query.device)
        sel_lens = torch.empty((B * Hq,), dtype=torch.int32, device=query.device)
        out = torch.empty((B, 1, Hq, D), dtype=query.dtype, device=query.device)
        ws = _lib.workspace(L.adakv_plan_workspace_bytes(geo, sp), query.device)
        _lib.raise_if_failed(ws)  # a failure an earlier call reported (host read, no sync)
        q3 = query[:, :, 0, :]
        if q3.stride(-1) != 1:
            q3 = q3.contiguous()
        o3 = out[:, 0]  # [B, Hq, D] view of the [B, 1, Hq, D] output
        if minmax:
            # Quest scores, then the same budget + top-k and block-sparse attention
            scores = torch.empty((B * Hq, cbuf.shape[2]), dtype=torch.float32,
                                 device=query.device)
            stream = _lib.stream_ptr(query.device)
            _lib.check(L.adakv_estimate_minmax(geo, _lib.view4(q3), st.mm[0].data_ptr(),
                                               st.mm[1].data_ptr(), None, scores.data_ptr(),
                                               scores.stride(0), stream))
            _lib.check(L.adakv_select(geo, sp, scores.data_ptr(), scores.stride(0), None,
                                      block_table.data_ptr(), width, sel_lens.data_ptr(),
                                      ws.data_ptr(), ws.numel(), stream))
            wa = _lib.workspace(L.adakv_attend_workspace_bytes(geo, width), query.device, "attend")
            _lib.check(L.adakv_attend(geo, _lib.view4(q3), _lib.view4(key), _lib.view4(value),
                                      block_table.data_ptr(), width, sel_lens.data_ptr(), None,
                                      sm_scale, _lib.view4(o3), wa.data_ptr(), wa.numel(), stream))
            if tracing_enabled() and B == 1:
                record_selection(block_table, sel_lens, (S + bs - 1) // bs)
            return out, None
        _lib.check(L.adakv_decode_step(
            geo, sp, _lib.view4(q3), _lib.view4(key), _lib.view4(value), None, None, 0,
            cbuf.data_ptr(), None, sm_scale, block_table.data_ptr(), width,
            sel_lens.data_ptr(), _lib.view4(o3), ws.data_ptr(), ws.numel(),
            _lib.stream_ptr(query.device)))
    if tracing_enabled() and B == 1:
        record_selection(block_table, sel_lens, (S + bs - 1) // bs)
    return out, None


AttentionInterface.register("adakv", adakv_attention_forward)


def install_adakv(model):
    """Route the model's attention through ``adakv_attention_forward``."""
    try:
        model.set_attn_implementation("adakv")
    except Exception:
        model.config._attn_implementation = "adakv"
    return model


def enable_adakv(**cfg):
    """Update the configuration (reference keys) and turn the sparse path on."""
    _ADAKV_CFG.update(cfg)
    _ADAKV_CFG["enabled"] = True
    _STATE.clear()
    _FROZEN.clear()  # frozen masks of a previous configuration


def disable_adakv():
    """Every call goes dense (SDPA) until ``enable_adakv``."""
    _ADAKV_CFG["enabled"] = False
    _STATE.clear()
    _FROZEN.clear()


def patch_model(model, block_size=16, avg_budget=16, **cfg):
    """``install_adakv`` + ``enable_adakv(block_size=..., avg_budget=..., **cfg)``."""
    install_adakv(model)
    enable_adakv(block_size=block_size, avg_budget=avg_budget, **cfg)
    return model
