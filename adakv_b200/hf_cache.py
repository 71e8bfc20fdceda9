"""Preallocated per-layer KV cache for a patched HuggingFace model.

    from adakv_b200.hf_cache import AdaKVStaticCache
    from adakv_b200.patch import patch_model
    patch_model(model, block_size=16, avg_budget=64)
    cache = AdaKVStaticCache(model.config, max_cache_len=prompt_len + max_new_tokens)
    model.generate(ids, past_key_values=cache, max_new_tokens=...)

HF's default ``DynamicCache`` concatenates every layer's keys and values on
every step (an O(S) copy per layer and token), and the reference rebuilds the
block centroids from the whole key cache on every decode step
(``adakv/patch.py:110``).  This cache holds each layer's K / V in one
preallocated ``[B, Hkv, max_cache_len, D]`` buffer and that layer's float32
centroid table ``[B, Hkv, ceil(max_cache_len / bs), D]`` beside it.  Every
``update`` (the prefill's prompt tokens, then one token per decode step) is
one ``adakv_kv_append`` launch: the new tokens are written into the buffers and
every block they touch gets its centroid recomputed in the same pass, reading
the new keys from the projection output rather than from the cache.  The
prefill therefore builds the table while it writes the cache, with one read of
the prompt keys (the reference builds it after prefill from the whole cache,
``adakv/attention.py:119-139``), and a decode step refreshes only the trailing
block.  ``update`` returns prefix views of the buffers, so nothing is copied;
``adakv_b200.patch.adakv_attention_forward`` recognises them and uses the
table as it stands.

Geometries the kernels do not cover (head_dim other than 64 / 128, a CPU
tensor) keep working: the tokens are copied with torch and the attention
function rebuilds its own table as it does for a ``DynamicCache``.
"""
from __future__ import annotations

import weakref

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _lib

# base address of a layer's key buffer -> the layer (for the attention function)
_BY_KEY_PTR: "weakref.WeakValueDictionary[int, AdaKVCacheLayer]" = weakref.WeakValueDictionary()


def layer_of(key: torch.Tensor, block_size: int):
    """The ``AdaKVCacheLayer`` whose key buffer ``key`` is a prefix view of, with
    a centroid table of ``block_size``-token blocks current for exactly
    ``key.shape[2]`` tokens, or None."""
    layer = _BY_KEY_PTR.get(key.data_ptr())
    if (layer is None or not layer.fused or layer.n != key.shape[2] or layer.keys is None
            or layer.block_size != block_size):
        return None
    if key.shape[:2] != layer._k.shape[:2] or key.stride() != layer._k.stride():
        return None
    return layer


class AdaKVCacheLayer(CacheLayerMixin):
    """One attention layer's preallocated K / V buffers and centroid table."""

    is_sliding = False
    is_compileable = False

    def __init__(self, max_cache_len: int, block_size: int = 16):
        super().__init__()
        if max_cache_len < 1:
            raise ValueError(f"max_cache_len must be >= 1 (got {max_cache_len})")
        if block_size not in (16, 32):
            raise ValueError(f"block_size must be 16 or 32 (got {block_size})")
        self.max_cache_len = int(max_cache_len)
        self.block_size = int(block_size)
        self.n = 0
        self.fused = False
        self.centroid = None
        self.max_batch_size = None
        self._k = self._v = None

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        B, Hkv, _, D = key_states.shape
        self.dtype, self.device = key_states.dtype, key_states.device
        self.max_batch_size = B
        shape = (B, Hkv, self.max_cache_len, D)
        self._k = torch.empty(shape, dtype=self.dtype, device=self.device)
        self._v = torch.empty(shape, dtype=self.dtype, device=self.device)
        self.fused = (self.device.type == "cuda" and D in (64, 128)
                      and self.dtype in _lib.TORCH_DTYPES)
        if self.fused:
            nb_cap = -(-self.max_cache_len // self.block_size)
            self.centroid = torch.empty((B, Hkv, nb_cap, D), dtype=torch.float32, device=self.device)
            _BY_KEY_PTR[self._k.data_ptr()] = self
        self.n = 0
        self.keys = self._k[:, :, :0]
        self.values = self._v[:, :, :0]
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        B, Hkv, n_new, D = key_states.shape
        if (B, Hkv, D) != (self._k.shape[0], self._k.shape[1], self._k.shape[3]):
            raise ValueError(f"key states {tuple(key_states.shape)} do not fit the cache "
                             f"{tuple(self._k.shape)}")
        if value_states.shape != key_states.shape:
            raise ValueError(f"value states {tuple(value_states.shape)} differ from the key "
                             f"states {tuple(key_states.shape)}")
        if key_states.dtype != self.dtype or value_states.dtype != self.dtype or \
                key_states.device != self.device or value_states.device != self.device:
            raise ValueError(f"key / value states must be {self.dtype} on {self.device}")
        S = self.n + n_new
        if S > self.max_cache_len:
            raise ValueError(f"AdaKVStaticCache holds {self.max_cache_len} tokens per layer; "
                             f"{S} requested")
        if n_new > 0:
            if self.fused:
                k = key_states if key_states.stride(-1) == 1 else key_states.contiguous()
                v = value_states if value_states.stride(-1) == 1 else value_states.contiguous()
                geo = _lib.geometry(B, Hkv, Hkv, D, self.block_size, S, self.centroid.shape[2],
                                    _lib.TORCH_DTYPES[self.dtype])
                with torch.cuda.device(self.device):
                    _lib.check(_lib.lib().adakv_kv_append(
                        geo, _lib.view4(self._k), _lib.view4(self._v), _lib.view4(k), _lib.view4(v),
                        n_new, None, self.centroid.data_ptr(), _lib.stream_ptr(self.device)))
            else:
                self._k[:, :, self.n:S].copy_(key_states)
                self._v[:, :, self.n:S].copy_(value_states)
        self.n = S
        self.keys = self._k[:, :, :S]
        self.values = self._v[:, :, :S]
        return self.keys, self.values

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.n + query_length, 0

    def get_seq_length(self) -> int:
        return self.n

    def get_max_cache_shape(self) -> int:
        return self.max_cache_len

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.n - abs(max_length)
        if 0 <= max_length < self.n:
            # the block holding the new end is recomputed by the next update
            # (adakv_kv_append rebuilds every block its tokens touch)
            self.n = max_length
            self.keys = self._k[:, :, :max_length]
            self.values = self._v[:, :, :max_length]

    def reset(self) -> None:
        self.n = 0
        if self.is_initialized:
            self.keys = self._k[:, :, :0]
            self.values = self._v[:, :, :0]

    def batch_repeat_interleave(self, repeats: int) -> None:
        raise NotImplementedError("AdaKVStaticCache has a fixed batch; beam search is not supported")

    def batch_select_indices(self, indices: torch.Tensor) -> None:
        raise NotImplementedError("AdaKVStaticCache has a fixed batch; beam search is not supported")

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        raise NotImplementedError("AdaKVStaticCache has a fixed batch; beam search is not supported")


class AdaKVStaticCache(Cache):
    """A ``Cache`` of ``num_layers`` (default: the config's
    ``num_hidden_layers``) ``AdaKVCacheLayer``s of ``max_cache_len`` tokens each."""

    def __init__(self, config=None, max_cache_len: int = 4096, block_size: int = 16,
                 num_layers: int | None = None):
        if num_layers is None:
            if config is None:
                raise ValueError("give a model config or num_layers")
            text = config.get_text_config() if hasattr(config, "get_text_config") else config
            num_layers = text.num_hidden_layers
        super().__init__(layers=[AdaKVCacheLayer(max_cache_len, block_size) for _ in range(num_layers)])
        self.block_size = int(block_size)
