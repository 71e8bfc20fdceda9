"""Host logic of the preallocated HF cache and the baselines' table helpers
(CPU tensors: the cache keeps its torch-copy route, no kernel runs)."""
import numpy as np
import pytest
import torch

from adakv_b200.baselines_rt import frozen_decode_block_table, mask_to_block_table
from adakv_b200.hf_cache import AdaKVCacheLayer, AdaKVStaticCache, layer_of
from oracle import adakv_oracle as O


def test_cache_layer_appends_in_place_and_reports_lengths():
    layer = AdaKVCacheLayer(max_cache_len=40, block_size=16)
    k = torch.randn(2, 3, 25, 8)
    v = torch.randn(2, 3, 25, 8)
    K, V = layer.update(k, v)
    assert layer.get_seq_length() == 25 and K.shape == (2, 3, 25, 8)
    assert torch.equal(K, k) and torch.equal(V, v)
    assert K.data_ptr() == layer.keys.data_ptr()  # a view of the preallocated buffer
    assert layer.get_mask_sizes(1) == (26, 0) and layer.get_max_cache_shape() == 40
    k2, v2 = torch.randn(2, 3, 1, 8), torch.randn(2, 3, 1, 8)
    K2, _ = layer.update(k2, v2)
    assert K2.shape[2] == 26 and torch.equal(K2[:, :, 25:], k2) and torch.equal(K2[:, :, :25], k)
    assert not layer.fused and layer_of(K2, 16) is None  # CPU: no centroid table
    layer.crop(20)
    assert layer.get_seq_length() == 20 and layer.keys.shape[2] == 20
    with pytest.raises(ValueError, match="holds 40"):
        layer.update(torch.randn(2, 3, 21, 8), torch.randn(2, 3, 21, 8))
    with pytest.raises(ValueError, match="do not fit"):
        layer.update(torch.randn(1, 3, 1, 8), torch.randn(1, 3, 1, 8))
    layer.reset()
    assert layer.get_seq_length() == 0
    with pytest.raises(NotImplementedError):
        layer.batch_repeat_interleave(2)


def test_static_cache_builds_one_layer_per_model_layer():
    class Cfg:
        num_hidden_layers = 3

        def get_text_config(self):
            return self

    cache = AdaKVStaticCache(Cfg(), max_cache_len=64, block_size=32)
    assert len(cache.layers) == 3 and cache.max_cache_len == 64
    cache.update(torch.randn(1, 2, 5, 8), torch.randn(1, 2, 5, 8), 1)
    assert cache.get_seq_length(1) == 5 and cache.get_seq_length(0) == 0
    with pytest.raises(ValueError):
        AdaKVCacheLayer(max_cache_len=64, block_size=24)
    with pytest.raises(ValueError):
        AdaKVStaticCache()


def test_frozen_decode_table_matches_oracle():
    rng = np.random.default_rng(7)
    H, nbp = 4, 20
    fmask = np.zeros((H, nbp), dtype=bool)
    for h in range(H):  # equal counts per head, sink and local included
        fmask[h, [0, 16, 17, 18, 19]] = True
        fmask[h, rng.choice(np.arange(1, 16), 3, replace=False)] = True
    for nb_now in (20, 21, 23):
        bt, sl = frozen_decode_block_table(torch.from_numpy(fmask), nb_now, 1, 4)
        ref = O.frozen_decode_mask(fmask, nb_now, 1, 4)
        got = np.zeros_like(ref)
        for h in range(H):
            got[h, bt[h, :int(sl[h])].numpy()] = True
            assert np.all(np.diff(bt[h, :int(sl[h])].numpy()) > 0)
        assert np.array_equal(got, ref)
    with pytest.raises(ValueError):
        mask_to_block_table(torch.tensor([[True, False], [True, True]]))
    with pytest.raises(ValueError):
        frozen_decode_block_table(torch.from_numpy(fmask), nbp - 1, 1, 4)


def test_cache_layer_rejects_mismatched_states():
    layer = AdaKVCacheLayer(max_cache_len=16, block_size=16)
    layer.update(torch.randn(1, 2, 3, 8), torch.randn(1, 2, 3, 8))
    with pytest.raises(ValueError, match="float32"):
        layer.update(torch.randn(1, 2, 1, 8, dtype=torch.float64), torch.randn(1, 2, 1, 8, dtype=torch.float64))
    with pytest.raises(ValueError, match="differ"):
        layer.update(torch.randn(1, 2, 1, 8), torch.randn(1, 2, 2, 8))
