"""cfg2 at full size: ragged batch of 64 sequences, contexts drawn from
[8K, 128K] (seeded), Llama-3.1-8B head shape, avg_budget 128, one launch
sequence for the whole batch.  Selections of sampled sequences are checked
against the oracle's budget + top-k on the GPU scores (exact up to the
documented near-ties) and outputs against a float64 evaluation over the
selected blocks."""
import numpy as np
import pytest
import torch

from adakv_b200.batch import BatchedDecoder
from adakv_b200.synth import ragged_seq_lens
from oracle import adakv_oracle as O

pytestmark = pytest.mark.gpu


def test_cfg2_ragged_batch_64():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    B, Hq, Hkv, D, bs = 64, 32, 8, 128, 16
    kw = dict(avg_budget=128, k_min=2, k_max=512)
    lens = ragged_seq_lens(0, B, 8192, 131072)
    cap = int(lens.max())
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(2)
    dec = BatchedDecoder(B, Hq, Hkv, D, bs, cap, torch.bfloat16, dev, **kw)
    for b in range(B):  # fill in place, one sequence at a time
        dec.k[b].normal_(generator=g)
        dec.v[b].normal_(generator=g)
    q = torch.randn((B, Hq, D), device=dev, generator=g).to(torch.bfloat16)
    # planted retrieval blocks on even KV heads of every sequence
    qm = q.float().view(B, Hkv, Hq // Hkv, D).mean(2)
    qhat = (qm / qm.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    for b in range(B):
        nb = -(-int(lens[b]) // bs)
        for h in range(0, Hkv, 2):
            for blk in torch.randint(0, nb, (4,), device=dev, generator=g).tolist():
                dec.k[b, h, blk * bs:(blk + 1) * bs] += 3.0 * qhat[b, h]
    dec.seq_lens.copy_(torch.from_numpy(lens))
    dec.host_seq_lens = [int(x) for x in lens]
    from adakv_b200 import _lib
    with torch.cuda.device(dec.device):
        _lib.check(_lib.lib().adakv_centroid_build(dec.geometry(), _lib.view4(dec.k),
                                                   dec.seq_lens.data_ptr(), dec.centroid.data_ptr(),
                                                   _lib.stream_ptr(dec.device)))
    scores = torch.zeros((B * Hq, dec.nb_cap), dtype=torch.float32, device=dev)
    dec.plan(q, scores_out=scores)
    sets = dec.selected_sets()
    out = dec.step(q).clone()
    assert dec.status() == 0
    torch.cuda.synchronize()
    sc_all = scores.view(B, Hq, -1).cpu().numpy()
    for b in (int(np.argmin(lens)), int(np.argmax(lens)), 7, 33, 63):
        nb = -(-int(lens[b]) // bs)
        sc = sc_all[b, :, :nb]
        k, raw = O.allocate_budget(sc, kw["avg_budget"], kw["k_min"], kw["k_max"], 1, 4, 1,
                                   return_raw=True)
        mask, _ = O.select_blocks(sc, k, 1, 4, 1)
        _, _, _, failures = O.compare_selection(sc, k, raw, mask, sets[b * Hq:(b + 1) * Hq], 1, 4, 1)
        assert not failures, (b, failures[:4])
        for h in (0, 13, 31):
            blocks = np.sort(sets[b * Hq + h])
            tok = (blocks[:, None] * bs + np.arange(bs)[None, :]).ravel()
            tok = torch.from_numpy(tok[tok < lens[b]]).to(dev)
            kk = dec.k[b, h // (Hq // Hkv), tok].double()
            vv = dec.v[b, h // (Hq // Hkv), tok].double()
            ref = torch.softmax((kk @ q[b, h].double()) / np.sqrt(D), 0) @ vv
            e = (out[b, h].double() - ref).abs().max().item()
            assert e < 2e-2, (b, h, e)
