"""BatchedDecoder.graphed: a decode step replayed from a CUDA graph gives the
same output, selection and cache state as the eager step, step after step
(two decoders with the same prefill, one stepped eagerly, one by replay)."""
import numpy as np
import pytest
import torch

from adakv_b200.batch import BatchedDecoder

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("advance", [True, False])
def test_graphed_step_matches_eager(advance):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    B, Hq, Hkv, D, bs, S, cap = 2, 8, 2, 128, 16, 3000, 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    K = torch.randn((B, Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    lens = [S, S - 700]
    kw = dict(avg_budget=32, k_min=2, k_max=64)
    eager = BatchedDecoder(B, Hq, Hkv, D, bs, cap, torch.bfloat16, "cuda", **kw)
    graph = BatchedDecoder(B, Hq, Hkv, D, bs, cap, torch.bfloat16, "cuda", **kw)
    eager.load(K, V, lens)
    graph.load(K, V, lens)
    gs = graph.graphed(n_new=1, advance=advance)
    for step in range(3):
        q = torch.randn((B, Hq, D), device="cuda", generator=g).to(torch.bfloat16)
        kn = torch.randn((B, Hkv, 1, D), device="cuda", generator=g).to(torch.bfloat16)
        vn = torch.randn((B, Hkv, 1, D), device="cuda", generator=g).to(torch.bfloat16)
        ref = eager.step(q, k_new=kn, v_new=vn, advance=advance).clone()
        gs.q.copy_(q)
        gs.k_new.copy_(kn)
        gs.v_new.copy_(vn)
        out = gs().clone()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"step {step}"
        for a, b in zip(graph.selected_sets(), eager.selected_sets()):
            assert np.array_equal(np.sort(a), np.sort(b))
        assert graph.host_seq_lens == eager.host_seq_lens
        assert torch.equal(graph.seq_lens, eager.seq_lens)
    assert torch.equal(graph.k, eager.k) and torch.equal(graph.centroid, eager.centroid)
    assert graph.status() == 0 and eager.status() == 0
