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


@pytest.mark.parametrize("path", [1, 2], ids=["chain", "one_kernel"])
def test_step_writes_output_into_pinned_host_memory(path):
    """``step(out=<page-locked host tensor>)``: the attention kernel writes the
    result straight into mapped host memory, bit-identical to the device output."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from adakv_b200 import _lib
    B, Hq, Hkv, D, bs, S = 1, 32, 8, 128, 16, 20000
    g = torch.Generator(device="cuda").manual_seed(4)
    K = torch.randn((B, Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn((B, Hkv, S, D), device="cuda", generator=g).to(torch.bfloat16)
    dec = BatchedDecoder(B, Hq, Hkv, D, bs, S, torch.bfloat16, "cuda", avg_budget=64, k_max=512)
    dec.load(K, V, [S])
    q = torch.randn((B, Hq, D), device="cuda", generator=g).to(torch.bfloat16)
    kn = torch.randn((B, Hkv, 1, D), device="cuda", generator=g).to(torch.bfloat16)
    host = torch.zeros((B, Hq, D), dtype=torch.bfloat16).pin_memory()
    _lib.debug_knob(_lib.KNOB_STEP_PATH, path)
    try:
        ref = dec.step(q, k_new=kn, v_new=kn, advance=False).clone()
        dec.step(q, k_new=kn, v_new=kn, advance=False, out=host)
        torch.cuda.synchronize()
        assert dec.last_path() == path
    finally:
        _lib.debug_knob(_lib.KNOB_STEP_PATH, 0)
    assert torch.equal(host, ref.cpu())
    with pytest.raises(ValueError):
        dec.step(q, out=torch.zeros((B, Hq, D), dtype=torch.bfloat16))  # pageable host memory
    assert dec.status() == 0


@pytest.mark.parametrize("nbytes", [16, 12288, 12290, 1 << 20])
def test_stage_copies_pinned_host_rows(nbytes):
    """adakv_stage (through ``batch.stage``): a page-locked host row, and a
    device tensor, copied into device memory byte for byte, also at an offset
    into a larger pinned buffer and with a tail that is not a multiple of 16."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from adakv_b200.batch import stage
    g = torch.Generator().manual_seed(nbytes)
    host = torch.randint(0, 256, (2 * nbytes + 64,), dtype=torch.uint8, generator=g).pin_memory()
    for off in (0, 48):
        src = host[off:off + nbytes]
        dst = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        stage(dst, src)
        torch.cuda.synchronize()
        assert torch.equal(dst.cpu(), src)
    dev_src = host[:nbytes].cuda()
    dst = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    stage(dst, dev_src)
    assert torch.equal(dst, dev_src)
    with pytest.raises(ValueError):
        stage(dst, host[:nbytes].clone())  # pageable host memory
    with pytest.raises(ValueError):
        stage(dst, host[:nbytes - 1])      # size mismatch
