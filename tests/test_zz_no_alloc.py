"""adakv_attend_noalloc (scratch in a fixed device array of the library, no
workspace) against adakv_attend (caller workspace) through the C ABI.

Kept in its own file, collected last, so it also runs after every other test
has used the library in the same process."""
import numpy as np
import pytest
import torch

from adakv_b200 import _lib
from adakv_b200.synth import make_decode_case, ragged_seq_lens

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2  # abs, bf16 outputs against the NumPy oracle


def _case(seed=7, B=3, Hq=16, Hkv=4, D=128, bs=16, S_max=3000):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    lens = ragged_seq_lens(seed, B, 200, S_max)
    case = make_decode_case(seed, B, Hq, Hkv, D, lens, bs, "bf16")
    rng = np.random.default_rng(seed + 1)
    nb_cap = (S_max + bs - 1) // bs
    width = 40
    table = np.zeros((B * Hq, width), dtype=np.int32)
    sel = np.zeros((B * Hq,), dtype=np.int32)
    for b in range(B):
        nb = (lens[b] + bs - 1) // bs
        for h in range(Hq):
            r = b * Hq + h
            n = int(rng.integers(0, min(width, nb) + 1))
            table[r, :n] = rng.permutation(nb)[:n]
            sel[r] = n
    dev = "cuda"
    q = torch.from_numpy(case.q).to(dev, torch.bfloat16)
    K = torch.zeros((B, Hkv, S_max, D), dtype=torch.bfloat16, device=dev)
    V = torch.zeros_like(K)
    for b in range(B):
        K[b, :, : lens[b]] = torch.from_numpy(case.K[b][:, : lens[b]]).to(dev, torch.bfloat16)
        V[b, :, : lens[b]] = torch.from_numpy(case.V[b][:, : lens[b]]).to(dev, torch.bfloat16)
    geo = _lib.geometry(B, Hq, Hkv, D, bs, S_max, nb_cap, _lib.DTYPE_BF16)
    return dict(geo=geo, q=q, K=K, V=V, table=torch.from_numpy(table).to(dev),
                sel=torch.from_numpy(sel).to(dev),
                seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev), width=width,
                scale=1.0 / np.sqrt(D), case=case, lens=lens, table_np=table, sel_np=sel, bs=bs)


def _attend_ws(c):
    L = _lib.lib()
    out = torch.empty_like(c["q"])
    nbytes = L.adakv_attend_workspace_bytes(c["geo"], c["width"])
    ws = torch.zeros((nbytes,), dtype=torch.uint8, device="cuda")
    _lib.check(L.adakv_attend(c["geo"], _lib.view4(c["q"]), _lib.view4(c["K"]), _lib.view4(c["V"]),
                              c["table"].data_ptr(), c["width"], c["sel"].data_ptr(),
                              c["seq_lens"].data_ptr(), c["scale"], _lib.view4(out),
                              ws.data_ptr(), nbytes, _lib.stream_ptr(out.device)))
    return out


def _attend_noalloc(c, status):
    L = _lib.lib()
    out = torch.empty_like(c["q"])
    _lib.check(L.adakv_attend_noalloc(c["geo"], _lib.view4(c["q"]), _lib.view4(c["K"]),
                                      _lib.view4(c["V"]), c["table"].data_ptr(), c["width"],
                                      c["sel"].data_ptr(), c["seq_lens"].data_ptr(), c["scale"],
                                      _lib.view4(out), status.data_ptr(),
                                      _lib.stream_ptr(out.device)))
    return out


def test_noalloc_attend_matches_workspace_attend_twice():
    """Same kernels, same launch shapes: the outputs are bit-identical to the
    workspace path on both calls (the second reuses the scratch the first left),
    and both match the NumPy oracle's attention over the same tables."""
    from oracle import adakv_oracle as O
    c = _case()
    ref = _attend_ws(c)
    status = torch.full((1,), 0xFF, dtype=torch.int32, device="cuda")
    for _ in range(2):  # two calls in a row reuse the same scratch
        out = _attend_noalloc(c, status)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), \
            f"differs from adakv_attend by {(out.float() - ref.float()).abs().max().item():.3e}"
        assert int(status.item()) == 0
    case, Hq = c["case"], c["q"].shape[1]
    got = out.float().cpu().numpy()
    for b, S in enumerate(c["lens"]):
        rows = slice(b * Hq, (b + 1) * Hq)
        want = O.attend_table(case.q[b], case.K[b, :, :S], case.V[b, :, :S], c["table_np"][rows],
                              c["sel_np"][rows], c["bs"], sm_scale=c["scale"])
        err = np.abs(got[b] - want).max()
        assert err <= BF16_TOL, f"sequence {b}: max abs err {err:.3e} against the oracle"
    # rows with an empty selection produce zeros, as in adakv_attend
    empty = (c["sel"] == 0).reshape(ref.shape[0], ref.shape[1])
    assert torch.all(out[empty] == 0)


def test_noalloc_attend_reports_bad_block_ids():
    c = _case(seed=9)
    c["table"][0, 0] = 1 << 20  # outside [0, nb): skipped and flagged
    c["sel"][0] = max(int(c["sel"][0].item()), 1)
    status = torch.zeros((1,), dtype=torch.int32, device="cuda")
    _attend_noalloc(c, status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.ST_BAD_BLOCK_ID
    c["table"][0, 0] = 0
    _attend_noalloc(c, status)  # the next call starts from a clear status word
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def test_noalloc_attend_rejects_oversized_geometry():
    c = _case()
    # 4096 rows x 2048 bitmap words x 4 B = 32 MiB > the fixed 4 MiB scratch
    big = _lib.geometry(256, 16, 4, 128, 16, 1 << 20, (1 << 20) // 16, _lib.DTYPE_BF16)
    out = torch.empty_like(c["q"])
    rc = _lib.lib().adakv_attend_noalloc(big, _lib.view4(c["q"]), _lib.view4(c["K"]),
                                         _lib.view4(c["V"]), c["table"].data_ptr(), c["width"],
                                         c["sel"].data_ptr(), c["seq_lens"].data_ptr(), c["scale"],
                                         _lib.view4(out), None, _lib.stream_ptr(out.device))
    assert rc == _lib.ERR_INVALID
    assert "maximum" in _lib.lib().adakv_last_error().decode()
