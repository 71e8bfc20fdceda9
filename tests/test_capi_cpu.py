"""C-ABI checks that need no GPU: the library loads, exports every function
``include/adakv_b200.h`` declares, and rejects bad arguments on the host
(before any CUDA call) with the documented codes and messages."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from adakv_b200 import _lib
from adakv_b200.build import LIB, build

HEADER = os.path.join(os.path.dirname(__file__), "..", "include", "adakv_b200.h")


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.lib()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(adakv_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ["adakv_abi_version", "adakv_last_error", "adakv_plan_table_width",
              "adakv_plan_workspace_bytes", "adakv_attend_workspace_bytes", "adakv_centroid_build",
              "adakv_kv_append", "adakv_centroid_refresh", "adakv_plan", "adakv_attend",
              "adakv_decode_step", "adakv_read_status"]:
        assert n in names, n


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s+(\w+)$", out, flags=re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for n in declared_functions():
        assert hasattr(lib, n)


def test_no_torch_in_the_abi():
    code = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    assert "torch" not in code.lower()
    out = subprocess.run(["ldd", LIB], capture_output=True, text=True).stdout
    assert "libtorch" not in out and "libc10" not in out


def test_abi_version(lib):
    assert lib.adakv_abi_version() == 2


def geo(**kw):
    d = dict(batch=1, n_q_heads=32, n_kv_heads=8, head_dim=128, block_size=16, max_seq_len=4096,
             nb_cap=256, dtype=_lib.DTYPE_BF16)
    d.update(kw)
    return _lib.Geometry(*[d[f] for f, _ in _lib.Geometry._fields_])


def params(**kw):
    d = dict(avg_budget=64.0, temperature=1.0, k_min=2, k_max=512, n_sink_blocks=1,
             n_local_blocks=4, c_min=1, policy=_lib.POLICY_ADAPTIVE, nucleus_p=0.9)
    d.update(kw)
    return _lib.SelectParams(*[d[f] for f, _ in _lib.SelectParams._fields_])


def test_table_width_and_workspace_sizes(lib):
    g, p = geo(), params()
    assert lib.adakv_plan_table_width(g, p) == 256          # min(k_max, nb_cap)
    assert lib.adakv_plan_table_width(g, params(k_max=64)) == 64
    assert lib.adakv_plan_table_width(g, params(k_max=2, n_sink_blocks=3, n_local_blocks=4)) == 8
    ws = lib.adakv_plan_workspace_bytes(g, p)
    assert ws > 0 and ws % 256 == 0
    assert lib.adakv_attend_workspace_bytes(g, 64) > 0
    assert lib.adakv_attend_workspace_bytes(g, 0) == 0


@pytest.mark.parametrize("bad,code,text", [
    (dict(n_q_heads=30), _lib.ERR_INVALID, "multiple"),
    (dict(head_dim=96), _lib.ERR_UNSUPPORTED, "head_dim"),
    (dict(block_size=8), _lib.ERR_UNSUPPORTED, "block_size"),
    (dict(nb_cap=10), _lib.ERR_INVALID, "nb_cap"),
    (dict(dtype=7), _lib.ERR_INVALID, "dtype"),
    (dict(batch=0), _lib.ERR_INVALID, "batch"),
    (dict(n_q_heads=64, n_kv_heads=2), _lib.ERR_UNSUPPORTED, "group"),
])
def test_geometry_validation(lib, bad, code, text):
    q = _lib.View(0x1000, 0, 128, 0)
    rc = lib.adakv_plan(geo(**bad), params(), q, 0x1000, None, 0x1000, 256, 0x1000, None, 0x1000,
                        1 << 30, None)
    assert rc == code
    assert text in lib.adakv_last_error().decode()


@pytest.mark.parametrize("bad,text", [
    (dict(policy=5), "budget_policy"),
    (dict(k_max=0), "k_max"),
    (dict(avg_budget=float("nan")), "avg_budget"),
    (dict(c_min=-1), "c_min"),
])
def test_param_validation(lib, bad, text):
    q = _lib.View(0x1000, 4096, 128, 0)
    rc = lib.adakv_plan(geo(), params(**bad), q, 0x1000, None, 0x1000, 512, 0x1000, None, 0x1000,
                        1 << 30, None)
    assert rc == _lib.ERR_INVALID
    assert text in lib.adakv_last_error().decode()


def test_pointer_and_workspace_validation(lib):
    g, p = geo(), params()
    good_q = _lib.View(0x1000, 4096, 128, 0)
    # misaligned q
    rc = lib.adakv_plan(g, p, _lib.View(0x1002, 4096, 128, 0), 0x1000, None, 0x1000, 512, 0x1000,
                        None, 0x1000, 1 << 30, None)
    assert rc == _lib.ERR_INVALID and "aligned" in lib.adakv_last_error().decode()
    # table too narrow
    rc = lib.adakv_plan(g, p, good_q, 0x1000, None, 0x1000, 8, 0x1000, None, 0x1000, 1 << 30, None)
    assert rc == _lib.ERR_INVALID and "table_width" in lib.adakv_last_error().decode()
    # workspace too small
    rc = lib.adakv_plan(g, p, good_q, 0x1000, None, 0x1000, 512, 0x1000, None, 0x1000, 64, None)
    assert rc == _lib.ERR_INVALID and "workspace" in lib.adakv_last_error().decode()
    # strides not multiples of 16 bytes
    kv = _lib.View(0x1000, 4096 * 128, 4096 * 128, 3)
    rc = lib.adakv_centroid_build(g, kv, None, 0x1000, None)
    assert rc == _lib.ERR_INVALID and "strides" in lib.adakv_last_error().decode()
    rc = lib.adakv_kv_append(g, kv, kv, kv, kv, 0, None, 0x1000, None)
    assert rc == _lib.ERR_INVALID


def test_python_wrappers_refuse_cpu_tensors():
    import torch
    from adakv_b200.attention import AdaKVCache
    from adakv_b200.kernels.block_sparse_decode import block_sparse_decode
    k = torch.zeros(2, 64, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        AdaKVCache(16).append_prefill(k, k)
    with pytest.raises(RuntimeError, match="CUDA"):
        block_sparse_decode(torch.zeros(4, 64), k, k, torch.zeros(4, 2, dtype=torch.int32),
                            torch.ones(4, dtype=torch.int32), 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        AdaKVCache(16, estimator="minmax").append_prefill(k, k)
    with pytest.raises(ValueError):
        AdaKVCache(16, estimator="bogus")


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def test_more_than_128_query_heads_are_rejected(lib):
    """The per-sequence entropy exchange covers at most 128 query heads: a larger
    geometry must fail on the host instead of dropping heads from the budget."""
    assert lib.adakv_plan_workspace_bytes(geo(n_q_heads=160, n_kv_heads=10), params()) == 0
    assert "128" in lib.adakv_last_error().decode()
    q = _lib.View(0x1000, 4096, 128, 0)
    rc = lib.adakv_decode_step(geo(n_q_heads=256, n_kv_heads=16), params(), q, q, q, None, None, 0,
                               0x1000, None, 0.1, 0x1000, 512, 0x1000, q, 0x1000, 1 << 30, None)
    assert rc == _lib.ERR_UNSUPPORTED and "128" in lib.adakv_last_error().decode()
    assert lib.adakv_plan_workspace_bytes(geo(n_q_heads=128, n_kv_heads=8), params()) > 0


def test_debug_knobs_validate_and_reset(lib):
    assert lib.adakv_debug_knob(99, 1) == _lib.ERR_INVALID
    assert lib.adakv_debug_knob(_lib.KNOB_WAIT_NS, -5) == _lib.ERR_INVALID
    assert lib.adakv_debug_knob(_lib.KNOB_STEP_PATH, 3) == _lib.ERR_INVALID
    assert lib.adakv_debug_knob(_lib.KNOB_STEP_CLUSTER, 3) == _lib.ERR_INVALID
    for knob, v in ((_lib.KNOB_WAIT_NS, 1000), (_lib.KNOB_FLAGS, 1), (_lib.KNOB_STEP_PATH, 1),
                    (_lib.KNOB_STEP_CLUSTER, 4)):
        assert lib.adakv_debug_knob(knob, v) == _lib.OK
        assert lib.adakv_debug_knob(knob, 0) == _lib.OK


def test_read_scores_and_status_sink_validate_on_the_host(lib):
    g = geo()
    ws = lib.adakv_plan_workspace_bytes(g, params())
    # nothing has run on this (fake, aligned) workspace address
    assert lib.adakv_read_scores(g, 0x100000, ws, 0x1000, 256, None) == _lib.ERR_INVALID
    assert "no decode step" in lib.adakv_last_error().decode()
    assert lib.adakv_read_scores(g, 0x100000, ws, 0x1000, 10, None) == _lib.ERR_INVALID
    assert lib.adakv_read_scores(g, 0x100000, 64, 0x1000, 256, None) == _lib.ERR_INVALID
    assert lib.adakv_set_status_sink(None, None, None) == _lib.ERR_INVALID


def test_one_kernel_step_workspace_covers_its_regions(lib):
    """Geometries the one-kernel step takes get its tagged-word regions too:
    scores (8 bytes per block and head), bitmaps and per-CTA partials."""
    small = lib.adakv_plan_workspace_bytes(geo(dtype=_lib.DTYPE_F32), params())
    fused = lib.adakv_plan_workspace_bytes(geo(), params())
    assert fused > small + 32 * 256 * 8


def test_noalloc_limit_counts_the_split_kv_partials(lib):
    """adakv_attend_noalloc's 4 MiB limit is adakv_attend_workspace_bytes: a
    geometry whose bitmaps alone are far below it but whose split-KV partials
    push it over is rejected on the host, with that byte count in the message."""
    g = geo(batch=128, n_q_heads=32, n_kv_heads=8, max_seq_len=65536, nb_cap=4096)
    need = lib.adakv_attend_workspace_bytes(g, 64)
    bitmaps = 128 * 32 * ((4096 + 31) // 32) * 4
    assert bitmaps + 512 < (4 << 20) < need
    v = _lib.View(0x1000, 1 << 20, 1 << 16, 128)
    rc = lib.adakv_attend_noalloc(g, v, v, v, 0x1000, 64, 0x1000, None, 0.1, v, None, None)
    assert rc == _lib.ERR_INVALID
    msg = lib.adakv_last_error().decode()
    assert str(need) in msg and "adakv_attend_workspace_bytes" in msg


def test_shard_selection_sizes_and_validation(lib):
    """The statistics-exchange selection: record size for the cfg4 shape,
    0 where it does not apply, and host-side argument checks that return
    before any CUDA call."""
    geo = _lib.geometry(1, 64, 8, 128, 16, 1 << 20, 65536, _lib.DTYPE_BF16)
    sp = _lib.select_params(256, 2, 1024, 1, 4, 1)
    cap_pad = 1020  # 1024 - 5 forced blocks, rounded up to an even count
    assert lib.adakv_shard_record_bytes(geo, sp) == 64 * (8 * 8 + cap_pad * 8)
    nuc = _lib.select_params(256, 2, 1024, 1, 4, 1, 1.0, "adaptive_nucleus")
    assert lib.adakv_shard_record_bytes(geo, nuc) == 0
    assert b"nucleus" in lib.adakv_last_error()
    geo2 = _lib.geometry(2, 64, 8, 128, 16, 1 << 20, 65536, _lib.DTYPE_BF16)
    assert lib.adakv_shard_record_bytes(geo2, sp) == 0
    wide = _lib.select_params(8000, 2, 8000, 1, 4, 1)
    assert lib.adakv_shard_record_bytes(geo, wide) == 0
    rec = ctypes.c_void_p(1 << 20)  # never dereferenced: validation fails first
    # a shard outside the sequence
    assert lib.adakv_shard_prep(geo, sp, rec, 40000, 40000, 40000, rec, None) == _lib.ERR_INVALID
    # misaligned record
    assert lib.adakv_shard_prep(geo, sp, rec, 32768, 0, 32768, 8, None) == _lib.ERR_INVALID
    # world / record stride
    assert lib.adakv_shard_clamp(geo, sp, rec, 32768, 0, 32768, rec, 1 << 20, 0, rec,
                                 None) == _lib.ERR_INVALID
    assert lib.adakv_shard_clamp(geo, sp, rec, 32768, 0, 32768, rec, 1000, 2, rec,
                                 None) == _lib.ERR_INVALID
    # rank outside the world
    assert lib.adakv_shard_finish(geo, sp, rec, 1 << 20, rec, 2, 2, 0, 32768, rec, 1024, rec,
                                  None, None) == _lib.ERR_INVALID
    # the adaptive policy needs the clamp terms; the table must be wide enough
    assert lib.adakv_shard_finish(geo, sp, rec, 1 << 20, None, 2, 0, 0, 32768, rec, 1024, rec,
                                  None, None) == _lib.ERR_INVALID
    assert lib.adakv_shard_finish(geo, sp, rec, 1 << 20, rec, 2, 0, 0, 32768, rec, 1000, rec,
                                  None, None) == _lib.ERR_INVALID


def test_peer_exchange_and_packed_combine_validate_on_the_host(lib):
    """Sizes of the peer-memory exchange buffer, and argument checks of the
    exchange and of the packed log-sum-exp merge that fail before any CUDA call."""
    assert lib.adakv_peer_buffer_bytes(2, 512) == 2 * 512 + (2 * 16 + 2) * 8
    assert lib.adakv_peer_buffer_bytes(0, 512) == 0
    assert lib.adakv_peer_buffer_bytes(2, 100) == 0
    buf = ctypes.c_void_p(1 << 20)  # never dereferenced
    assert lib.adakv_peer_exchange(buf, 512, buf, 0, 0, 512, buf, None, None) == _lib.ERR_INVALID
    assert lib.adakv_peer_exchange(buf, 512, buf, 2, 2, 512, buf, None, None) == _lib.ERR_INVALID
    assert lib.adakv_peer_exchange(buf, 100, buf, 2, 0, 512, buf, None, None) == _lib.ERR_INVALID
    assert lib.adakv_peer_exchange(buf, 1024, buf, 2, 0, 512, buf, None, None) == _lib.ERR_INVALID
    out = _lib.View(1 << 20, 64 * 128, 128, 0)
    assert lib.adakv_combine_packed(2, 1, 64, 128, _lib.DTYPE_BF16, buf, 64 * 128,
                                    out, None) == _lib.ERR_INVALID
    assert b"part_stride" in lib.adakv_last_error()
