"""ctypes binding of ``libadakv_b200.so`` (the C ABI in ``include/adakv_b200.h``).

The library is built in-tree by :mod:`adakv_b200.build`.  Loading fails loudly
when it is missing: there is no CPU or eager-torch fallback for any operator.
Torch is used only to hand device pointers and the current CUDA stream to the
library; no torch type crosses the C ABI.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

# the package's own build; ADAKV_LIB names another copy of the library (an
# installed build, or an alternative build to compare against)
LIB_PATH = os.environ.get("ADAKV_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                       "libadakv_b200.so")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
POLICY_FIXED, POLICY_ADAPTIVE, POLICY_NUCLEUS = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
ST_WAIT_TIMEOUT, ST_BAD_BLOCK_ID, ST_BAD_SEL_LEN, ST_BAD_SEQ_LEN = 1, 2, 4, 8

TORCH_DTYPES = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}
POLICIES = {"fixed": POLICY_FIXED, "adaptive": POLICY_ADAPTIVE,
            "adaptive_nucleus": POLICY_NUCLEUS}


class Geometry(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("n_q_heads", ctypes.c_int32),
                ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("block_size", ctypes.c_int32), ("max_seq_len", ctypes.c_int32),
                ("nb_cap", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class View(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_s", ctypes.c_int64)]


class SelectParams(ctypes.Structure):
    _fields_ = [("avg_budget", ctypes.c_double), ("temperature", ctypes.c_double),
                ("k_min", ctypes.c_int32), ("k_max", ctypes.c_int32),
                ("n_sink_blocks", ctypes.c_int32), ("n_local_blocks", ctypes.c_int32),
                ("c_min", ctypes.c_int32), ("policy", ctypes.c_int32),
                ("nucleus_p", ctypes.c_double)]


_P = ctypes.POINTER
_vp = ctypes.c_void_p
_SIGNATURES = {
    "adakv_abi_version": (ctypes.c_int, []),
    "adakv_last_error": (ctypes.c_char_p, []),
    "adakv_plan_table_width": (ctypes.c_int32, [_P(Geometry), _P(SelectParams)]),
    "adakv_plan_workspace_bytes": (ctypes.c_size_t, [_P(Geometry), _P(SelectParams)]),
    "adakv_attend_workspace_bytes": (ctypes.c_size_t, [_P(Geometry), ctypes.c_int32]),
    "adakv_centroid_build": (ctypes.c_int, [_P(Geometry), _P(View), _vp, _vp, _vp]),
    "adakv_kv_append": (ctypes.c_int, [_P(Geometry), _P(View), _P(View), _P(View), _P(View),
                                       ctypes.c_int32, _vp, _vp, _vp]),
    "adakv_centroid_refresh": (ctypes.c_int, [_P(Geometry), _P(View), ctypes.c_int32, _vp, _vp,
                                              _vp]),
    "adakv_plan": (ctypes.c_int, [_P(Geometry), _P(SelectParams), _P(View), _vp, _vp, _vp,
                                  ctypes.c_int32, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "adakv_attend": (ctypes.c_int, [_P(Geometry), _P(View), _P(View), _P(View), _vp,
                                    ctypes.c_int32, _vp, _vp, ctypes.c_float, _P(View), _vp,
                                    ctypes.c_size_t, _vp]),
    "adakv_decode_step": (ctypes.c_int, [_P(Geometry), _P(SelectParams), _P(View), _P(View),
                                         _P(View), _P(View), _P(View), ctypes.c_int32, _vp, _vp,
                                         ctypes.c_float, _vp, ctypes.c_int32, _vp, _P(View), _vp,
                                         ctypes.c_size_t, _vp]),
    "adakv_read_status": (ctypes.c_int, [_vp, _P(ctypes.c_uint32), _vp]),
    "adakv_estimate": (ctypes.c_int, [_P(Geometry), _P(View), _vp, _vp, _vp, ctypes.c_int32, _vp,
                                      ctypes.c_size_t, _vp]),
    "adakv_select": (ctypes.c_int, [_P(Geometry), _P(SelectParams), _vp, ctypes.c_int32, _vp, _vp,
                                    ctypes.c_int32, _vp, _vp, ctypes.c_size_t, _vp]),
    "adakv_attend_partial": (ctypes.c_int, [_P(Geometry), _P(View), _P(View), _P(View), _vp,
                                            ctypes.c_int32, _vp, ctypes.c_int32, _vp,
                                            ctypes.c_float, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "adakv_combine": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_int32, _vp, _vp, _P(View), _vp]),
    "adakv_combine_packed": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_int64,
                                            _P(View), _vp]),
    "adakv_peer_buffer_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_size_t]),
    "adakv_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, _P(ctypes.c_void_p), _vp]),
    "adakv_peer_free": (ctypes.c_int, [_vp]),
    "adakv_peer_open": (ctypes.c_int, [_vp, _P(ctypes.c_void_p)]),
    "adakv_peer_close": (ctypes.c_int, [_vp]),
    "adakv_peer_exchange": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_size_t, _vp, _vp, _vp]),
    "adakv_shard_record_bytes": (ctypes.c_size_t, [_P(Geometry), _P(SelectParams)]),
    "adakv_shard_prep": (ctypes.c_int, [_P(Geometry), _P(SelectParams), _vp, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_int32, _vp, _vp]),
    "adakv_shard_clamp": (ctypes.c_int, [_P(Geometry), _P(SelectParams), _vp, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_size_t,
                                         ctypes.c_int32, _vp, _vp]),
    "adakv_shard_finish": (ctypes.c_int, [_P(Geometry), _P(SelectParams), _vp, ctypes.c_size_t,
                                          _vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, _vp, ctypes.c_int32, _vp, _vp, _vp]),
    "adakv_minmax_build": (ctypes.c_int, [_P(Geometry), _P(View), _vp, _vp, _vp, _vp]),
    "adakv_minmax_refresh": (ctypes.c_int, [_P(Geometry), _P(View), ctypes.c_int32, _vp, _vp, _vp,
                                            _vp]),
    "adakv_estimate_minmax": (ctypes.c_int, [_P(Geometry), _P(View), _vp, _vp, _vp, _vp,
                                             ctypes.c_int32, _vp]),
    "adakv_attend_noalloc": (ctypes.c_int, [_P(Geometry), _P(View), _P(View), _P(View), _vp,
                                            ctypes.c_int32, _vp, _vp, ctypes.c_float, _P(View),
                                            _vp, _vp]),
    "adakv_set_status_sink": (ctypes.c_int, [_vp, _vp, _vp]),
    "adakv_read_scores": (ctypes.c_int, [_P(Geometry), _vp, ctypes.c_size_t, _vp, ctypes.c_int32,
                                         _vp]),
    "adakv_debug_knob": (ctypes.c_int, [ctypes.c_int32, ctypes.c_int64]),
    "adakv_last_path": (ctypes.c_int, [_vp]),
    "adakv_debug_timeline": (ctypes.c_int, [_P(Geometry), _vp, ctypes.c_size_t, _vp, ctypes.c_int32,
                                            _vp]),
    "adakv_importance_workspace_bytes": (ctypes.c_size_t, [_P(Geometry), ctypes.c_int32]),
    "adakv_stage": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t, _vp]),
    "adakv_key_importance": (ctypes.c_int, [_P(Geometry), _P(View), _P(View), ctypes.c_int32,
                                            ctypes.c_float, _vp, ctypes.c_int32, _vp, ctypes.c_size_t,
                                            _vp]),
}

KNOB_WAIT_NS, KNOB_FLAGS, KNOB_STEP_PATH, KNOB_STEP_CLUSTER = 1, 2, 3, 4

_lib = None
_lock = threading.Lock()


def lib():
    """Load (once) and return the C library; raises if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m adakv_b200.build` "
                        "(there is no CPU fallback for the AdaKV CUDA path)")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(rc: int) -> None:
    """Raise the reference's exception type for a non-zero return code."""
    if rc == OK:
        return
    msg = lib().adakv_last_error().decode(errors="replace")
    if rc == ERR_INVALID:
        raise ValueError(msg)
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("adakv_b200 runs on CUDA tensors only (no CPU fallback); "
                               "use the oracle package for CPU reference checks")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return TORCH_DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16")


def view4(t: torch.Tensor) -> View:
    """[B, H, S, D] (or [B, H, D] for q / out) view with a contiguous last dim."""
    if t.stride(-1) != 1:
        raise ValueError("the head_dim axis must be contiguous")
    if t.dim() == 4:
        return View(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))
    if t.dim() == 3:
        return View(t.data_ptr(), t.stride(0), t.stride(1), 0)
    raise ValueError(f"expected a 3-D or 4-D tensor, got {tuple(t.shape)}")


def stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def select_params(avg_budget, k_min=2, k_max=64, n_sink_blocks=1, n_local_blocks=4, c_min=1,
                  temperature=1.0, budget_policy="adaptive", nucleus_p=0.9) -> SelectParams:
    if budget_policy not in POLICIES:
        raise ValueError(f"unknown budget policy: {budget_policy!r}")
    return SelectParams(float(avg_budget), float(temperature), int(k_min), int(k_max),
                        int(n_sink_blocks), int(n_local_blocks), int(c_min),
                        POLICIES[budget_policy], float(nucleus_p))


def geometry(batch, n_q_heads, n_kv_heads, head_dim, block_size, max_seq_len, nb_cap,
             dtype) -> Geometry:
    return Geometry(int(batch), int(n_q_heads), int(n_kv_heads), int(head_dim), int(block_size),
                    int(max_seq_len), int(nb_cap), int(dtype))


# ---------------------------------------------------------------------------
# device status surfaced on the host without synchronising
# ---------------------------------------------------------------------------
class StatusSink:
    """A page-locked host word the kernels of one workspace write their
    ``ADAKV_ST_*`` bits to (``adakv_set_status_sink``).  :meth:`raise_if_set`
    is a plain host read: a failed step (a bounded device wait that ran out,
    a bad block id or sequence length) raises on the next call that checks,
    without a device synchronisation on the decode path."""

    def __init__(self, ws: torch.Tensor):
        self.word = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._view = self.word.numpy()
        with torch.cuda.device(ws.device):
            rc = lib().adakv_set_status_sink(ws.data_ptr(), self.word.data_ptr(),
                                             stream_ptr(ws.device))
        self.ok = rc == OK
        if not self.ok:
            raise RuntimeError("adakv_set_status_sink failed: "
                               + lib().adakv_last_error().decode(errors="replace"))

    def bits(self) -> int:
        return int(self._view[0])

    def clear(self) -> None:
        self._view[0] = 0

    def raise_if_set(self) -> None:
        bits = self.bits()
        if bits:
            raise RuntimeError(describe_status(bits))


def describe_status(bits: int) -> str:
    names = []
    if bits & ST_WAIT_TIMEOUT:
        names.append("a bounded device wait timed out (results of that call are not valid)")
    if bits & ST_BAD_BLOCK_ID:
        names.append("a block table entry was outside [0, n_blocks)")
    if bits & ST_BAD_SEL_LEN:
        names.append("a sel_lens entry exceeded the table width")
    if bits & ST_BAD_SEQ_LEN:
        names.append("a sequence length was outside [1, max_seq_len]")
    return f"adakv device status 0x{bits:x}: " + "; ".join(names or ["unknown bits"])


# ---------------------------------------------------------------------------
# workspace: one zero-initialised device buffer per (device, stream, kind),
# grown on demand, each with its status sink.  Calls that share one are
# ordered by their stream.
# ---------------------------------------------------------------------------
_workspaces: dict = {}
_sinks: dict = {}


def workspace(nbytes: int, device, kind: str = "plan") -> torch.Tensor:
    """The cached workspace of ``kind`` for the current stream of ``device``
    (zeroed on allocation, status sink attached).  While the stream is being
    captured into a CUDA graph, nothing may be allocated or synchronised: the
    workspace the same ``kind`` already has on this device is reused (the
    capture is ordered after the eager calls that created it)."""
    device = torch.device(device)
    key = (device.index, stream_ptr(device), kind)
    ws = _workspaces.get(key)
    if (ws is None or ws.numel() < nbytes) and torch.cuda.is_current_stream_capturing():
        for (idx, _, k), w in _workspaces.items():
            if idx == device.index and k == kind and w.numel() >= nbytes:
                return w
        raise ValueError(f"no {kind!r} workspace of {nbytes} bytes exists on cuda:{device.index}: "
                         "make one eager call before capturing the stream")
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
        _sinks[ws.data_ptr()] = StatusSink(ws)
    return ws


def sink_of(ws: torch.Tensor):
    return _sinks.get(ws.data_ptr())


def raise_if_failed(ws: torch.Tensor) -> None:
    """Raise if a kernel that used ``ws`` reported a status bit (host read, no sync)."""
    s = _sinks.get(ws.data_ptr())
    if s is not None:
        s.raise_if_set()


def read_status(ws: torch.Tensor) -> int:
    """Synchronise and return (and clear) the device status bits of a workspace."""
    out = ctypes.c_uint32(0)
    check(lib().adakv_read_status(ws.data_ptr(), ctypes.byref(out), stream_ptr(ws.device)))
    s = _sinks.get(ws.data_ptr())
    if s is not None:
        s.clear()
    return int(out.value)


def debug_knob(knob: int, value: int) -> None:
    """Test-only process-wide knobs (``adakv_debug_knob``); 0 restores the default."""
    check(lib().adakv_debug_knob(int(knob), int(value)))
