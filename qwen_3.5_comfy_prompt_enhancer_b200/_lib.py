"""Bindings of the qlin C ABI (``include/qlin.h``).

``load()`` returns the ctypes handle of ``libqlin.so`` (diagnostics, the plan
query and the multi-GPU helpers); ``ext()`` returns the compiled torch-tensor
binding ``_qlin_ext`` that the Python entry points call.  Both are built
in-tree next to this file by ``build.py``.  There is no fallback: if either is
missing or fails to load, every entry point raises.
"""
import ctypes
import importlib
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqlin.so")

_P = ctypes.c_void_p
_I = ctypes.c_int64

# name -> argument types (every function returns int status unless listed in _RESTYPES)
SIGNATURES = {
    "qlin_version": [],
    "qlin_status_string": [ctypes.c_int],
    "qlin_last_error": [],
    "qlin_device_fault": [ctypes.c_int],
    "qlin_set_wait_limit_ns": [_I],
    "qlin_gemm_i8": [_P, _P, _I, _I, _P, _P, _I, _P, _I, _P, _I, _P],
    "qlin_gemm_w4": [_P, _P, _I, _I, _P, _P, _P, _I, _I, _P, _I, _P, _I, _P],
    "qlin_proj3": [_P, _P, _I, _I, _P, _P, _I, _P, _P, _I, _P, _P, _I, _P, _I, _P],
    "qlin_proj3_w4": [_P, _P, _I, _I, _P, _P, _P, _I, _P, _P, _P, _I, _P, _P, _P, _I, _I, _P, _I, _P],
    "qlin_mlp_gate_up": [_P, _P, _I, _I, _P, _P, _P, _P, _I, _P, _I, _P],
    "qlin_mlp_gate_up_quant": [_P, _P, _I, _I, _P, _P, _P, _P, _I, _P, _P, _P],
    "qlin_mlp_gate_up_quant_w4": [_P, _P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P],
    "qlin_quant_row": [_P, _I, _I, _I, _P, _P, _P],
    "qlin_rmsnorm_quant": [_P, _I, _P, _I, _I, ctypes.c_float, ctypes.c_int, _P, _P, _P],
    "qlin_norm_gated_quant": [_P, _P, _I, _P, _I, _I, _I, ctypes.c_float, _P, _P, _P],
    "qlin_norm_gated": [_P, _P, _I, _P, _I, _I, _I, ctypes.c_float, _P, _P],
    "qlin_gate_mul_quant": [_P, _P, _I, _I, _I, _I, _P, _P, _P],
    "qlin_silu_mul_quant": [_P, _P, _I, _I, _P, _P, _P],
    "qlin_gate_proj": [_P, _P, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P],
    "qlin_qk_norm_rope": [_P, _I, _P, _P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P, ctypes.c_float, ctypes.c_int,
                          ctypes.c_int, _I, _I, _P],
    "qlin_attn_decode": [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, ctypes.c_int, _I, _I, _P],
    "qlin_delta_decode": [_P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qlin_conv_silu": [_P, _I, _P, _I, _P, _P, _I, _I, ctypes.c_int, _P],
    "qlin_conv_state_update": [_P, _I, _P, _I, _I, _I, _I, _P],
    "qlin_conv_silu_update": [_P, _I, _P, _I, _P, _P, _I, _I, _P],
    "qlin_attn_prefill": [_P, _P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_int, _P],
    "qlin_delta_prefill": [_P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qlin_plan_small_m": [ctypes.c_int, ctypes.c_int, _I, _I, _I, _I, ctypes.c_int, _P],
    "qlin_max_active_clusters": [ctypes.c_int, ctypes.c_int, _I, ctypes.c_int, _I, ctypes.POINTER(ctypes.c_int64)],
    "qlin_ipc_get_handle": [_P, _P, ctypes.POINTER(ctypes.c_int64)],
    "qlin_ipc_open": [_P, _I, ctypes.POINTER(ctypes.c_void_p)],
    "qlin_ipc_close": [_P, _I],
    "qlin_dev_alloc": [_I, ctypes.POINTER(ctypes.c_void_p)],
    "qlin_dev_free": [_P],
    "qlin_peer_allgather": [_P, _P, _P, _P, _I, ctypes.c_int, ctypes.c_int, _P, _P],
    "qlin_peer_ll_bytes": [_P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)],
    "qlin_peer_allgather_ll": [_P, _I, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P],
    "qlin_peer_allgather_fenced": [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P],
    "qlin_peer_ll_send": [_P, _I, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P],
    "qlin_peer_ll_recv": [_P, _I, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P],
    "qlin_tp_gemm_w4_ll": [_I, _I, _P, _P, _P, _I, _I, _P, _I, _P, _I, _P, _P, ctypes.c_int, _P, _I, _P, _P,
                           ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P],
    "qlin_plan_dp": [ctypes.c_int, ctypes.c_int, _I, _I, _I, _I, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)],
    "qlin_peer_allgather_static": [_P, _I, _P, _P],
}
_RESTYPES = {
    "qlin_status_string": ctypes.c_char_p,
    "qlin_last_error": ctypes.c_char_p,
}


class GatherPart(ctypes.Structure):
    """``qlin_gather_part`` of include/qlin.h."""
    _fields_ = [("src", ctypes.c_void_p), ("src_ld", ctypes.c_int64), ("rows", ctypes.c_int64),
                ("row_bytes", ctypes.c_int64), ("dst_off", ctypes.c_int64), ("dst_ld", ctypes.c_int64)]


PEER_STATE_WORDS = 16  # QLIN_PEER_STATE_WORDS

_lib = None
_lock = threading.Lock()


def load():
    """Load (once) and return the ctypes handle of libqlin.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"qlin native library not found at {LIB_PATH}; build it first "
                    "(python -c 'import __graft_entry__ as g; g.build()')")
            lib = ctypes.CDLL(LIB_PATH)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


_ext = None


def ext():
    """Import (once) and return the ``_qlin_ext`` binding module."""
    global _ext
    if _ext is not None:
        return _ext
    load()  # same library, and the clearer error when it is missing
    with _lock:
        if _ext is None:
            try:
                _ext = importlib.import_module("._qlin_ext", __package__)
            except ImportError as e:
                raise RuntimeError(
                    f"qlin Python binding _qlin_ext not importable from {HERE} ({e}); build it first "
                    "(python -c 'import __graft_entry__ as g; g.build()')") from e
    return _ext


class QlinError(RuntimeError):
    """A qlin entry point returned a non-zero status."""

    def __init__(self, fn, status):
        lib = load()
        self.status = status
        msg = lib.qlin_last_error().decode(errors="replace")
        super().__init__(f"{fn}: {lib.qlin_status_string(status).decode()} ({status}): {msg}")


def check(fn, status):
    if status != 0:
        raise QlinError(fn, status)


PLAN_FIELDS = ("split", "gmax", "bs", "rb", "ab", "nbb", "smem", "mr", "alias", "level")


def plan_small_m(wbits, gate_up, M, K, tiles, wgrp=64, sms=148):
    """Launch plan of the small-M kernel (``qlin_plan_small_m``) as a dict."""
    out = (ctypes.c_int64 * len(PLAN_FIELDS))()
    check("qlin_plan_small_m", load().qlin_plan_small_m(wbits, int(bool(gate_up)), M, K, tiles, wgrp, sms, out))
    return dict(zip(PLAN_FIELDS, list(out)))
