"""ctypes binding of ``libtaomate_b200.so`` (the C ABI in include/taomate_b200.h).

The library is built in-tree by :mod:`taomate_b200.build`.  Loading fails
loudly: there is no fallback implementation of any entry point.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

from . import build as _build

_LIB: Optional[ctypes.CDLL] = None
_LOCK = threading.Lock()

TM_OK = 0
TM_ERR_INVALID_ARGUMENT = 1
TM_ERR_ALIGNMENT = 2
TM_ERR_UNSUPPORTED = 3
TM_ERR_CUDA = 4
TM_ERR_DEVICE = 5

TM_DTYPE_BF16 = 0
TM_DTYPE_F32 = 1
TM_KV_SOURCE_CACHE = 0
TM_KV_SOURCE_NEW = 1

c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p


class NormRopeJob(ctypes.Structure):
    _fields_ = [("x", c_vp), ("out", c_vp), ("norm_weight", c_vp), ("cos", c_vp), ("sin", c_vp),
                ("x_batch_stride", c_i64), ("x_row_stride", c_i64),
                ("out_group_stride", c_i64), ("out_batch_stride", c_i64),
                ("out_row_stride", c_i64),
                ("pe_batch_stride", c_i64), ("pe_head_stride", c_i64), ("pe_row_stride", c_i64),
                ("L", c_i64)]


class AttentionExt(ctypes.Structure):
    _fields_ = [("device_tiles", c_vp), ("workspace", c_vp), ("workspace_bytes", c_i64),
                ("rows_per_rank", ctypes.c_int32), ("head_base", ctypes.c_int32),
                ("out_delta", c_i64 * 8), ("gate_logits", c_vp), ("gate_batch_stride", c_i64),
                ("gate_row_stride", c_i64), ("parts", c_vp), ("parts_bytes", c_i64),
                ("part_splits", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class CopySpan(ctypes.Structure):
    _fields_ = [("src", c_vp), ("dst", c_vp), ("rows", c_i64), ("src_row_stride", c_i64),
                ("dst_row_stride", c_i64)]


class KVSpan(ctypes.Structure):
    _fields_ = [("source", ctypes.c_int32), ("row_start", ctypes.c_int32),
                ("rows", ctypes.c_int32)]


class AdaSource(ctypes.Structure):
    _fields_ = [("table", c_vp), ("ts", c_vp), ("ts_batch_stride", c_i64),
                ("ts_row_stride", c_i64), ("ts_row_div", ctypes.c_int32),
                ("ts_row_offset", ctypes.c_int32)]


class NormOutput(ctypes.Structure):
    _fields_ = [("out", c_vp), ("batch_stride", c_i64), ("row_stride", c_i64),
                ("mod", AdaSource), ("scale_index", ctypes.c_int32),
                ("shift_index", ctypes.c_int32)]


# name -> (restype, argtypes)
_SIGS = {
    "tm_abi_version": (ctypes.c_int, []),
    "tm_last_error": (ctypes.c_char_p, []),
    "tm_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "tm_rope_tables_split": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(c_i64), ctypes.c_int, ctypes.c_int,
                                            ctypes.c_double, ctypes.POINTER(ctypes.c_double),
                                            c_i64, ctypes.c_int, c_i64, c_vp]),
    "tm_norm_rope": (ctypes.c_int, [ctypes.POINTER(NormRopeJob), ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                    c_vp]),
    "tm_copy_rows": (ctypes.c_int, [ctypes.POINTER(CopySpan), ctypes.c_int, c_i64, c_vp]),
    "tm_strided_copy5": (ctypes.c_int, [c_vp, c_vp, ctypes.POINTER(c_i64), ctypes.POINTER(c_i64),
                                        ctypes.POINTER(c_i64), ctypes.c_int, c_vp]),
    "tm_attention_fwd": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                        c_vp, c_vp, c_i64, c_i64, c_i64,
                                        ctypes.POINTER(KVSpan), ctypes.c_int, c_vp, c_i64, c_i64,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, c_vp]),
    "tm_attention_fwd_ws": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                           c_vp, c_vp, c_i64, c_i64, c_i64,
                                           ctypes.POINTER(KVSpan), ctypes.c_int, c_vp, c_i64,
                                           c_i64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_float, c_vp, c_i64, c_vp]),
    "tm_attention_workspace_bytes": (c_i64, [ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, c_i64]),
    "tm_attention_partial_bytes": (c_i64, [ctypes.c_int] * 5),
    "tm_attention_partial_splits": (ctypes.c_int, [ctypes.c_int] * 4 + [c_i64]),
    "tm_attention_plan": (ctypes.c_int, [ctypes.c_int] * 4 + [c_i64, c_i64] +
                          [ctypes.POINTER(ctypes.c_int)] * 3),
    "tm_attention_combine": (ctypes.c_int, [c_vp, ctypes.c_int, c_i64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp, c_i64,
                                            c_i64, c_vp, c_i64, c_i64, c_vp]),
    "tm_attention_tiles": (ctypes.c_int, [ctypes.POINTER(KVSpan), ctypes.c_int, c_i64, c_i64,
                                          c_vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "tm_attention_fwd_dev_tiles": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64,
                                                  c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                                  ctypes.POINTER(KVSpan), ctypes.c_int, c_vp, c_vp,
                                                  c_i64, c_i64, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_int, ctypes.c_int, ctypes.c_float, c_vp,
                                                  c_i64, c_vp]),
    "tm_norm_rope_peer": (ctypes.c_int, [ctypes.POINTER(NormRopeJob), ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                         ctypes.POINTER(c_i64), c_vp]),
    "tm_attention_fwd_ext": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                            c_vp, c_vp, c_i64, c_i64, c_i64,
                                            ctypes.POINTER(KVSpan), ctypes.c_int, c_vp, c_i64,
                                            c_i64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_float,
                                            ctypes.POINTER(AttentionExt), c_vp]),
    "tm_peer_alloc": (ctypes.c_int, [c_i64, ctypes.POINTER(c_vp), c_vp]),
    "tm_peer_free": (ctypes.c_int, [c_vp]),
    "tm_peer_open": (ctypes.c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "tm_peer_close": (ctypes.c_int, [c_vp]),
    "tm_peer_flag_bytes": (c_i64, []),
    "tm_peer_signal": (ctypes.c_int, [ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int, c_vp,
                                      ctypes.c_int, c_vp]),
    "tm_peer_wait": (ctypes.c_int, [c_vp, ctypes.c_int, c_vp, ctypes.c_int, c_vp]),
    "tm_peer_exchange": (ctypes.c_int, [ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int, c_vp,
                                        c_vp, ctypes.c_int, c_vp]),
    "tm_peer_set_wait_limit": (c_i64, [c_i64]),
    "tm_residual_norm": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64,
                                        ctypes.POINTER(AdaSource), ctypes.c_int, c_vp, c_i64,
                                        c_i64, ctypes.POINTER(NormOutput), ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, c_vp]),
    "tm_gelu_tanh": (ctypes.c_int, [c_vp, c_i64, c_vp]),
    "tm_attention_fwd_noalloc": (ctypes.c_int, [c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64,
                                                c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                                ctypes.POINTER(KVSpan), ctypes.c_int, c_vp,
                                                c_i64, c_i64, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_float, c_vp]),
}

EXPORTED = tuple(_SIGS)


def lib_path() -> str:
    """The in-tree build, or the library named by ``TAOMATE_B200_LIB``."""
    return os.environ.get("TAOMATE_B200_LIB") or _build.LIB


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) and bind the library."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = lib_path()
        if build_if_missing and path == _build.LIB and _build.needs_build():
            _build.build()
        if not os.path.exists(path):
            raise RuntimeError(f"taomate_b200 native library not found at {path}; "
                               "run `python -m taomate_b200.build`")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


class TMError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    """Map a tm_status to the exception types the reference raises."""
    if status == TM_OK:
        return
    msg = (load().tm_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if msg else what
    if status in (TM_ERR_INVALID_ARGUMENT, TM_ERR_ALIGNMENT):
        raise ValueError(text)
    if status == TM_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise TMError(text)


LAUNCHES = 0  # kernel launches issued through this binding (for launch accounting)


def launched(n: int = 1) -> None:
    global LAUNCHES
    LAUNCHES += n


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """All tensors on one CUDA device; the kernels have no CPU implementation."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("taomate_b200 kernels run on CUDA tensors only "
                               f"(got a tensor on {t.device})")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def device_error() -> int:
    """Read and clear the device error flag (synchronises the device)."""
    code = ctypes.c_int(0)
    check(load().tm_device_error(ctypes.byref(code)), "tm_device_error")
    return code.value
