"""ctypes binding of librace_b200.so (the C ABI declared in include/race_b200.h).

The library is the only compute path: if it is missing or cannot be loaded
the error propagates; there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librace_b200.so")

RACE_OK = 0
RACE_ERR_TOO_LARGE = 6
RACE_ERR_DEVICE = 7
RACE_FLAG_STRICT_TMA = 1
RACE_FLAG_NORMALIZE_QK = 2
RACE_DEV_TIMEOUT = 1
RACE_DEV_STUCK = 2
RACE_F32 = 0
RACE_BF16 = 1
RACE_NORM_BUCKET = 0
RACE_NORM_GLOBAL = 1

SYMBOLS = (
    "race_version", "race_strerror", "race_last_cuda_error", "race_query",
    "race_forward", "race_backward", "race_forward_reduce", "race_forward_readout",
    "race_backward_q", "race_backward_kv", "race_add_offset", "race_forward_static",
    "race_probs", "race_probs_workspace", "race_probs_backward",
    "race_forward_ex", "race_forward_readout_ex", "race_backward_ex", "race_backward_q_ex",
    "race_last_kernels", "race_status_clear", "race_device_status",
    "race_comm_unique_id", "race_comm_init", "race_comm_destroy", "race_set_comm",
    "race_comm_error",
)


class RaceTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_m", ctypes.c_int64),
                ("stride_b", ctypes.c_int64), ("stride_h", ctypes.c_int64),
                ("stride_t", ctypes.c_int64)]


class RaceDesc(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("causal", ctypes.c_int32),
                ("head_dim", ctypes.c_int32), ("num_bits", ctypes.c_int32),
                ("num_tables", ctypes.c_int32), ("ensembles", ctypes.c_int32),
                ("batch", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("tokens", ctypes.c_int64), ("chunk", ctypes.c_int32),
                ("shared_planes", ctypes.c_int32), ("eps", ctypes.c_float),
                ("normalize", ctypes.c_int32), ("flags", ctypes.c_uint32),
                ("wait_polls", ctypes.c_int32)]


class RaceSizes(ctypes.Structure):
    _fields_ = [("state_bytes", ctypes.c_size_t), ("gstate_bytes", ctypes.c_size_t),
                ("workspace_bytes", ctypes.c_size_t), ("total_bytes", ctypes.c_size_t),
                ("slot_floats", ctypes.c_int32), ("chunk", ctypes.c_int32),
                ("num_chunks", ctypes.c_int64)]


class RaceError(RuntimeError):
    pass


_lib = None
_lock = threading.Lock()

_T = RaceTensor
_P = ctypes.c_void_p
_SIGS = {
    "race_version": ([], ctypes.c_char_p),
    "race_strerror": ([ctypes.c_int], ctypes.c_char_p),
    "race_last_cuda_error": ([], ctypes.c_char_p),
    "race_last_kernels": ([], ctypes.c_char_p),
    "race_status_clear": ([_P, ctypes.c_size_t, _P], ctypes.c_int),
    "race_device_status": ([_P, ctypes.c_size_t, _P, _P], ctypes.c_int),
    "race_comm_unique_id": ([_P], ctypes.c_int),
    "race_comm_init": ([ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _P, ctypes.c_int],
                       ctypes.c_int),
    "race_comm_destroy": ([_P], ctypes.c_int),
    "race_set_comm": ([_P], ctypes.c_int),
    "race_comm_error": ([], ctypes.c_char_p),
    "race_query": ([ctypes.POINTER(RaceDesc), ctypes.POINTER(RaceSizes)], ctypes.c_int),
    "race_forward": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _T, _P, _P, ctypes.c_size_t, _P],
                     ctypes.c_int),
    "race_backward": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _T, _T, _T, _T, _P, _P, _P,
                       ctypes.c_size_t, _P], ctypes.c_int),
    "race_forward_reduce": ([ctypes.POINTER(RaceDesc), _T, _T, _P, _P, _P, _P, _P, ctypes.c_size_t,
                             _P], ctypes.c_int),
    "race_forward_readout": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _T, _P,
                              ctypes.c_size_t, _P], ctypes.c_int),
    "race_backward_q": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _T, _T, _P, _P, _P, _P,
                         ctypes.c_size_t, _P], ctypes.c_int),
    "race_backward_kv": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _P, _T, _T, _T, _P, _P,
                          ctypes.c_size_t, _P], ctypes.c_int),
    "race_add_offset": ([ctypes.POINTER(RaceDesc), _P, _P, ctypes.c_int, _P], ctypes.c_int),
    "race_forward_static": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _T, _P], ctypes.c_int),
    "race_forward_ex": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _T, _P, _P, _P,
                         ctypes.c_size_t, _P], ctypes.c_int),
    "race_forward_readout_ex": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _T, _P, _P,
                                 ctypes.c_size_t, _P], ctypes.c_int),
    "race_backward_ex": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _T, _P, _T, _T, _T,
                          _P, _P, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "race_backward_q_ex": ([ctypes.POINTER(RaceDesc), _T, _T, _T, _P, _P, _P, _T, _P, _T, _P, _P,
                            _P, _P, ctypes.c_size_t, _P], ctypes.c_int),
    "race_probs": ([ctypes.POINTER(RaceDesc), _T, _P, _P, _P, _P], ctypes.c_int),
    "race_probs_workspace": ([ctypes.POINTER(RaceDesc)], ctypes.c_size_t),
    "race_probs_backward": ([ctypes.POINTER(RaceDesc), _T, _P, _P, _P, _T, _P, ctypes.c_int, _P,
                             ctypes.c_size_t, _P], ctypes.c_int),
}


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the library with its prototypes set."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RaceError(
                f"{path} is not built; run `python -m race_attention_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def last_kernels() -> list:
    """Kernels the most recent entry-point call on this thread launched."""
    txt = load().race_last_kernels().decode()
    return [k for k in txt.split(",") if k] if txt else []


def check(rc: int) -> None:
    if rc != RACE_OK:
        lib = load()
        msg = lib.race_strerror(rc).decode()
        if rc in (2, 5):
            extra = lib.race_last_cuda_error().decode()
            if extra:
                msg += ": " + extra
        raise RaceError(f"race_b200 error {rc}: {msg}")
