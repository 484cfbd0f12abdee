"""ctypes binding of libdbl_gdn2.so, the C ABI declared in include/dbl_gdn2.h.

The structures below mirror the header field by field (``tests/test_abi.py`` compiles the header
with gcc and checks every size and offset).  Loading fails loudly when the library has not been
built: the hot path has no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libdbl_gdn2.so")

DBL_OK = 0
DBL_ERR_INVALID_ARGUMENT = 1
DBL_ERR_UNSUPPORTED = 2
DBL_ERR_CUDA = 3
DBL_ERR_WORKSPACE = 4
DBL_ERR_TIMEOUT = 5
DBL_F32 = 0
DBL_BF16 = 1

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("time", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("dtype", _i32), ("chunk_size", _i32), ("scale", ctypes.c_float),
        ("q", _vp), ("k", _vp), ("v", _vp),
        ("q_stride", _i64 * 4), ("k_stride", _i64 * 4), ("v_stride", _i64 * 4),
        ("alpha", _vp), ("beta", _vp),
        ("alpha_stride", _i64 * 3), ("beta_stride", _i64 * 3),
        ("valid", _vp), ("reset", _vp), ("initial_state", _vp),
        ("out", _vp), ("out_stride", _i64 * 4),
        ("final_state", _vp),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("dtype", _i32), ("scale", ctypes.c_float),
        ("q", _vp), ("k", _vp), ("v", _vp),
        ("q_stride", _i64 * 3), ("k_stride", _i64 * 3), ("v_stride", _i64 * 3),
        ("alpha", _vp), ("beta", _vp),
        ("state", _vp), ("out", _vp), ("out_stride", _i64 * 3),
    ]


class TrainingScanArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("time", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("dtype", _i32), ("chunk_size", _i32),
        ("q", _vp), ("k", _vp), ("v", _vp),
        ("alpha", _vp), ("erase", _vp), ("write", _vp),
        ("valid", _vp), ("reset", _vp), ("initial_state", _vp),
        ("output", _vp), ("final_state", _vp), ("scores", _vp),
    ]


class TrainingScanBackwardArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("time", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("chunk_size", _i32),
        ("q", _vp), ("k", _vp), ("v", _vp),
        ("alpha", _vp), ("erase", _vp), ("write", _vp),
        ("valid", _vp), ("reset", _vp), ("initial_state", _vp),
        ("grad_output", _vp), ("grad_final_state", _vp), ("grad_scores", _vp),
        ("dq", _vp), ("dk", _vp), ("dv", _vp), ("dalpha", _vp), ("derase", _vp), ("dwrite", _vp),
        ("dinitial", _vp),
    ]


class Gdn2PrologueArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("time", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("conv_width", _i64), ("in_dtype", _i32), ("out_dtype", _i32),
        ("proj_q", _vp), ("proj_k", _vp), ("proj_v", _vp),
        ("proj_decay", _vp), ("proj_erase", _vp), ("proj_write", _vp),
        ("conv_q", _vp), ("conv_k", _vp), ("conv_v", _vp),
        ("decay_bias", _vp), ("decay_scale", _vp), ("valid", _vp), ("reset", _vp),
        ("q", _vp), ("k", _vp), ("v", _vp), ("alpha", _vp), ("erase", _vp), ("write", _vp),
    ]


class Gdn2ScanArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("time", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("dtype", _i32),
        ("q", _vp), ("k", _vp), ("v", _vp),
        ("alpha", _vp), ("erase", _vp), ("write", _vp),
        ("doc_start", _vp), ("doc_end", _vp),
        ("output", _vp),
    ]


class RelayMergeArgs(ctypes.Structure):
    _fields_ = [
        ("n_seq", _i64), ("heads", _i64), ("head_dim", _i64), ("prefix_len", _i64), ("own_cap", _i64),
        ("dtype", _i32), ("scale", ctypes.c_float),
        ("q", _vp), ("prefix_k", _vp), ("prefix_v", _vp), ("own_k", _vp), ("own_v", _vp),
        ("own_len", _vp), ("out", _vp), ("row_max", _vp), ("row_sum", _vp),
    ]


class Gdn2ScanBackwardArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("time", _i64), ("heads", _i64), ("key_dim", _i64), ("value_dim", _i64),
        ("dtype", _i32),
        ("q", _vp), ("k", _vp), ("v", _vp), ("alpha", _vp), ("erase", _vp), ("write", _vp),
        ("doc_start", _vp), ("doc_end", _vp), ("grad_output", _vp),
        ("dq", _vp), ("dk", _vp), ("dv", _vp), ("dalpha", _vp), ("derase", _vp), ("dwrite", _vp),
    ]


class RelayAttentionArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("heads", _i64), ("time", _i64), ("head_dim", _i64), ("documents", _i64),
        ("dtype", _i32),
        ("q", _vp), ("k", _vp), ("v", _vp), ("relay_k", _vp), ("relay_v", _vp),
        ("doc_id", _vp), ("doc_start", _vp), ("doc_end", _vp),
        ("o", _vp), ("normalization", _vp),
    ]


# (name, restype, argtypes) for every function in include/dbl_gdn2.h
EXPORTS = [
    ("dbl_status_string", ctypes.c_char_p, [ctypes.c_int]),
    ("dbl_last_error", ctypes.c_char_p, []),
    ("dbl_abi_version", ctypes.c_int, []),
    ("dbl_device_error", ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    ("dbl_gdn2_prefill", ctypes.c_int, [ctypes.POINTER(PrefillArgs), _vp]),
    ("dbl_gdn2_span_transition", ctypes.c_int, [ctypes.POINTER(PrefillArgs), _vp, _vp]),
    ("dbl_gdn2_decode_step", ctypes.c_int, [ctypes.POINTER(DecodeArgs), _vp]),
    ("dbl_gdn_training_scan", ctypes.c_int, [ctypes.POINTER(TrainingScanArgs), _vp]),
    ("dbl_gdn_training_scan_backward_workspace_bytes", ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, _i32]),
    ("dbl_gdn_training_scan_backward", ctypes.c_int,
     [ctypes.POINTER(TrainingScanBackwardArgs), _vp, ctypes.c_size_t, _vp]),
    ("dbl_gdn_training_scan_context_bytes", ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, _i32]),
    ("dbl_gdn_training_scan_save", ctypes.c_int, [ctypes.POINTER(TrainingScanArgs), _vp, ctypes.c_size_t, _vp]),
    ("dbl_gdn_training_scan_backward_saved", ctypes.c_int,
     [ctypes.POINTER(TrainingScanBackwardArgs), _vp, ctypes.c_size_t, _vp, ctypes.c_size_t, _vp]),
    ("dbl_gdn2_scan_backward_workspace_bytes", ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, _i32]),
    ("dbl_gdn2_scan_backward", ctypes.c_int, [ctypes.POINTER(Gdn2ScanBackwardArgs), _vp, ctypes.c_size_t, _vp]),
    ("dbl_gdn2_prologue", ctypes.c_int, [ctypes.POINTER(Gdn2PrologueArgs), _vp]),
    ("dbl_gdn2_scan", ctypes.c_int, [ctypes.POINTER(Gdn2ScanArgs), _vp]),
    ("dbl_relay_merge_workspace_bytes", ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64]),
    ("dbl_relay_merge_decode", ctypes.c_int,
     [ctypes.POINTER(RelayMergeArgs), _vp, ctypes.c_size_t, _vp]),
    ("dbl_relay_merge_decode_noalloc", ctypes.c_int, [ctypes.POINTER(RelayMergeArgs), _vp]),
    ("dbl_relay_merge_call_workspace_bytes", ctypes.c_size_t, [ctypes.POINTER(RelayMergeArgs)]),
    ("dbl_relay_attention_forward", ctypes.c_int, [ctypes.POINTER(RelayAttentionArgs), _vp]),
    ("dbl_gdn2_span_fold", ctypes.c_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp]),
    ("dbl_gdn2_prefill_segmented_workspace_bytes", ctypes.c_size_t, [ctypes.POINTER(PrefillArgs), _i64]),
    ("dbl_gdn2_prefill_segmented", ctypes.c_int, [ctypes.POINTER(PrefillArgs), _i64, _vp, ctypes.c_size_t, _vp]),
    ("dbl_gdn2_prefill_time_sharded_workspace_bytes", ctypes.c_size_t,
     [ctypes.POINTER(PrefillArgs), ctypes.c_int, _i64]),
    ("dbl_gdn2_prefill_time_sharded", ctypes.c_int,
     [ctypes.POINTER(PrefillArgs), ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(_vp), _i64,
      ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_size_t)]),
]

RELAY_NOALLOC_SCRATCH_BYTES = 16 << 20  # DBL_RELAY_NOALLOC_SCRATCH_BYTES

_lib = None
_lock = threading.Lock()


class DblError(RuntimeError):
    """A non-OK status from libdbl_gdn2 (the reference panics on the same conditions)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libdbl_gdn2.so (once).  Raises when it is missing: there is no fallback."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build the CUDA library with "
                        "`python -m delta_block_lm_b200.build` (the GDN-2 path has no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, res, args in EXPORTS:
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(status: int) -> None:
    if status != DBL_OK:
        L = lib()
        msg = L.dbl_last_error().decode()
        kind = L.dbl_status_string(status).decode()
        raise DblError(status, f"{kind}: {msg}")
