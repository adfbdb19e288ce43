"""ctypes binding of ``libgdn_b200.so`` (the C ABI declared in ``include/gdn_b200.h``).

The library is loaded once, from this package's ``_lib`` folder. There is no fallback:
if the library is missing or cannot be loaded, every operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libgdn_b200.so")

(OK, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_NULL, ERR_LAUNCH, ERR_DEVICE_TIMEOUT, ERR_UNSUPPORTED, ERR_SCRATCH,
 ERR_WORKSPACE) = range(10)
F32, BF16 = 0, 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t


class GateInputs(ctypes.Structure):
    """``gdn_gate_inputs``: the raw gate projections for the ``*_gates`` entry points."""

    _fields_ = [("b", _p), ("b_row_stride", _i64), ("a", _p), ("a_row_stride", _i64), ("dt_bias", _p),
                ("dt_bias_dtype", _i32), ("log_decay_rate", _p), ("valid", _p)]


# name -> argument types, in declaration order of include/gdn_b200.h
SIGNATURES: dict[str, list] = {
    "gdn_status_string": [_i32],
    "gdn_abi_version": [],
    "gdn_device_error": [_p, _i32],
    "gdn_probe_bounded_wait": [_i64, _p],
    "gdn_recurrent": [_p, _p, _p, _i32, _p, _p, _i32, _p, _p, _p, _p, _p, _p,
                      _i64, _i64, _i64, _i64, _i64, _i64,
                      _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p],
    "gdn_recurrent_gates": [_p, _p, _p, _i32, ctypes.POINTER(GateInputs), _p, _p, _p, _p, _p, _p,
                            _i64, _i64, _i64, _i64, _i64, _i64,
                            _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p],
    "gdn_recurrent_deltas": [_p, _p, _p, _i32, _p, _p, _i32, _p, _p, _p,
                             _i64, _i64, _i64, _i64, _i64, _i64,
                             _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p],
    "gdn_recurrent_deltas_gated_norm": [_p, _p, _p, _p, _p, _i32, _p, _p, _p, _f32, _p, _p,
                                        _i64, _i64, _i64, _i64, _i64, _i64,
                                        _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p],
    "gdn_delta_commit": [_p, _p, _i32, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_delta_commit_layers": [_p, _p, _i32, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                _i64, _p],
    "gdn_verify_layer_deltas": [_p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _p, _p, _p, _p, _p,
                                _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32, _p],
    "gdn_chunk_prefill": [_p, _p, _p, _p, _p, _i32, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                          _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _sz, _p],
    "gdn_chunk_prefill_gates": [_p, _p, _p, ctypes.POINTER(GateInputs), _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _sz, _p],
    "gdn_chunk_prefill_gated_norm": [_p, _p, _p, _p, _p, _i32, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                     _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _p, _f32, _p,
                                     _p, _sz, _p],
    "gdn_chunk_prefill_workspace_size": [_i64, _i64, _i64, _i32],
    "gdn_snapshot_commit": [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_conv1d_silu": [_p, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p],
    "gdn_conv1d_silu_step": [_p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p],
    "gdn_conv_step": [_p, _p, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_conv_state_commit": [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_gated_rmsnorm": [_p, _p, _p, _p, _i64, _i64, _f32, _p],
    "gdn_delta_gates": [_p, _i64, _p, _i64, _p, _i32, _p, _p, _p, _p, _i64, _i64, _p],
    "gdn_decode_attention": [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _p,
                             _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _sz, _p],
    "gdn_decode_attention_workspace_size": [_i64, _i64, _i64, _i64],
    "gdn_rotary": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_rotate_into_cache": [_p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _i64, _i64,
                              _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_in_proj_conv": [_p, _i64, _p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_in_proj_fp8_workspace_size": [_i64, _i64],
    "gdn_in_proj_fp8_prefill_workspace_size": [_i64, _i64, _i64, _i64],
    "gdn_in_proj_conv_fp8": [_p, _i64, _p, _i64, _p, _p, _p, _p, _i64, _p, _p, _sz, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "gdn_decode_layer": [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                         _f32, _f32, _p],
    "gdn_decode_layer_noalloc": [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _f32, _f32, _p],
}

RESTYPES = {"gdn_status_string": ctypes.c_char_p, "gdn_chunk_prefill_workspace_size": ctypes.c_size_t,
            "gdn_decode_attention_workspace_size": ctypes.c_size_t, "gdn_in_proj_fp8_workspace_size": ctypes.c_size_t,
            "gdn_in_proj_fp8_prefill_workspace_size": ctypes.c_size_t}

_lock = threading.Lock()
_lib = None


class LibraryError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the library (once). Raises if it is missing: there is no other implementation."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise LibraryError(f"{LIB_PATH} is missing; build it with `python -m jeeves_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = lib
        return lib


def status_text(status: int) -> str:
    return load().gdn_status_string(status).decode()


def check(status: int, what: str) -> None:
    """Map a C status to the reference's error convention: ValueError for bad input, RuntimeError otherwise."""
    if status == OK:
        return
    text = f"{what}: {status_text(status)} (status {status})"
    if status in (ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_NULL, ERR_UNSUPPORTED, ERR_SCRATCH, ERR_WORKSPACE):
        raise ValueError(text)
    raise RuntimeError(text)
