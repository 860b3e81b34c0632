"""ctypes binding of libictc_cuda.so (the C ABI declared in include/ictc_cuda.h).

The library is loaded from this folder only.  There is no fallback: if it is
missing or was built for another ABI version, every CUDA-backend operation
raises.  Tensor arguments are passed as raw device pointers; the stream is
torch's current stream for the tensors' device.
"""
import ctypes
import os
import threading

import torch

LIBRARY_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libictc_cuda.so")
ABI_VERSION = 2

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64

# name -> argtypes (all return int status unless listed in _RESTYPES)
_SIGNATURES = {
    "ictc_version": [],
    "ictc_last_error": [],
    "ictc_tp_plan_create": [_i, _i, _i, _i, _i, _i, _p, _p, _i64, _i, _i, ctypes.POINTER(_p)],
    "ictc_tp_plan_destroy": [_p],
    "ictc_tp_plan_info": [_p, ctypes.POINTER(_i64), _i],
    "ictc_tp_plan_status": [_p, ctypes.POINTER(ctypes.c_int32), _i],
    "ictc_tp_forward": [_p, _p, _p, _p, _p, _p, _i64, _p],
    "ictc_tp_backward": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "ictc_tp_message_forward": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "ictc_tp_message_backward": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p],
    "ictc_harmonics_table_size": [_i],
    "ictc_sc_table_rows": [_i, _i, _i],
    "ictc_sc_fold": [_p, _p, _p, _i, _i, _i, _i, _i64, _i64, _i, _p],
    "ictc_sc_directional": [_p, _p, _p, _p, _p, _i64, _p, _i, _i, _i, _i, _p],
    "ictc_sc_hvp": [_p, _p, _p, _p, _p, _i64, _p, _p, _i, _i, _i, _i, _p],
    "ictc_sc_table_grad": [_p, _p, _p, _p, _p, _i64, _p, _i, _i, _i, _i, _i, _p],
    "ictc_sc_tile_nodes": [],
    "ictc_sc_forward": [_p, _p, _p, _p, _i64, _p, _i, _i, _i, _i, _p],
    "ictc_sc_backward": [_p, _p, _p, _p, _i64, _p, _p, _i, _i, _i, _i, _p],
    "ictc_neighbor_workspace_bytes": [_i64, _p, ctypes.c_float],
    "ictc_neighbor_count": [_p, _i64, _p, ctypes.c_float, _p, _i64, _p, _p],
    "ictc_neighbor_fill": [_p, _i64, _p, ctypes.c_float, _p, _i64, _p, _p, _p, _p, _p],
    "ictc_neighbor_count_receivers": [_p, _i64, _i64, _p, ctypes.c_float, _p, _i64, _p, _p],
    "ictc_neighbor_fill_receivers": [_p, _i64, _i64, _p, ctypes.c_float, _p, _i64, _p, _p, _p, _p, _p],
    "ictc_neighbor_noalloc_scratch_bytes": [],
    "ictc_neighbor_list_noalloc": [_p, _i64, _p, ctypes.c_float, _p, _p, _p, _p, _i64, _p],
    "ictc_direction_harmonics": [_p, _p, _p, _p, _p, _p, _i64, _i, _i, _p],
    "ictc_edge_geometry": [_p, _i64, ctypes.c_float, _i, _i, _i, _p, _p, _p, _p],
    "ictc_edge_geometry_backward": [_p, _p, _p, _i64, ctypes.c_float, _i, _i, _i, _p, _p],
    "ictc_channel_mix_tile_nodes": [],
    "ictc_channel_mix": [_p, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i, _i, _i, ctypes.c_float, _i,
                         _p],
    "ictc_radial_image_bytes": [_i, _i, _i],
    "ictc_wait_selftest": [_p, _i64, _i, _p],
    "ictc_radial_pack": [_p, _p, _p, _p, _i, _i, _i, _p, _i64],
    "ictc_radial_forward": [_p, _p, _p, _i64, _i, _i, _i, _p, _p],
    "ictc_radial_backward": [_p, _p, _p, _p, _p, _i64, _i, _i, _i, _p, _p],
}
_RESTYPES = {"ictc_last_error": ctypes.c_char_p, "ictc_sc_table_rows": _i64,
             "ictc_neighbor_workspace_bytes": _i64, "ictc_neighbor_noalloc_scratch_bytes": _i64,
             "ictc_radial_image_bytes": _i64}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    pass


def library():
    """Load (once) and return the ctypes handle of libictc_cuda.so."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIBRARY_PATH):
            raise NativeError(f"libictc_cuda.so not found at {LIBRARY_PATH}; run __graft_entry__.build()")
        lib = ctypes.CDLL(LIBRARY_PATH)
        for name, args in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, _i)
        version = lib.ictc_version()
        if version != ABI_VERSION:
            raise NativeError(f"libictc_cuda.so ABI {version} != expected {ABI_VERSION}; rebuild it")
        _lib = lib
        return lib


def exported_symbols():
    return tuple(_SIGNATURES)


def check(status, what):
    if status != 0:
        message = library().ictc_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed (status {status}): {message}")


def ptr(tensor):
    """Device pointer of a contiguous tensor, or NULL for None."""
    if tensor is None:
        return None
    return ctypes.c_void_p(tensor.data_ptr())


def stream_of(tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(tensor.device).cuda_stream)


def call(name, *args):
    check(getattr(library(), name)(*args), name)
