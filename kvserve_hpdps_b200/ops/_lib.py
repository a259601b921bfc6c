"""ctypes binding of ``libkvs_b200.so`` (built in-tree by ``ops/build.py``).

The structures below mirror ``csrc/kvs_types.h`` field for field; their
sizes are checked against the library at load time.

Loading policy: the library is loaded from this directory only.  When it is
missing, CPU-only callers get a clear error on first use; on a machine with a
CUDA device the import of any device op raises instead of falling back to a
slower path (a fallback would hide a broken build).
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import (POINTER, c_double, c_float, c_int, c_longlong, c_uint8, c_uint32,
                    c_uint64, c_ulonglong, c_void_p)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkvs_b200.so")

MAX_HEADS = 16


class PagedKV(ctypes.Structure):
    _fields_ = [("base", c_void_p), ("block_stride", c_longlong), ("kv_stride", c_longlong),
                ("slot_stride", c_longlong), ("head_stride", c_longlong),
                ("num_blocks", c_int), ("block_size", c_int), ("hnd", c_int), ("pad_", c_int)]


class ReqTable(ctypes.Structure):
    _fields_ = [("block_table", c_void_p), ("bt_off", c_void_p), ("n_tokens", c_void_p),
                ("n_rows", c_void_p), ("tile_prefix", c_void_p), ("slot", c_void_p),
                ("code_off", c_void_p), ("meta_off", c_void_p), ("row_off", c_void_p),
                ("num_req", c_int)]


class LayerParams(ctypes.Structure):
    _fields_ = [("H", c_int), ("n_groups", c_int),
                ("key_levels", c_float * MAX_HEADS), ("value_levels", c_float * MAX_HEADS),
                ("key_bits", c_int * MAX_HEADS), ("value_bits", c_int * MAX_HEADS),
                ("group_of_head", c_int * MAX_HEADS),
                ("seg_prefix", c_int * (2 * MAX_HEADS + 1)),
                ("sign_bits", (c_uint32 * 4) * MAX_HEADS),
                ("clamp_top", c_int), ("transform", c_int), ("out_scale", c_float)]


class LayerLaunch(ctypes.Structure):
    _fields_ = [("kvs", c_void_p), ("maps", c_void_p), ("lps", c_void_p), ("rt", ReqTable),
                ("bmat", c_void_p), ("bmat_stride", c_longlong), ("codes", c_void_p),
                ("meta", c_void_p), ("kstat", c_void_p), ("vstat", c_void_p), ("err", c_void_p),
                ("total_tiles", c_int), ("num_heads", c_int), ("engine", c_int),
                ("stream", c_void_p), ("trace", c_void_p), ("trace_jobs", c_int),
                ("vparam", c_void_p), ("ck", c_void_p), ("ck_off", c_longlong)]


class RansMsg(ctypes.Structure):
    """Where an encoded rANS stream goes inside a transfer message."""
    _fields_ = [("prefix", c_uint32 * 4), ("has_prefix", c_int), ("pad_", c_int),
                ("msg_off", c_longlong), ("ck", c_void_p), ("trailer", c_void_p),
                ("counter", c_void_p), ("flag", c_void_p), ("flag_value", c_uint32),
                ("pad2_", c_int)]


class RawItem(ctypes.Structure):
    _fields_ = [("bt_off", c_longlong), ("flat_off", c_longlong), ("slot", c_int),
                ("nblocks", c_int)]


class RawLaunch(ctypes.Structure):
    _fields_ = [("kvs", c_void_p), ("items", c_void_p), ("unit_prefix", c_void_p),
                ("block_table", c_void_p), ("flat", c_void_p), ("err", c_void_p), ("ck", c_void_p),
                ("trailer", c_void_p), ("counter", c_void_p), ("flag", c_void_p),
                ("n_units", c_longlong), ("n_items", c_int), ("dir", c_int),
                ("block_bytes", c_int), ("elem_bytes", c_int), ("flag_value", c_uint32),
                ("pad_", c_int)]


_lock = threading.Lock()
_lib = None


def _declare(lib: ctypes.CDLL) -> None:
    P = c_void_p
    sig = {
        "kvs_layer_launch_size": ([], c_int),
        "kvs_init_key_stats": ([P, c_longlong, P], c_int),
        "kvs_layer_params_size": ([], c_int),
        "kvs_paged_kv_size": ([], c_int),
        "kvs_make_plane_maps": ([POINTER(PagedKV), c_int, P], c_int),
        "kvs_stats": ([POINTER(LayerLaunch)], c_int),
        "kvs_quant": ([POINTER(LayerLaunch)], c_int),
        "kvs_value_params": ([POINTER(LayerLaunch), c_int], c_int),
        "kvs_dequant_inverse": ([POINTER(LayerLaunch)], c_int),
        "kvs_rans_max_bytes": ([c_uint64, c_uint32], c_uint64),
        "kvs_rans_staging_bytes": ([c_uint64, c_uint32], c_uint64),
        "kvs_rans_encode": ([P, c_uint64, c_uint32, P, P, P, P, P, P], c_int),
        "kvs_rans_msg_size": ([], c_int),
        "kvs_rans_sizes_words": ([c_uint64, c_uint32], c_uint64),
        "kvs_rans_decode": ([P, c_uint64, P, c_uint64, c_uint32, P, P], c_int),
        "kvs_lc_max_bytes": ([c_uint64], c_uint64),
        "kvs_lc_staging_bytes": ([c_uint64], c_uint64),
        "kvs_lc_encode": ([P, c_uint64, P, P, P, P, P], c_int),
        "kvs_lc_decode": ([P, c_uint64, P, c_uint64, P, P], c_int),
        "kvs_cpu_rans_max_bytes": ([c_uint64, c_uint32], c_uint64),
        "kvs_cpu_rans_encode": ([P, c_uint64, c_uint32, P, c_uint64], c_uint64),
        "kvs_cpu_rans_decode": ([P, c_uint64, P, c_uint64], c_int),
        "kvs_cpu_lc_max_bytes": ([c_uint64], c_uint64),
        "kvs_cpu_lc_encode": ([P, c_uint64, P, c_uint64], c_uint64),
        "kvs_cpu_lc_decode": ([P, c_uint64, P, c_uint64], c_int),
        "kvs_cpu_bitpack": ([P, c_uint64, c_int, P], None),
        "kvs_cpu_bitunpack": ([P, c_uint64, c_int, P], None),
        "kvs_checksum": ([P, c_int, P, c_int, P], c_int),
        "kvs_checksum_verify": ([P, c_int, P, P, P, c_int, P], c_int),
        "kvs_block_copy": ([POINTER(PagedKV), P, c_int, c_longlong, P, c_int, P, P, c_uint32, P,
                            P], c_int),
        "kvs_raw_launch_size": ([], c_int),
        "kvs_raw_item_size": ([], c_int),
        "kvs_paged_raw": ([POINTER(RawLaunch), c_int, P], c_int),
        "kvs_copy16": ([P, P, c_longlong, P, P, c_uint32, c_int, P], c_int),
        "kvs_copy_segments": ([P, c_int, c_int, P, P, c_uint32, P, P, P], c_int),
        "kvs_zero2": ([P, P], c_int),
        "kvs_wait_flag": ([P, c_uint32, c_uint64, P, P, P], c_int),
        "kvs_set_flag": ([P, c_uint32, P], c_int),
        "kvs_probe_push": ([P, P, c_longlong, P, c_int, P], c_int),
        "kvs_kv_error": ([P, P, c_longlong, P, P, P], c_int),
        "kvs_logit_agreement": ([P, P, c_int, c_int, P, P], c_int),
        "kvs_device_count": ([], c_int),
        "kvs_malloc": ([c_int, c_uint64, POINTER(c_void_p)], c_int),
        "kvs_free": ([c_int, P], c_int),
        "kvs_memset": ([P, c_int, c_uint64, P], c_int),
        "kvs_ipc_get_handle": ([c_int, P, POINTER(c_uint8)], c_int),
        "kvs_ipc_open_handle": ([c_int, POINTER(c_uint8), POINTER(c_void_p)], c_int),
        "kvs_ipc_close_handle": ([c_int, P], c_int),
        "kvs_can_access_peer": ([c_int, c_int], c_int),
        "kvs_enable_peer_access": ([c_int, c_int], c_int),
        "kvs_last_error_string": ([], ctypes.c_char_p),
        "kvs_stream_sync": ([P], c_int),
        "kvs_library_version": ([], c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res


def lib() -> ctypes.CDLL:
    """The loaded native library (raises with a build hint when missing)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"native library {LIB_PATH} is missing; build it with "
                    "`python -m kvserve_hpdps_b200.ops.build`")
            handle = ctypes.CDLL(LIB_PATH)
            _declare(handle)
            for name, cls in (("kvs_layer_launch_size", LayerLaunch),
                              ("kvs_layer_params_size", LayerParams),
                              ("kvs_paged_kv_size", PagedKV),
                              ("kvs_raw_launch_size", RawLaunch),
                              ("kvs_rans_msg_size", RansMsg),
                              ("kvs_raw_item_size", RawItem)):
                got = getattr(handle, name)()
                if got != ctypes.sizeof(cls):
                    raise RuntimeError(f"{cls.__name__} size mismatch: C {got} vs Python "
                                       f"{ctypes.sizeof(cls)}")
            _lib = handle
    return _lib


def available() -> bool:
    try:
        lib()
        return True
    except (RuntimeError, OSError):
        return False


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with code {rc}: "
                           f"{lib().kvs_last_error_string().decode(errors='replace')}")


__all__ = ["lib", "available", "check", "PagedKV", "ReqTable", "LayerParams", "LayerLaunch",
           "RansMsg",
           "MAX_HEADS", "c_double", "c_ulonglong"]
