"""ctypes binding of the C ABI in include/crukx_b200.h (libcrukx_b200.so, built in-tree).

There is no fallback: if the library is missing the import fails with instructions, and every
compute entry point needs a CUDA device.
"""

from __future__ import annotations

import array
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcrukx_b200.so")

CRX_OK, CRX_VALUE_ERROR, CRX_CORRUPT, CRX_CUDA_ERROR, CRX_NO_MEMORY, CRX_BAD_ARGUMENT, CRX_NEED_MORE = range(7)

EXPORTS = [
    "crx_wire_version", "crx_ctx_create", "crx_ctx_destroy", "crx_ctx_launches", "crx_parse_device_launches",
    "crx_ctx_profile",
    "crx_ctx_kernel_times", "crx_encode", "crx_encoded_size", "crx_encoded_copy",
    "crx_encoded_changes", "crx_encoded_checksums", "crx_encoded_free", "crx_parse", "crx_update_n_tensors",
    "crx_update_changes", "crx_update_tensor", "crx_update_group", "crx_update_tensor_table", "crx_update_n_tables", "crx_update_table",
    "crx_update_table_entries", "crx_update_n_blocks", "crx_update_block_bits", "crx_update_payload",
    "crx_update_free", "crx_apply", "crx_huffman_lengths", "crx_checksum", "crx_checksum_noalloc",
    "crx_encode_device", "crx_encoded_copy_device", "crx_parse_head", "crx_parse_device",
    "crx_encode_global", "crx_encoded_part", "crx_encoded_part_copy", "crx_apply_versioned",
    "crx_ctx_hist_cache_hits", "crx_alloc_calls", "crx_size_stats", "crx_apply_to_host",
    "crx_ctx_kernel_gaps", "crx_encoded_parse_device",
]

# collective callbacks of crx_encode_global
SUM_U64_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int64)
ALLGATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int64))

_lib = None
_lock = threading.RLock()   # context() calls load() while holding it


def load():
    """The loaded library (ctypes.CDLL) with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build the CUDA library first "
                              "(python -m crukx_sync_b200.build, or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        P, I32, I64, U64, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_size_t
        CP = ctypes.c_char_p
        sig = {
            "crx_wire_version": ([], ctypes.c_int),
            "crx_ctx_create": ([ctypes.c_int, ctypes.POINTER(P), CP, SZ], ctypes.c_int),
            "crx_ctx_destroy": ([P], None),
            "crx_ctx_launches": ([P], U64),
            "crx_parse_device_launches": ([], U64),
            "crx_ctx_profile": ([P, ctypes.c_int], ctypes.c_int),
            "crx_ctx_kernel_times": ([P, CP, SZ, P, P, I32], I32),
            "crx_encode": ([P, I32, P, P, P, P, P, P, P, P, ctypes.POINTER(P), CP, SZ], ctypes.c_int),
            "crx_encoded_size": ([P], I64),
            "crx_encoded_copy": ([P, P, I64], ctypes.c_int),
            "crx_encoded_changes": ([P], I64),
            "crx_encoded_checksums": ([P, P, P], None),
            "crx_encoded_free": ([P], None),
            "crx_parse": ([P, I64, ctypes.POINTER(P), CP, SZ], ctypes.c_int),
            "crx_update_n_tensors": ([P], I64),
            "crx_update_changes": ([P], I64),
            "crx_update_tensor": ([P, I64, P, P, P, P, P], ctypes.c_int),
            "crx_update_group": ([P, I64, I32, P, P, P], ctypes.c_int),
            "crx_update_tensor_table": ([P, P, P, P, P], ctypes.c_int),
            "crx_update_n_tables": ([P], I32),
            "crx_update_table": ([P, I32, P, P], ctypes.c_int),
            "crx_update_table_entries": ([P, I32, P, P], ctypes.c_int),
            "crx_update_n_blocks": ([P], I64),
            "crx_update_block_bits": ([P, P], ctypes.c_int),
            "crx_update_payload": ([P, P, P], ctypes.c_int),
            "crx_update_free": ([P], None),
            "crx_apply": ([P, P, P, P, P, P, P, CP, SZ], ctypes.c_int),
            "crx_huffman_lengths": ([P, I64, P], ctypes.c_int),
            "crx_checksum": ([P, P, I64, P, P, CP, SZ], ctypes.c_int),
            "crx_checksum_noalloc": ([P, I64, P, P, CP, SZ], ctypes.c_int),
            "crx_encode_device": ([P, I32, P, P, P, P, P, P, P, P, ctypes.POINTER(P), CP, SZ], ctypes.c_int),
            "crx_encoded_copy_device": ([P, P, I64, P], ctypes.c_int),
            "crx_parse_head": ([P, I64, I64, ctypes.c_uint8, ctypes.POINTER(P), ctypes.POINTER(I64), CP, SZ],
                               ctypes.c_int),
            "crx_parse_device": ([P, I64, P, ctypes.POINTER(P), CP, SZ], ctypes.c_int),
            "crx_encode_global": ([P, I32, P, P, P, P, P, P, P, P, I32, I32, SUM_U64_FN, ALLGATHER_FN, P,
                                   ctypes.POINTER(P), CP, SZ], ctypes.c_int),
            "crx_encoded_part": ([P, P, P, P, P, P, P], ctypes.c_int),
            "crx_encoded_part_copy": ([P, P, P, P, P], ctypes.c_int),
            "crx_apply_versioned": ([P, P, P, P, P, P, P, P, P, CP, SZ], ctypes.c_int),
            "crx_ctx_hist_cache_hits": ([P], U64),
            "crx_alloc_calls": ([], U64),
            "crx_size_stats": ([P, I32, P, P, P, P, P, CP, SZ], ctypes.c_int),
            "crx_apply_to_host": ([P, P, P, P, P, P, P, P, CP, SZ], ctypes.c_int),
            "crx_ctx_kernel_gaps": ([P, CP, SZ, P, I32], I32),
            "crx_encoded_parse_device": ([P, P, ctypes.POINTER(P), CP, SZ], ctypes.c_int),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


_ctx = {}


def context(device_index: int):
    """The library context of one CUDA device (created once, kept for the process)."""
    c = _ctx.get(device_index)
    if c is None:
        with _lock:
            c = _ctx.get(device_index)
            if c is None:
                L = load()
                h = ctypes.c_void_p()
                err = ctypes.create_string_buffer(512)
                st = L.crx_ctx_create(device_index, ctypes.byref(h), err, 512)
                if st != CRX_OK:
                    raise RuntimeError(f"crukx_sync_b200: cannot create a context on cuda:{device_index}: "
                                       f"{err.value.decode(errors='replace')}")
                c = _ctx[device_index] = h
    return c


class CBuf:
    """Values for a C array argument, passed as a plain pointer: an array.array is built an order
    of magnitude faster than a ctypes array of hundreds of elements."""

    __slots__ = ("a", "_as_parameter_")

    def __init__(self, typecode: str, values):
        self.a = array.array(typecode, values)
        if not self.a:
            self.a.append(0)
        self._as_parameter_ = ctypes.c_void_p(self.a.buffer_info()[0])

    def __len__(self):
        return len(self.a)


def ptr_array(values):
    return CBuf("Q", values)
