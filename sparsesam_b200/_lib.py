"""ctypes binding of libsparsesam_b200.so (the C ABI declared in include/sparsesam.h).

Loading never falls back to anything: if the shared object is missing the
caller gets a RuntimeError telling it to build the library first.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_f64 = ctypes.c_double
c_size = ctypes.c_size_t
c_ptr = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/sparsesam.h.
SIGNATURES: dict[str, tuple] = {
    "ssam_version": (c_int, []),
    "ssam_status_string": (ctypes.c_char_p, [c_int]),
    "ssam_device_error": (c_int, [c_int]),
    "ssam_zorder": (c_int, [c_int, c_int, c_ptr, c_ptr, c_ptr]),
    "ssam_stripe_sort_perm": (c_int, [c_ptr, c_i64, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                      c_ptr, c_ptr, c_ptr, c_ptr, c_ptr]),
    "ssam_a_shape_n_init": (c_int, [c_int, c_int, c_f64, c_int]),
    "ssam_a_shape_mask": (c_int, [c_int, c_int, c_int, c_int, c_int, c_ptr]),
    "ssam_check_wait_timeout": (c_int, [c_ptr]),
    "ssam_hilbert_order": (c_int, [c_int, c_int, c_ptr, c_ptr, c_ptr]),
    "ssam_sparse_attn_workspace_size": (c_size, [c_int, c_int, c_int, c_int]),
    "ssam_sparse_attn_fwd": (c_int, [c_ptr, c_i64, c_int, c_int, c_int, c_int, c_ptr, c_ptr, c_ptr,
                                     c_int, c_int, c_int, c_f32, c_ptr, c_i64, c_ptr, c_int, c_int, c_ptr, c_ptr,
                                     c_size, c_ptr]),
    "ssam_keep_select": (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_ptr, c_ptr, c_ptr]),
    "ssam_zstride_keep_n": (c_int, [c_int, c_f64]),
    "ssam_zstride_keep": (c_int, [c_int, c_int, c_int, c_int, c_ptr, c_ptr, c_ptr]),
    "ssam_layernorm_gather": (c_int, [c_ptr, c_i64, c_ptr, c_int, c_int, c_ptr, c_ptr, c_f32, c_ptr, c_i64,
                                      c_ptr]),
    "ssam_window_rows": (c_int, [c_int, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_gemm_bf16": (c_int, [c_ptr, c_i64, c_ptr, c_i64, c_int, c_int, c_int, c_ptr, c_int, c_ptr, c_i64,
                               c_ptr, c_ptr]),
    "ssam_rc_mlp_workspace_size": (c_size, [c_int, c_int, c_int]),
    "ssam_rc_mlp_fwd": (c_int, [c_ptr, c_i64, c_ptr, c_int, c_int, c_int, c_ptr, c_ptr, c_f32, c_ptr, c_ptr,
                                c_ptr, c_ptr, c_ptr, c_size, c_ptr]),
    "ssam_patch_im2col": (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_broadcast_rows": (c_int, [c_ptr, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_im2col3x3_nhwc": (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_nhwc_to_nchw": (c_int, [c_ptr, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_conv3x3_nhwc": (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_ptr, c_int, c_ptr, c_ptr, c_ptr]),
    "ssam_gemm_bf16_addend": (c_int, [c_ptr, c_i64, c_ptr, c_i64, c_int, c_int, c_int, c_ptr, c_ptr, c_int, c_ptr,
                                      c_ptr]),
    "ssam_layernorm_rows": (c_int, [c_ptr, c_int, c_int, c_ptr, c_ptr, c_f32, c_ptr, c_int, c_ptr]),
    "ssam_layernorm_nchw": (c_int, [c_ptr, c_int, c_int, c_int, c_ptr, c_ptr, c_f32, c_ptr, c_ptr]),
    "ssam_layernorm_gelu_half": (c_int, [c_ptr, c_i64, c_int, c_ptr, c_ptr, c_f32, c_int, c_int, c_ptr, c_ptr]),
    "ssam_layernorm_rows_copy": (c_int, [c_ptr, c_int, c_int, c_ptr, c_ptr, c_f32, c_ptr, c_ptr, c_ptr]),
    "ssam_split_bf16x2": (c_int, [c_ptr, c_int, c_int, c_ptr, c_ptr]),
    "ssam_split_bf16x3": (c_int, [c_ptr, c_int, c_int, c_ptr, c_ptr]),
    "ssam_window_of_raster": (c_int, [c_int, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_fill_pad_rows": (c_int, [c_ptr, c_i64, c_ptr, c_int, c_int, c_ptr, c_ptr]),
    "ssam_patch_im2col_split3": (c_int, [c_ptr, c_int, c_int, c_int, c_int, c_int, c_ptr, c_ptr]),
    "ssam_rc_mlp_fwd_noalloc": (c_int, [c_ptr, c_i64, c_ptr, c_int, c_int, c_int, c_ptr, c_ptr, c_f32, c_ptr, c_ptr,
                                        c_ptr, c_ptr, c_ptr]),
}

SSAM_OK = 0
SSAM_ERR_INVALID = 1
SSAM_ERR_ALIGN = 2
SSAM_ERR_UNSUPPORTED = 3
SSAM_ERR_CUDA = 4
SSAM_ERR_TIMEOUT = 5

SSAM_EPI_BF16 = 0
SSAM_EPI_GELU_BF16 = 1
SSAM_EPI_ADD_F32 = 2
SSAM_EPI_F32 = 3

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

# Kernels each entry point enqueues (for launch accounting); host-only calls are 0.
KERNELS_PER_CALL = {
    "ssam_zorder": 1, "ssam_stripe_sort_perm": 1, "ssam_sparse_attn_fwd": 1, "ssam_keep_select": 1,
    "ssam_check_wait_timeout": 1, "ssam_hilbert_order": 1,
    "ssam_layernorm_gather": 1, "ssam_window_rows": 1, "ssam_gemm_bf16": 1, "ssam_rc_mlp_fwd": 3,
    "ssam_patch_im2col": 1, "ssam_broadcast_rows": 1, "ssam_im2col3x3_nhwc": 1, "ssam_nhwc_to_nchw": 1,
    "ssam_conv3x3_nhwc": 1, "ssam_gemm_bf16_addend": 1,
    "ssam_layernorm_rows": 1, "ssam_layernorm_nchw": 1, "ssam_layernorm_rows_copy": 1, "ssam_split_bf16x2": 1,
    "ssam_layernorm_gelu_half": 1,
    "ssam_rc_mlp_fwd_noalloc": 3,
    "ssam_split_bf16x3": 1, "ssam_patch_im2col_split3": 1, "ssam_window_of_raster": 1, "ssam_fill_pad_rows": 1,
    "ssam_zstride_keep": 1,
}
launch_count = 0  # kernels enqueued through call() since import (read by bench.py)


class SparseSAMError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status} ({message})")
        self.fn = fn
        self.status = status


def lib_path() -> str:
    return _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Load the shared object once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python -m sparsesam_b200.build` "
                    "(or __graft_entry__.build()); there is no fallback implementation")
            handle = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name, None)
                if fn is None:
                    continue  # reported by missing_symbols(); calling it raises AttributeError
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def missing_symbols() -> list[str]:
    """Entry points declared in include/sparsesam.h that the loaded library lacks."""
    handle = load()
    return [n for n in SIGNATURES if getattr(handle, n, None) is None]


def call(name: str, *args, launches: int | None = None) -> int:
    """Invoke an entry point and raise SparseSAMError on a non-zero status.

    ``launches`` overrides the entry's kernel count for calls whose count depends
    on the arguments (the global-grid attention adds its bias pre-pass)."""
    global launch_count
    fn = getattr(load(), name)
    st = fn(*args)
    launch_count += KERNELS_PER_CALL.get(name, 0) if launches is None else launches
    if st != SSAM_OK:
        msg = load().ssam_status_string(st).decode()
        raise SparseSAMError(name, st, msg)
    return st
