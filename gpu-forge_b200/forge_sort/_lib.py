"""ctypes binding of libforgesort.so (declarations in include/forgesort.h).

The library is built in-tree by gpu-forge_b200/build.py.  There is no CPU or
torch fallback: if the shared library is missing or fails to load, importing
forge_sort raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libforgesort.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

# fs_dtype (include/forgesort.h)
U32, I32, F32, U64, I64, F64 = range(6)

IPC_HANDLE_BYTES = 64  # FS_IPC_HANDLE_BYTES

# fs_status
OK = 0
E_DEVICE_NOT_FOUND = 1
E_KERNEL_IMAGE = 2
E_GPU_EXECUTION = 3
E_LENGTH_MISMATCH = 4
E_TIMEOUT = 5
E_NCCL = 6
E_OOM = 7
E_INVALID = 8

# Every symbol include/forgesort.h declares, with (restype, argtypes).
_vp, _u64, _i32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int
_pp = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = {
    "fs_create": (_i32, [_i32, _vp, _pp]),
    "fs_destroy": (_i32, [_vp]),
    "fs_last_error": (ctypes.c_char_p, [_vp]),
    "fs_set_stream": (_i32, [_vp, _vp]),
    "fs_synchronize": (_i32, [_vp]),
    "fs_alloc": (_i32, [_vp, ctypes.c_size_t, _i32, _pp]),
    "fs_free": (_i32, [_vp, _vp]),
    "fs_sort_keys": (_i32, [_vp, _i32, _vp, _u64, _i32]),
    "fs_sort_pairs": (_i32, [_vp, _i32, _vp, _vp, _u64, _i32]),
    "fs_argsort": (_i32, [_vp, _i32, _vp, _vp, _u64, _i32]),
    "fs_host_sort_keys": (_i32, [_vp, _i32, _vp, _u64]),
    "fs_host_sort_pairs": (_i32, [_vp, _i32, _vp, _u64, _vp, _u64]),
    "fs_host_argsort": (_i32, [_vp, _i32, _vp, _vp, _u64]),
    "fs_sort_keys_copy": (_i32, [_vp, _i32, _vp, _vp, _u64, _i32]),
    "fs_host_sort_keys_copy": (_i32, [_vp, _i32, _vp, _vp, _u64]),
    "fs_set_kernel_timing": (_i32, [_vp, _i32]),
    "fs_last_kernel_times": (_i32, [_vp, ctypes.POINTER(ctypes.c_float), _i32]),
    "fs_partition": (_i32, [_vp, _i32, _vp, _u64, _u64, _vp, _vp, _i32, _vp, _vp, _i32]),
    "fs_host_sort_keys_copy_async": (_i32, [_vp, _i32, _vp, _vp, _u64]),
    "fs_gather": (_i32, [_vp, _i32, _vp, _u64, _vp, _vp, _u64, _i32]),
    "fs_sort_pairs_copy": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _u64, _i32]),
    "fs_partition_dispatch_pairs": (_i32, [_vp, _i32, _vp, _vp, _u64, _u64, _vp, _vp, _i32, _vp, _vp, _i32]),
    "fs_stream_create": (_i32, [_i32, _vp]),
    "fs_stream_synchronize": (_i32, [_vp]),
    "fs_stream_destroy": (_i32, [_vp]),
    "fs_mg_create": (_i32, [_vp, _i32, _pp]),
    "fs_mg_destroy": (_i32, [_vp]),
    "fs_mg_last_error": (ctypes.c_char_p, [_vp]),
    "fs_mg_sort_keys": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp]),
    "fs_mg_sort_pairs": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "fs_partition_count": (_i32, [_vp, _i32, _vp, _u64, _u64, _vp, _vp, _i32, _vp]),
    "fs_partition_dispatch": (_i32, [_vp, _i32, _vp, _u64, _u64, _vp, _vp, _i32, _vp, _i32]),
    "fs_partition_count_async": (_i32, [_vp, _i32, _vp, _u64, _u64, _vp, _vp, _i32, _vp]),
    "fs_partition_dispatch_matrix": (_i32, [_vp, _i32, _vp, _vp, _i32, _u64, _u64, _vp, _vp, _i32, _vp, _i32, _vp,
                                            _vp, _i32]),
    "fs_ipc_export": (_i32, [_vp, _vp, _vp]),
    "fs_ipc_open": (_i32, [_vp, _vp, _pp]),
    "fs_ipc_close": (_i32, [_vp, _vp]),
    "fs_sort_keys_noalloc": (_i32, [_i32, _vp, _u64, _vp]),
    "fs_buffer_create": (_i32, [_vp, _u64, _pp]),
    "fs_buffer_destroy": (_i32, [_vp]),
    "fs_buffer_host": (_vp, [_vp]),
    "fs_buffer_device": (_vp, [_vp]),
    "fs_buffer_bytes": (_u64, [_vp]),
    "fs_buffer_host_read": (_i32, [_vp]),
    "fs_buffer_host_write": (_i32, [_vp]),
    "fs_buffer_device_use": (_i32, [_vp, _u64]),
    "fs_sort_buffer": (_i32, [_vp, _i32, _vp, _u64, _i32]),
    "fs_sort_pairs_buffer": (_i32, [_vp, _i32, _vp, _vp, _u64, _i32]),
    "fs_scratch_bytes": (_u64, [_vp]),
    "fs_last_launch_count": (_i32, [_vp]),
    "fs_abi_version": (_i32, []),
}
# include/forgesort_bench.h
BENCH_SIGNATURES = {
    "fs_generate": (_i32, [_i32, _u64, _u64, _u64, _vp, _vp]),
    "fs_set_wait_timeout_ms": (_i32, [_vp, _u64]),
    "fs_set_single_launch_max": (_i32, [_vp, _u64]),
    "fs_test_inject": (_i32, [_vp, _i32, _i32]),
}
TEST_WITHHOLD_COPY, TEST_FAIL_ALLOC, TEST_SKIP_ARRIVAL = 1, 2, 3
GEN_U32, GEN_U64, GEN_SKEW_U32 = 0, 1, 2

_lib = None


def load(path: str = LIB_PATH):
    """Load the C-ABI library (cached).  Raises OSError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise OSError(
            f"{path} not found: build it with `python gpu-forge_b200/build.py` "
            "(forge_sort has no fallback implementation)")
    L = ctypes.CDLL(path)
    for name, (res, args) in {**SIGNATURES, **BENCH_SIGNATURES}.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L
