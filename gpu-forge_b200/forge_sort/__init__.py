"""forge_sort -- B200 (sm_100a) radix sort behind forge-sort's GpuSorter API.

The compute path is libforgesort.so (hand-written CUDA, include/forgesort.h);
this package is the host-side mirror of the reference's Rust API
(kavanaghpatrick/gpu-forge metal-forge-compute/forge-sort/src/lib.rs).
"""
from ._lib import LIB_PATH, load as load_library  # noqa: F401
from .errors import (DeviceNotFound, GpuExecution, LengthMismatch,  # noqa: F401
                     ShaderCompilation, SortError)
from .multigpu import MultiGpuSorter  # noqa: F401
from .sorter import SORT_KEY, GpuSorter, SortBuffer, dtype_name  # noqa: F401

__all__ = [
    "GpuSorter", "SortBuffer", "MultiGpuSorter", "SortError", "DeviceNotFound", "ShaderCompilation",
    "GpuExecution", "LengthMismatch", "SORT_KEY", "dtype_name",
]
