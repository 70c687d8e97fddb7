"""SortError -- the four variants and Display strings of forge-sort's error
enum (metal-forge-compute/forge-sort/src/lib.rs:94-104; strings pinned by the
reference test at src/lib.rs:3034-3049).  DeviceNotFound keeps the
reference's wording for source compatibility; on this build it means that no
CUDA device was found."""
from __future__ import annotations

from . import _lib


class SortError(Exception):
    """Base class; str(e) is the reference's Display string."""


class DeviceNotFound(SortError):
    def __init__(self):
        super().__init__("no Metal GPU device found")


class ShaderCompilation(SortError):
    """Kernel image could not be loaded for this GPU."""

    def __init__(self, msg: str):
        self.msg = msg
        super().__init__(f"shader compilation failed: {msg}")


class GpuExecution(SortError):
    def __init__(self, msg: str):
        self.msg = msg
        super().__init__(f"GPU execution failed: {msg}")


class LengthMismatch(SortError):
    def __init__(self, keys: int, values: int):
        self.keys = keys
        self.values = values
        super().__init__(f"length mismatch: keys={keys}, values={values}")


def from_status(rc: int, text: str, *, keys: int = 0, values: int = 0) -> SortError:
    """Map an fs_status (include/forgesort.h) to the SortError variant."""
    if rc == _lib.E_DEVICE_NOT_FOUND:
        return DeviceNotFound()
    if rc == _lib.E_KERNEL_IMAGE:
        return ShaderCompilation(text)
    if rc == _lib.E_LENGTH_MISMATCH:
        return LengthMismatch(keys, values)
    return GpuExecution(text)
