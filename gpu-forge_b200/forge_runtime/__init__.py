"""forge_runtime -- the sort side of gpu-forge's forge-runtime crate
(metal-forge-compute/forge-runtime/src): a shared device + stream
(ForgeContext, context.rs:16-55), a permutation apply (GpuGather,
gather.rs:27-140) and a stream-ordered pipeline of sort and gather stages
(Pipeline, pipeline.rs:41-140).

The reference encodes every stage into one Metal command buffer and waits
once in execute().  Here the command buffer is the context's CUDA stream:
each stage enqueues its kernels on it without waiting, the stream runs them
in submission order (each stage sees the previous stage's writes), and
execute() synchronises the stream once and reports any device-side failure
a stage left behind.

Filter stages come from forge-filter, which this build does not include:
Pipeline.filter raises NotImplementedError.
"""
from __future__ import annotations

import ctypes

import numpy as np

from forge_sort import _lib
from forge_sort.errors import SortError, from_status
from forge_sort.sorter import _DT, GpuSorter, SortBuffer

__all__ = ["ForgeContext", "Buffer", "GpuGather", "GatherError", "Pipeline", "PipelineError"]


# -- errors (gather.rs:17-24, pipeline.rs:41-54) ---------------------------------
class GatherError(Exception):
    """Base class; str(e) is the reference's Display string."""


class _GatherShaderCompilation(GatherError):
    def __init__(self, msg: str):
        self.msg = msg
        super().__init__(f"shader compilation failed: {msg}")


class _GatherGpuExecution(GatherError):
    def __init__(self, msg: str):
        self.msg = msg
        super().__init__(f"GPU execution failed: {msg}")


GatherError.ShaderCompilation = _GatherShaderCompilation
GatherError.GpuExecution = _GatherGpuExecution


class PipelineError(Exception):
    """Base class; str(e) is the reference's Display string."""


class _PipelineCommandBuffer(PipelineError):
    def __init__(self):
        super().__init__("failed to create command buffer")


class _PipelineEncoder(PipelineError):
    def __init__(self):
        super().__init__("failed to create compute encoder")


class _PipelineGpuExecution(PipelineError):
    def __init__(self, msg: str):
        self.msg = msg
        super().__init__(f"GPU execution failed: {msg}")


class _PipelineSort(PipelineError):
    def __init__(self, err: SortError):
        self.err = err
        super().__init__(f"sort error: {err}")


PipelineError.CommandBuffer = _PipelineCommandBuffer
PipelineError.Encoder = _PipelineEncoder
PipelineError.GpuExecution = _PipelineGpuExecution
PipelineError.Sort = _PipelineSort


# -- context (context.rs) ----------------------------------------------------------
class Buffer:
    """A buffer from ForgeContext.alloc_buffer: page-locked host memory that
    the host reads and writes directly and the kernels reach through the same
    address (the discrete-GPU form of a StorageModeShared MTLBuffer)."""

    def __init__(self, ctx: "ForgeContext", ptr: int, size: int):
        self._ctx = ctx
        self._ptr = ptr
        self._size = size

    def device_ptr(self) -> int:
        return self._ptr

    metal_buffer = device_ptr

    def length(self) -> int:
        """Size in bytes."""
        return self._size

    def view(self, dtype) -> np.ndarray:
        """Writable numpy view of the whole buffer as `dtype` elements."""
        dt = np.dtype(dtype)
        if self._size < dt.itemsize:
            return np.empty(0, dt)
        raw = (ctypes.c_uint8 * self._size).from_address(self._ptr)
        return np.frombuffer(raw, dtype=dt, count=self._size // dt.itemsize)

    def free(self) -> None:
        if self._ptr:
            self._ctx._alloc.free_device(self._ptr)
            self._ptr = 0


class ForgeContext:
    """One CUDA device and one stream, shared by the sorters and gathers made
    with_context(ctx.device(), ctx.queue()).  Raises forge_sort's
    DeviceNotFound when there is no CUDA device (the reference panics).
    close() destroys the stream and frees the buffers from alloc_buffer:
    sorters and gathers bound to queue() must not be used after it."""

    def __init__(self, device: int = 0):
        L = _lib.load()
        st = ctypes.c_void_p()
        rc = L.fs_stream_create(int(device), ctypes.byref(st))
        if rc != _lib.OK:
            raise from_status(rc, L.fs_last_error(None).decode())
        self._device = int(device)
        self._stream = int(st.value)
        self._alloc = GpuSorter(self._device, self._stream)  # owns alloc_buffer memory
        self._buffers = []

    @classmethod
    def new(cls) -> "ForgeContext":
        return cls(0)

    def device(self) -> int:
        return self._device

    def queue(self) -> int:
        """The cudaStream_t handle (the command queue)."""
        return self._stream

    def alloc_buffer(self, size: int) -> Buffer:
        """`size` bytes the host and the device both reach (context.rs:35-44)."""
        ptr = ctypes.c_void_p()
        self._alloc._call(_lib.load().fs_alloc(self._alloc._h, max(int(size), 1), 1, ctypes.byref(ptr)))
        b = Buffer(self, int(ptr.value), int(size))
        self._buffers.append(b)
        return b

    def synchronize(self) -> None:
        L = _lib.load()
        rc = L.fs_stream_synchronize(ctypes.c_void_p(self._stream))
        if rc != _lib.OK:
            raise from_status(rc, L.fs_last_error(None).decode())

    def close(self) -> None:
        if getattr(self, "_stream", 0):
            for b in self._buffers:
                b.free()
            self._alloc.close()
            _lib.load().fs_stream_destroy(ctypes.c_void_p(self._stream))
            self._stream = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr(x) -> int:
    if isinstance(x, int):
        return x
    return int(x.device_ptr())


def _elements(x, width: int):
    """Element count of a buffer object of `width`-byte elements, if known."""
    if isinstance(x, SortBuffer):
        return x.len() * _DT[x.dtype][2] // width
    if isinstance(x, Buffer):
        return x.length() // width
    return None


# -- gather (gather.rs) ------------------------------------------------------------
class GpuGather:
    """output[i] = source[indices[i]] for u32 or u64 elements and u32 indices.

    Unlike the reference kernel, every index is checked against the source's
    length: an index past it is skipped and reported as GpuExecution when the
    work is waited for.  The source length comes from the buffer object (a
    ForgeContext Buffer or a SortBuffer) or from `source_len` when a raw
    device address is passed."""

    def __init__(self, device: int = 0, stream=None):
        try:
            self._s = GpuSorter(device, stream)
        except SortError as e:
            raise GatherError.ShaderCompilation(str(e)) from None

    @classmethod
    def new(cls) -> "GpuGather":
        return cls(0, None)

    @classmethod
    def with_context(cls, device: int, queue) -> "GpuGather":
        return cls(device, queue)

    def encode_gather(self, stream, source, indices, output, count: int, is_64bit: bool,
                      source_len=None) -> None:
        """Enqueue on `stream` without waiting (gather.rs:77-117)."""
        width = 8 if is_64bit else 4
        src_n = source_len if source_len is not None else _elements(source, width)
        if src_n is None:
            raise ValueError("source_len is required when source is a raw device address")
        if stream is not None:
            self._s.set_stream(stream)
        try:
            self._s.gather_device(width, _ptr(source), int(src_n), _ptr(indices), _ptr(output), int(count),
                                  sync=False)
        except SortError as e:
            raise GatherError.GpuExecution(str(e)) from None

    def synchronize(self) -> None:
        try:
            self._s.synchronize()
        except SortError as e:
            raise GatherError.GpuExecution(e.msg if hasattr(e, "msg") else str(e)) from None

    def _gather_sync(self, source, indices, output, count, is_64bit, source_len):
        self.encode_gather(None, source, indices, output, count, is_64bit, source_len)
        self.synchronize()

    def gather_u32(self, source, indices, output, count: int, source_len=None) -> None:
        self._gather_sync(source, indices, output, count, False, source_len)

    def gather_u64(self, source, indices, output, count: int, source_len=None) -> None:
        self._gather_sync(source, indices, output, count, True, source_len)

    def close(self) -> None:
        self._s.close()


# -- pipeline (pipeline.rs) ----------------------------------------------------------
class Pipeline:
    """Sort and gather stages enqueued on the context's stream; execute()
    waits once.  Stages run in the order they were added."""

    def __init__(self, ctx: ForgeContext):
        if not getattr(ctx, "_stream", 0):
            raise PipelineError.CommandBuffer()
        self._ctx = ctx
        self._users = []  # sorters / gathers with work in flight

    @classmethod
    def new(cls, ctx: ForgeContext) -> "Pipeline":
        return cls(ctx)

    def _track(self, obj) -> None:
        if all(o is not obj for o in self._users):
            self._users.append(obj)

    def filter(self, *args, **kwargs):
        raise NotImplementedError("filter stages need forge-filter, which this build does not include")

    def sort(self, gpu_sorter: GpuSorter, buf: SortBuffer) -> None:
        """Enqueue an in-place sort of a SortBuffer<u32> (pipeline.rs:98-105).
        The sorter is rebound to the context's stream (encode_sort)."""
        try:
            gpu_sorter.encode_sort(self._ctx.queue(), buf)
        except SortError as e:
            raise PipelineError.Sort(e) from None
        self._track(gpu_sorter)

    def gather(self, gpu_gather: GpuGather, source, indices, output, count: int, is_64bit: bool,
               source_len=None) -> None:
        """Enqueue output[i] = source[indices[i]] (pipeline.rs:107-122)."""
        gpu_gather.encode_gather(self._ctx.queue(), source, indices, output, count, is_64bit, source_len)
        self._track(gpu_gather)

    def execute(self) -> None:
        """Wait for every stage, then report the first device-side failure
        (pipeline.rs:124-139)."""
        first = None
        try:
            self._ctx.synchronize()
        except SortError as e:
            first = str(e)
        for o in self._users:
            try:
                o.synchronize()
            except (SortError, GatherError) as e:
                if first is None:
                    first = getattr(e, "msg", str(e))
        self._users = []
        if first is not None:
            raise PipelineError.GpuExecution(first)
