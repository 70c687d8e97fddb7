"""GpuSorter / SortBuffer -- the forge-sort API over the CUDA C ABI.

Mirrors metal-forge-compute/forge-sort/src/lib.rs of kavanaghpatrick/gpu-forge
method for method (names, argument meaning, n <= 1 short-cuts, error
variants); every call goes through libforgesort.so (include/forgesort.h).

Type mapping from the Rust API:
  &mut [u32] / &[f32] ...   -> 1-D C-contiguous numpy arrays of that dtype
  Vec<u32> (argsort result) -> numpy uint32 array
  SortBuffer<T>             -> SortBuffer (device memory + page-locked host
                               mirror kept coherent lazily: sorts stay in HBM,
                               as_slice() copies back only what they changed)
  MTLDevice / command queue -> CUDA device ordinal / cudaStream_t handle
  Result<_, SortError>      -> return value, or raises SortError
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from .errors import (DeviceNotFound, GpuExecution, LengthMismatch,  # noqa: F401
                     ShaderCompilation, SortError, from_status)

_DT = {
    "u32": (_lib.U32, np.uint32, 4),
    "i32": (_lib.I32, np.int32, 4),
    "f32": (_lib.F32, np.float32, 4),
    "u64": (_lib.U64, np.uint64, 8),
    "i64": (_lib.I64, np.int64, 8),
    "f64": (_lib.F64, np.float64, 8),
}
_NP_TO_NAME = {np.dtype(v[1]): k for k, v in _DT.items()}

# SortKey constants (src/lib.rs:29-88): KEY_SIZE, NEEDS_TRANSFORM, IS_64BIT,
# TRANSFORM_MODE_FORWARD, TRANSFORM_MODE_INVERSE.
SORT_KEY = {
    "u32": (4, False, False, 0, 0),
    "i32": (4, True, False, 0, 0),
    "f32": (4, True, False, 1, 2),
    "u64": (8, False, True, 0, 0),
    "i64": (8, True, True, 0, 0),
    "f64": (8, True, True, 1, 2),
}


def dtype_name(dt) -> str:
    """'u32' | 'i32' | 'f32' | 'u64' | 'i64' | 'f64' from a name or numpy dtype."""
    if isinstance(dt, str) and dt in _DT:
        return dt
    try:
        return _NP_TO_NAME[np.dtype(dt)]
    except (TypeError, KeyError):
        raise TypeError(f"not a SortKey type: {dt!r} (u32, i32, f32, u64, i64, f64)") from None


_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream's handle


def _stream_handle(stream) -> Optional[int]:
    """Accept None (the sorter's own stream), an int cudaStream_t (0 also
    means the sorter's own stream, as NULL does in the C ABI), or an object
    with .cuda_stream such as a torch.cuda.Stream.  torch's default stream
    reports handle 0; it is the legacy default stream, so it is passed as
    cudaStreamLegacy and the work really runs on it."""
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream or None
    h = getattr(stream, "cuda_stream", None)
    if h is None:
        raise TypeError("stream must be None, an int cudaStream_t, or have .cuda_stream")
    return int(h) or _CUDA_STREAM_LEGACY


def _check_array(a, name: str, want: str) -> np.ndarray:
    if not isinstance(a, np.ndarray):
        raise TypeError(f"{name} must be a numpy array of {want}")
    if a.dtype != np.dtype(_DT[want][1]):
        raise TypeError(f"{name} has dtype {a.dtype}, expected {np.dtype(_DT[want][1])}")
    if a.ndim != 1 or not a.flags.c_contiguous:
        raise TypeError(f"{name} must be 1-D and C-contiguous")
    if not a.flags.writeable:
        raise TypeError(f"{name} must be writeable")
    return a


class SortBuffer:
    """A buffer the host and the GPU share (reference SortBuffer<T>,
    src/lib.rs:160-281): device memory plus a page-locked host mirror, kept
    coherent lazily by the library (fs_buffer_*).  Sorting a buffer sorts the
    device copy in place and copies nothing back, so repeated sorts of a
    buffer the host does not touch run at device speed.  as_slice() /
    copy_to_slice() bring the host mirror up to date first; as_mut_slice() /
    copy_from_slice() mark the device copy stale, so the next sort copies over
    what the host wrote.  A view returned by as_mut_slice() is a host write
    session: call as_mut_slice() again before writing after a sort (in Rust
    the borrow checker enforces this)."""

    def __init__(self, sorter: "GpuSorter", dt: str, handle: int, length: int, capacity: int,
                 owned: bool = True):
        self._sorter = sorter
        self.dtype = dt
        self._h = handle
        self._len = length
        self._cap = capacity
        self._owned = owned
        L = _lib.load()
        self._host = int(L.fs_buffer_host(ctypes.c_void_p(handle)) or 0)
        self._dev = int(L.fs_buffer_device(ctypes.c_void_p(handle)) or 0)

    @property
    def handle(self) -> int:
        """The library's buffer object (fs_buffer*)."""
        return self._h

    def _check(self, rc: int) -> None:
        if rc != _lib.OK:
            raise from_status(rc, _lib.load().fs_last_error(None).decode())

    # -- reference accessors --------------------------------------------------
    def len(self) -> int:
        return self._len

    def __len__(self) -> int:
        return self._len

    def is_empty(self) -> bool:
        return self._len == 0

    def capacity(self) -> int:
        return self._cap

    def _view(self, count: int) -> np.ndarray:
        npdt = np.dtype(_DT[self.dtype][1])
        if count == 0:
            return np.empty(0, npdt)
        raw = (ctypes.c_uint8 * (count * npdt.itemsize)).from_address(self._host)
        return np.frombuffer(raw, dtype=npdt, count=count)

    def _host_read(self) -> None:
        self._sorter._host_access()
        self._check(_lib.load().fs_buffer_host_read(ctypes.c_void_p(self._h)))

    def _host_write(self) -> None:
        self._sorter._host_access()
        self._check(_lib.load().fs_buffer_host_write(ctypes.c_void_p(self._h)))

    def as_mut_slice(self) -> np.ndarray:
        """Writable view of all `capacity` elements (write, then set_len)."""
        self._host_write()
        return self._view(self._cap)

    def as_slice(self) -> np.ndarray:
        """View of the first len() elements (sorted results after a sort)."""
        self._host_read()
        v = self._view(self._len)
        v.flags.writeable = False
        return v

    def set_len(self, length: int) -> None:
        if length > self._cap:
            raise AssertionError(f"len {length} exceeds capacity {self._cap}")
        self._len = length

    def copy_from_slice(self, data) -> None:
        data = np.ascontiguousarray(data, dtype=_DT[self.dtype][1])
        if data.size > self._cap:
            raise AssertionError(f"data len {data.size} exceeds capacity {self._cap}")
        self._host_write()
        self._view(data.size)[:] = data
        self._len = data.size

    def copy_to_slice(self, dest: np.ndarray) -> None:
        n = min(self._len, dest.size)
        self._host_read()
        dest[:n] = self._view(n)

    def device_ptr(self) -> int:
        """Device address of element 0 (replaces metal_buffer()), for other
        device code: the device copy is made current for len() elements and
        counted as written, so a later host read waits for the device."""
        self._sorter._host_access()
        self._check(_lib.load().fs_buffer_device_use(ctypes.c_void_p(self._h), self._len * _DT[self.dtype][2]))
        return self._dev

    metal_buffer = device_ptr  # deprecated alias of the reference's accessor

    @classmethod
    def from_raw_parts(cls, sorter: "GpuSorter", dt, handle: int, length: int, capacity: int):
        """Re-wrap a buffer object given up by into_raw_parts (owned again)."""
        if length > capacity:
            raise AssertionError(f"len {length} exceeds capacity {capacity}")
        name = dtype_name(dt)
        if capacity * _DT[name][2] > int(_lib.load().fs_buffer_bytes(ctypes.c_void_p(handle))):
            raise AssertionError("capacity exceeds the buffer object's size")
        return cls(sorter, name, handle, length, capacity, owned=True)

    def into_raw_parts(self):
        """Give up ownership: returns (buffer object handle, len, capacity);
        free it with from_raw_parts(...).free() or fs_buffer_destroy."""
        self._owned = False
        h, self._h = self._h, 0
        return h, self._len, self._cap

    def free(self) -> None:
        if self._owned and self._h:
            _lib.load().fs_buffer_destroy(ctypes.c_void_p(self._h))
        self._h = 0
        self._owned = False

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class GpuSorter:
    """GPU radix sort for u32/i32/f32/u64/i64/f64 keys on one CUDA device.

    new() / GpuSorter() create a private stream on device 0;
    with_context(device, stream) enqueues on the caller's stream
    (src/lib.rs:596-686).  Calls are synchronous unless stated otherwise.
    """

    def __init__(self, device: int = 0, stream=None):
        L = _lib.load()
        h = ctypes.c_void_p()
        rc = L.fs_create(int(device), _stream_handle(stream), ctypes.byref(h))
        if rc != _lib.OK:
            raise from_status(rc, L.fs_last_error(None).decode())
        self._h = h
        self.device = int(device)
        self.stream_handle = _stream_handle(stream)  # None: the sorter's own stream
        self._pending = False

    @classmethod
    def new(cls) -> "GpuSorter":
        return cls(0, None)

    @classmethod
    def with_context(cls, device: int, stream) -> "GpuSorter":
        return cls(device, stream)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().fs_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- plumbing ---------------------------------------------------------------
    def _err_text(self) -> str:
        return _lib.load().fs_last_error(self._h).decode()

    def _call(self, rc: int, **kw) -> None:
        if rc == _lib.OK:
            return
        if rc == _lib.E_INVALID:
            raise ValueError(self._err_text())
        raise from_status(rc, self._err_text(), **kw)

    def _host_access(self) -> None:
        # encode_sort leaves work in flight; the host must not touch buffer
        # pages until it has finished.
        if self._pending:
            self.synchronize()

    def synchronize(self) -> None:
        self._pending = False
        self._call(_lib.load().fs_synchronize(self._h))

    def set_stream(self, stream) -> None:
        self._call(_lib.load().fs_set_stream(self._h, _stream_handle(stream)))
        self.stream_handle = _stream_handle(stream)

    def scratch_bytes(self) -> int:
        return int(_lib.load().fs_scratch_bytes(self._h))

    def last_launch_count(self) -> int:
        return int(_lib.load().fs_last_launch_count(self._h))

    def set_wait_timeout_ms(self, ms: int) -> None:
        """Bound on every device-side wait of this sorter (default 2000 ms)."""
        self._call(_lib.load().fs_set_wait_timeout_ms(self._h, int(ms)))

    def set_single_launch_max(self, key_bytes: int) -> None:
        """Keys-only 32-bit sorts of up to `key_bytes` bytes of keys run as
        one cooperative launch (default 8 MiB; 0: always the chained kernels)."""
        self._call(_lib.load().fs_set_single_launch_max(self._h, int(key_bytes)))

    def _test_inject(self, kind: int, arg: int = 0) -> None:
        """Failure-path test hook (fs_test_inject): arm one injected failure."""
        self._call(_lib.load().fs_test_inject(self._h, int(kind), int(arg)))

    # -- zero-copy buffers (src/lib.rs:694-738, 1000-1117, 2301-2590) -----------
    def alloc_sort_buffer(self, dt, capacity: int) -> SortBuffer:
        name = dtype_name(dt)
        h = ctypes.c_void_p()
        self._call(_lib.load().fs_buffer_create(self._h, max(capacity, 1) * _DT[name][2], ctypes.byref(h)))
        return SortBuffer(self, name, h.value, 0, capacity)

    def _sort_buf(self, buf: SortBuffer, want: str, sync: bool = True) -> None:
        if buf.dtype != want:
            raise TypeError(f"SortBuffer<{buf.dtype}> passed where SortBuffer<{want}> is required")
        if buf.len() <= 1:
            return
        self._call(_lib.load().fs_sort_buffer(self._h, _DT[want][0], ctypes.c_void_p(buf.handle), buf.len(),
                                              int(sync)))
        self._pending = self._pending or not sync

    def sort_buffer(self, buf: SortBuffer) -> None:
        self._sort_buf(buf, "u32")

    def sort_i32_buffer(self, buf: SortBuffer) -> None:
        self._sort_buf(buf, "i32")

    def sort_f32_buffer(self, buf: SortBuffer) -> None:
        self._sort_buf(buf, "f32")

    def sort_u64_buffer(self, buf: SortBuffer) -> None:
        self._sort_buf(buf, "u64")

    def sort_i64_buffer(self, buf: SortBuffer) -> None:
        self._sort_buf(buf, "i64")

    def sort_f64_buffer(self, buf: SortBuffer) -> None:
        self._sort_buf(buf, "f64")

    def sort_pairs_buffer(self, keys: SortBuffer, values: SortBuffer) -> None:
        """Zero-copy stable key/value sort (additive: not in the reference)."""
        if values.dtype != "u32":
            raise TypeError("values must be a SortBuffer<u32>")
        if keys.len() != values.len():
            raise LengthMismatch(keys.len(), values.len())
        if keys.len() <= 1:
            return
        self._call(_lib.load().fs_sort_pairs_buffer(self._h, _DT[keys.dtype][0], ctypes.c_void_p(keys.handle),
                                                    ctypes.c_void_p(values.handle), keys.len(), 1))

    def encode_sort(self, stream, buf: SortBuffer) -> None:
        """Enqueue an in-place u32 sort of `buf` on `stream` without waiting
        (src/lib.rs:749-785: the caller commits and waits).  Reading the
        buffer afterwards (as_slice) waits for the sort."""
        if buf.dtype != "u32":
            raise TypeError("encode_sort takes a SortBuffer<u32>")
        if buf.len() <= 1:
            return
        h = _stream_handle(stream)
        if h is not None:
            self.set_stream(h)
        self._sort_buf(buf, "u32", sync=False)

    # -- host slices (src/lib.rs:791-998, 2238-2485) --------------------------
    def _sort_host(self, data, want: str) -> None:
        a = _check_array(data, "data", want)
        if a.size <= 1:
            return
        self._call(_lib.load().fs_host_sort_keys(self._h, _DT[want][0], ctypes.c_void_p(a.ctypes.data),
                                                 a.size))

    def sort_u32(self, data) -> None:
        self._sort_host(data, "u32")

    def sort_i32(self, data) -> None:
        self._sort_host(data, "i32")

    def sort_f32(self, data) -> None:
        self._sort_host(data, "f32")

    def sort_u64(self, data) -> None:
        self._sort_host(data, "u64")

    def sort_i64(self, data) -> None:
        self._sort_host(data, "i64")

    def sort_f64(self, data) -> None:
        self._sort_host(data, "f64")

    # -- argsort (src/lib.rs:1675-1921, 2595-2825) ----------------------------
    def _argsort_host(self, data, want: str) -> np.ndarray:
        if not isinstance(data, np.ndarray) or data.dtype != np.dtype(_DT[want][1]) or data.ndim != 1:
            raise TypeError(f"data must be a 1-D numpy array of {np.dtype(_DT[want][1])}")
        a = np.ascontiguousarray(data)
        n = a.size
        if n == 0:
            return np.empty(0, np.uint32)
        if n == 1:
            return np.zeros(1, np.uint32)
        out = np.empty(n, np.uint32)
        self._call(_lib.load().fs_host_argsort(self._h, _DT[want][0], ctypes.c_void_p(a.ctypes.data),
                                               ctypes.c_void_p(out.ctypes.data), n))
        return out

    def argsort_u32(self, data) -> np.ndarray:
        return self._argsort_host(data, "u32")

    def argsort_i32(self, data) -> np.ndarray:
        return self._argsort_host(data, "i32")

    def argsort_f32(self, data) -> np.ndarray:
        return self._argsort_host(data, "f32")

    def argsort_u64(self, data) -> np.ndarray:
        return self._argsort_host(data, "u64")

    def argsort_i64(self, data) -> np.ndarray:
        return self._argsort_host(data, "i64")

    def argsort_f64(self, data) -> np.ndarray:
        return self._argsort_host(data, "f64")

    # -- pairs (src/lib.rs:1923-2236, 2826-3015) ------------------------------
    def _pairs_host(self, keys, values, want: str) -> None:
        k = _check_array(keys, "keys", want)
        v = _check_array(values, "values", "u32")
        self._call(_lib.load().fs_host_sort_pairs(self._h, _DT[want][0], ctypes.c_void_p(k.ctypes.data), k.size,
                                                  ctypes.c_void_p(v.ctypes.data), v.size),
                   keys=k.size, values=v.size)

    def sort_pairs_u32(self, keys, values) -> None:
        self._pairs_host(keys, values, "u32")

    def sort_pairs_i32(self, keys, values) -> None:
        self._pairs_host(keys, values, "i32")

    def sort_pairs_f32(self, keys, values) -> None:
        self._pairs_host(keys, values, "f32")

    def sort_pairs_u64(self, keys, values) -> None:
        self._pairs_host(keys, values, "u64")

    def sort_pairs_i64(self, keys, values) -> None:
        self._pairs_host(keys, values, "i64")

    def sort_pairs_f64(self, keys, values) -> None:
        """Additive: the reference has no sort_pairs_f64."""
        self._pairs_host(keys, values, "f64")

    # -- raw device pointers (bench, sample sort, torch interop) --------------
    def sort_device(self, dt, ptr: int, n: int, sync: bool = True) -> None:
        name = dtype_name(dt)
        self._call(_lib.load().fs_sort_keys(self._h, _DT[name][0], ctypes.c_void_p(ptr), n, int(sync)))
        self._pending = self._pending or not sync

    def sort_pairs_device(self, dt, kptr: int, vptr: int, n: int, sync: bool = True) -> None:
        name = dtype_name(dt)
        self._call(_lib.load().fs_sort_pairs(self._h, _DT[name][0], ctypes.c_void_p(kptr), ctypes.c_void_p(vptr),
                                             n, int(sync)))
        self._pending = self._pending or not sync

    def argsort_device(self, dt, kptr: int, idx_ptr: int, n: int, sync: bool = True) -> None:
        name = dtype_name(dt)
        self._call(_lib.load().fs_argsort(self._h, _DT[name][0], ctypes.c_void_p(kptr), ctypes.c_void_p(idx_ptr),
                                          n, int(sync)))
        self._pending = self._pending or not sync

    def sort_device_copy(self, dt, in_ptr: int, out_ptr: int, n: int, sync: bool = True) -> None:
        """Out-of-place sort of device keys: in_ptr is left untouched."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_sort_keys_copy(self._h, _DT[name][0], ctypes.c_void_p(in_ptr),
                                                 ctypes.c_void_p(out_ptr), n, int(sync)))
        self._pending = self._pending or not sync

    def sort_pairs_device_copy(self, dt, kin: int, vin: int, kout: int, vout: int, n: int,
                               sync: bool = True) -> None:
        """Out-of-place stable pairs sort of device memory; vin == 0 takes the
        input positions as values.  The inputs are left untouched."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_sort_pairs_copy(self._h, _DT[name][0], ctypes.c_void_p(kin),
                                                  ctypes.c_void_p(vin or None), ctypes.c_void_p(kout),
                                                  ctypes.c_void_p(vout), n, int(sync)))
        self._pending = self._pending or not sync

    def host_sort_copy_async_ptr(self, dt, host_in: int, host_out: int, n: int) -> None:
        """Enqueue host-memory out-of-place sort (H2D + sort + D2H) and return;
        consecutive calls overlap their copies.  synchronize() waits."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_host_sort_keys_copy_async(self._h, _DT[name][0], ctypes.c_void_p(host_in),
                                                            ctypes.c_void_p(host_out), n))
        self._pending = True

    def host_sort_copy_ptr(self, dt, host_in: int, host_out: int, n: int) -> None:
        """Host-memory out-of-place sort: H2D + sort + D2H (synchronous)."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_host_sort_keys_copy(self._h, _DT[name][0], ctypes.c_void_p(host_in),
                                                      ctypes.c_void_p(host_out), n))

    def set_kernel_timing(self, on: bool) -> None:
        self._call(_lib.load().fs_set_kernel_timing(self._h, int(on)))

    def last_kernel_times(self, cap: int = 24):
        """Per-kernel device times (ms) of the last sort, launch order:
        histogram, plan, pass 0..P-1, finalize."""
        buf = (ctypes.c_float * cap)()
        k = _lib.load().fs_last_kernel_times(self._h, buf, cap)
        if k < 0:
            self._call(-k)
        return [float(buf[i]) for i in range(k)]

    def partition_device(self, dt, in_ptr: int, n: int, gpos_base: int, spl_keys_ptr: int, spl_gpos_ptr: int,
                         nsplit: int, out_ptr: int, counts_ptr: int, sync: bool = True) -> None:
        """Stable splitter partition (multi-GPU sample sort step), device pointers."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_partition(self._h, _DT[name][0], ctypes.c_void_p(in_ptr), n, gpos_base,
                                            ctypes.c_void_p(spl_keys_ptr), ctypes.c_void_p(spl_gpos_ptr), nsplit,
                                            ctypes.c_void_p(out_ptr), ctypes.c_void_p(counts_ptr), int(sync)))
        self._pending = self._pending or not sync

    def partition_count(self, dt, in_ptr: int, n: int, gpos_base: int, spl_keys_ptr: int, spl_gpos_ptr: int,
                        nsplit: int) -> list:
        """Dispatch step 1: bucket sizes of n device keys (host list of
        nsplit+1 ints); waits for the stream."""
        name = dtype_name(dt)
        out = (ctypes.c_uint64 * (nsplit + 1))()
        self._call(_lib.load().fs_partition_count(self._h, _DT[name][0], ctypes.c_void_p(in_ptr), n, gpos_base,
                                                  ctypes.c_void_p(spl_keys_ptr), ctypes.c_void_p(spl_gpos_ptr),
                                                  nsplit, out))
        return [int(x) for x in out]

    def partition_count_async(self, dt, in_ptr: int, n: int, gpos_base: int, spl_keys_ptr: int,
                              spl_gpos_ptr: int, nsplit: int, counts_dev_ptr: int) -> None:
        """Dispatch step 1 without a host round trip: the nsplit+1 bucket
        sizes go to device memory (u64), stream-ordered."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_partition_count_async(
            self._h, _DT[name][0], ctypes.c_void_p(in_ptr), n, gpos_base, ctypes.c_void_p(spl_keys_ptr),
            ctypes.c_void_p(spl_gpos_ptr), nsplit, ctypes.c_void_p(counts_dev_ptr)))
        self._pending = True

    def partition_dispatch_matrix(self, dt, in_ptr: int, n: int, gpos_base: int, spl_keys_ptr: int,
                                  spl_gpos_ptr: int, nsplit: int, send_matrix_ptr: int, rank: int, inbox_keys,
                                  inbox_vals=None, vals_ptr: int = 0, payload: bool = False,
                                  sync: bool = False) -> None:
        """Dispatch step 2 with the destinations computed on the device from
        the all-gathered send matrix (device, (nsplit+1)^2 u64) and this
        rank's index; inbox_keys / inbox_vals are the peers' inbox bases."""
        name = dtype_name(dt)
        G = nsplit + 1
        kt = (ctypes.c_void_p * G)(*[ctypes.c_void_p(int(p)) for p in inbox_keys])
        vt = (ctypes.c_void_p * G)(*[ctypes.c_void_p(int(p)) for p in inbox_vals]) if payload else None
        self._call(_lib.load().fs_partition_dispatch_matrix(
            self._h, _DT[name][0], ctypes.c_void_p(in_ptr), ctypes.c_void_p(vals_ptr or None), int(payload), n,
            gpos_base, ctypes.c_void_p(spl_keys_ptr), ctypes.c_void_p(spl_gpos_ptr), nsplit,
            ctypes.c_void_p(send_matrix_ptr), int(rank), kt, vt, int(sync)))
        self._pending = self._pending or not sync

    def partition_dispatch(self, dt, in_ptr: int, n: int, gpos_base: int, spl_keys_ptr: int, spl_gpos_ptr: int,
                           nsplit: int, dst_ptrs, sync: bool = False) -> None:
        """Dispatch step 2: store bucket b's keys at dst_ptrs[b] (device
        pointers, possibly peer GPUs' memory opened with ipc_open)."""
        name = dtype_name(dt)
        tab = (ctypes.c_void_p * (nsplit + 1))(*[ctypes.c_void_p(int(p)) for p in dst_ptrs])
        self._call(_lib.load().fs_partition_dispatch(self._h, _DT[name][0], ctypes.c_void_p(in_ptr), n, gpos_base,
                                                     ctypes.c_void_p(spl_keys_ptr), ctypes.c_void_p(spl_gpos_ptr),
                                                     nsplit, tab, int(sync)))
        self._pending = self._pending or not sync

    def partition_dispatch_pairs(self, dt, in_ptr: int, vals_ptr: int, n: int, gpos_base: int, spl_keys_ptr: int,
                                 spl_gpos_ptr: int, nsplit: int, dst_ptrs, vdst_ptrs, sync: bool = False) -> None:
        """Dispatch step 2 with a u32 payload: value i goes to vdst_ptrs[b]
        beside key i; vals_ptr == 0 sends global positions gpos_base + i."""
        name = dtype_name(dt)
        tab = (ctypes.c_void_p * (nsplit + 1))(*[ctypes.c_void_p(int(p)) for p in dst_ptrs])
        vtab = (ctypes.c_void_p * (nsplit + 1))(*[ctypes.c_void_p(int(p)) for p in vdst_ptrs])
        self._call(_lib.load().fs_partition_dispatch_pairs(
            self._h, _DT[name][0], ctypes.c_void_p(in_ptr), ctypes.c_void_p(vals_ptr or None), n, gpos_base,
            ctypes.c_void_p(spl_keys_ptr), ctypes.c_void_p(spl_gpos_ptr), nsplit, tab, vtab, int(sync)))
        self._pending = self._pending or not sync

    def gather_device(self, width: int, src_ptr: int, src_n: int, idx_ptr: int, dst_ptr: int, n: int,
                      sync: bool = True) -> None:
        """dst[i] = src[idx[i]] on device memory (width 4 or 8 bytes per
        element, u32 indices) -- forge-runtime's GpuGather."""
        self._call(_lib.load().fs_gather(self._h, int(width), ctypes.c_void_p(src_ptr), src_n,
                                         ctypes.c_void_p(idx_ptr), ctypes.c_void_p(dst_ptr), n, int(sync)))
        self._pending = self._pending or not sync

    def alloc_device(self, nbytes: int) -> int:
        """Plain device memory (cudaMalloc) owned by the sorter; free_device()."""
        ptr = ctypes.c_void_p()
        self._call(_lib.load().fs_alloc(self._h, nbytes, 0, ctypes.byref(ptr)))
        return int(ptr.value)

    def free_device(self, ptr: int) -> None:
        self._call(_lib.load().fs_free(self._h, ctypes.c_void_p(ptr)))

    def ipc_export(self, ptr: int) -> bytes:
        h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        self._call(_lib.load().fs_ipc_export(self._h, ctypes.c_void_p(ptr), h))
        return bytes(h)

    def ipc_open(self, handle: bytes) -> int:
        h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(handle)
        ptr = ctypes.c_void_p()
        self._call(_lib.load().fs_ipc_open(self._h, h, ctypes.byref(ptr)))
        return int(ptr.value)

    def ipc_close(self, ptr: int) -> None:
        self._call(_lib.load().fs_ipc_close(self._h, ctypes.c_void_p(ptr)))

    def host_sort_ptr(self, dt, host_ptr: int, n: int) -> None:
        """sort_<dt> on raw (e.g. pinned) host memory; H2D + sort + D2H."""
        name = dtype_name(dt)
        self._call(_lib.load().fs_host_sort_keys(self._h, _DT[name][0], ctypes.c_void_p(host_ptr), n))
