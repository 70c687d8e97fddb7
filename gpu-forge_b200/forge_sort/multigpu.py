"""MultiGpuSorter -- the sample sort over several GPUs of this process
(fs_mg_* in include/forgesort.h).

No counterpart in the reference (forge-sort is single-device).  The shards
are torch tensors, one per device; sort() returns the pieces of the globally
sorted sequence, piece i on device i, and concatenating them in device order
gives the sorted input bit for bit.  The one-process-per-GPU form of the
same algorithm is samplesort.SampleSorter.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence

from . import _lib
from .errors import from_status
from .sorter import _DT, dtype_name


class MultiGpuSorter:
    def __init__(self, devices: Sequence[int]):
        L = _lib.load()
        arr = (ctypes.c_int * len(devices))(*[int(d) for d in devices])
        h = ctypes.c_void_p()
        rc = L.fs_mg_create(arr, len(devices), ctypes.byref(h))
        if rc != _lib.OK:
            raise from_status(rc, L.fs_last_error(None).decode() or "fs_mg_create failed")
        self._h = h
        self.devices = [int(d) for d in devices]

    @classmethod
    def new(cls, devices: Sequence[int]) -> "MultiGpuSorter":
        return cls(devices)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().fs_mg_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, name, shards, what="shard", size=None):
        G = len(self.devices)
        if len(shards) != G:
            raise ValueError(f"{len(shards)} {what}s for {G} devices")
        for i, t in enumerate(shards):
            if t.device.type != "cuda" or t.device.index != self.devices[i] or not t.is_contiguous():
                raise ValueError(f"{what} {i} must be a contiguous tensor on cuda:{self.devices[i]}")
            want = size if size is not None else _DT[name][2]
            if t.element_size() != want:
                raise TypeError(f"{what} {i} has {t.element_size()}-byte elements, {want} needed")

    def _run(self, name, shards, vals, payload: bool, headroom: float):
        import torch
        G = len(self.devices)
        total = sum(t.numel() for t in shards)
        cap = [int(total / G * headroom) + 1024] * G
        L = _lib.load()
        U64 = ctypes.c_uint64 * G
        PV = ctypes.c_void_p * G
        for _attempt in range(2):
            outs = [torch.empty(cap[i], dtype=shards[i].dtype, device=shards[i].device) for i in range(G)]
            vouts = [torch.empty(cap[i], dtype=torch.int32, device=shards[i].device) for i in range(G)] \
                if payload else None
            for t in shards:
                torch.cuda.current_stream(t.device).synchronize()  # shards ready
            out_n = U64()
            sp, sn = PV(*[t.data_ptr() for t in shards]), U64(*[t.numel() for t in shards])
            op = PV(*[t.data_ptr() for t in outs])
            if payload:
                vp = PV(*[v.data_ptr() for v in vals]) if vals is not None else None
                rc = L.fs_mg_sort_pairs(self._h, _DT[name][0], sp, vp, sn, op, PV(*[v.data_ptr() for v in vouts]),
                                        U64(*cap), out_n)
            else:
                rc = L.fs_mg_sort_keys(self._h, _DT[name][0], sp, sn, op, U64(*cap), out_n)
            if rc == _lib.OK:
                keys = [outs[i][: out_n[i]] for i in range(G)]
                return (keys, [vouts[i][: out_n[i]] for i in range(G)]) if payload else keys
            if rc == _lib.E_INVALID and any(out_n[i] > cap[i] for i in range(G)):
                cap = [max(cap[i], int(out_n[i])) for i in range(G)]  # resize and retry once
                continue
            raise from_status(rc, L.fs_mg_last_error(self._h).decode())
        raise RuntimeError("MultiGpuSorter: output sizing failed")

    def sort(self, dt, shards: List, headroom: float = 1.125) -> List:
        """Sort the concatenation of `shards` (1-D torch tensors holding raw
        key bits, shard i on devices[i]); returns the sorted pieces."""
        name = dtype_name(dt)
        self._check(name, shards)
        return self._run(name, shards, None, False, headroom)

    def sort_pairs(self, dt, shards: List, values: List, headroom: float = 1.125):
        """Stable sort of (key, value) pairs by key across the devices:
        values[i] is an int32 tensor of u32 values beside shards[i].  Returns
        (key pieces, value pieces); equal keys keep their global input
        order."""
        name = dtype_name(dt)
        self._check(name, shards)
        self._check(name, values, "value", 4)
        if any(v.numel() != t.numel() for v, t in zip(values, shards)):
            raise ValueError("one value per key")
        return self._run(name, shards, values, True, headroom)

    def argsort(self, dt, shards: List, headroom: float = 1.125):
        """Stable argsort across the devices: (key pieces, position pieces),
        positions into the concatenated shards as u32 in int32 tensors (at
        most 2^32 keys in total)."""
        name = dtype_name(dt)
        self._check(name, shards)
        return self._run(name, shards, None, True, headroom)

    # the per-type names of the boundary (MultiGpuSorter::sort_u32 / sort_u64)
    def sort_u32(self, shards: List, headroom: float = 1.125) -> List:
        return self.sort("u32", shards, headroom)

    def sort_u64(self, shards: List, headroom: float = 1.125) -> List:
        return self.sort("u64", shards, headroom)
