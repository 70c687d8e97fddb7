"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the CPU oracle.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker or the timed CPU reference.  The product path
(gpu-forge_b200/forge_sort) never imports it.

The oracle restates the results forge-sort's own tests pin
(kavanaghpatrick/gpu-forge, metal-forge-compute/forge-sort):
  * keys    -> Rust sort_unstable / sort_by(total_cmp) order
               (tests/correctness_f32.rs:115-212, correctness_f64.rs:110-180)
  * argsort -> stable sort_by_key (tests/correctness_argsort.rs:42-56)
  * pairs   -> stable sort_by_key, values follow (correctness_sort_pairs.rs:35-45)
See oracle.cpp for the C++ restatement and the input generators.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# fs_dtype numbering (include/forgesort.h)
DTYPES = {"u32": 0, "i32": 1, "f32": 2, "u64": 3, "i64": 4, "f64": 5}
NP_DTYPE = {
    "u32": np.uint32, "i32": np.int32, "f32": np.float32,
    "u64": np.uint64, "i64": np.int64, "f64": np.float64,
}
BITS_DTYPE = {"u32": np.uint32, "i32": np.uint32, "f32": np.uint32,
              "u64": np.uint64, "i64": np.uint64, "f64": np.uint64}

_lib = None


def build() -> None:
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u64, vp, i32 = ctypes.c_uint64, ctypes.c_void_p, ctypes.c_int
        L.orc_xs_jump.restype = u64
        L.orc_xs_jump.argtypes = [u64, u64]
        for f in ("orc_gen_u64", "orc_gen_u32", "orc_gen_skew_u32"):
            getattr(L, f).argtypes = [u64, u64, u64, vp]
        L.orc_gen_f32_mix.argtypes = [u64, u64, vp]
        L.orc_gen_f64_logu.argtypes = [u64, u64, vp]
        L.orc_gen_zipf_u32.argtypes = [u64, u64, ctypes.c_double, ctypes.c_uint32, vp]
        L.orc_fnv1a64.restype = u64
        L.orc_fnv1a64.argtypes = [vp, u64]
        L.orc_sort_keys.argtypes = [i32, vp, u64]
        L.orc_par_sort_keys.argtypes = [i32, vp, u64, i32]
        L.orc_argsort.argtypes = [i32, vp, vp, u64]
        L.orc_sort_pairs.argtypes = [i32, vp, vp, u64]
        L.orc_radix_sort.argtypes = [i32, vp, vp, u64]
        L.orc_par_argsort.argtypes = [i32, vp, vp, u64, i32]
        L.orc_par_sort_pairs.argtypes = [i32, vp, vp, u64, i32]
        L.orc_max_threads.restype = i32
        for f, t in (("orc_to_ordered32", ctypes.c_uint32), ("orc_from_ordered32", ctypes.c_uint32),
                     ("orc_to_ordered64", u64), ("orc_from_ordered64", u64)):
            getattr(L, f).restype = t
            getattr(L, f).argtypes = [t, i32]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


# ------------------------------------------------------------------ generators
def gen(dist: str, n: int, seed: int = 42, start: int = 0) -> np.ndarray:
    """Seeded synthetic inputs (BASELINE configs D1-D5).

    dist: u32 | i32 | u64 | i64 | skew_u32 | f32_mix | f64_logu | zipf_u32
    Returned arrays carry the natural dtype (int/float views of the bits).
    """
    L = lib()
    if dist in ("u32", "i32"):
        out = np.empty(n, np.uint32)
        L.orc_gen_u32(seed, start, n, _ptr(out))
        return out.view(np.int32) if dist == "i32" else out
    if dist in ("u64", "i64"):
        out = np.empty(n, np.uint64)
        L.orc_gen_u64(seed, start, n, _ptr(out))
        return out.view(np.int64) if dist == "i64" else out
    if dist == "skew_u32":
        out = np.empty(n, np.uint32)
        L.orc_gen_skew_u32(seed, start, n, _ptr(out))
        return out
    if dist == "f32_mix":
        out = np.empty(n, np.uint32)
        L.orc_gen_f32_mix(seed, n, _ptr(out))
        return out.view(np.float32)
    if dist == "f64_logu":
        out = np.empty(n, np.uint64)
        L.orc_gen_f64_logu(seed, n, _ptr(out))
        return out.view(np.float64)
    if dist == "zipf_u32":
        out = np.empty(n, np.uint32)
        L.orc_gen_zipf_u32(seed, n, 1.1, 1 << 16, _ptr(out))
        return out
    raise ValueError(f"unknown distribution {dist}")


def fnv1a64(a: np.ndarray) -> int:
    a = np.ascontiguousarray(a)
    return int(lib().orc_fnv1a64(_ptr(a), a.nbytes))


# ------------------------------------------------------------------ oracles
def _bits(a: np.ndarray, dt: str) -> np.ndarray:
    return np.ascontiguousarray(a).view(BITS_DTYPE[dt])


def sort_keys(a: np.ndarray, dt: str) -> np.ndarray:
    """Sorted copy in Rust sort_unstable / total_cmp order (bit-exact)."""
    out = np.array(a, dtype=NP_DTYPE[dt], copy=True, order="C")
    lib().orc_sort_keys(DTYPES[dt], _ptr(out), out.size)
    return out


def par_sort_keys(a: np.ndarray, dt: str, threads: int = 0) -> np.ndarray:
    out = np.array(a, dtype=NP_DTYPE[dt], copy=True, order="C")
    lib().orc_par_sort_keys(DTYPES[dt], _ptr(out), out.size, threads)
    return out


def radix_sort_keys(a: np.ndarray, dt: str) -> np.ndarray:
    out = np.array(a, dtype=NP_DTYPE[dt], copy=True, order="C")
    lib().orc_radix_sort(DTYPES[dt], _ptr(out), None, out.size)
    return out


def argsort(a: np.ndarray, dt: str) -> np.ndarray:
    """Stable sorting permutation (u32), ties in index order."""
    a = np.ascontiguousarray(a, dtype=NP_DTYPE[dt])
    idx = np.empty(a.size, np.uint32)
    lib().orc_argsort(DTYPES[dt], _ptr(a), _ptr(idx), a.size)
    return idx


def sort_pairs(keys: np.ndarray, vals: np.ndarray, dt: str):
    """Stable sort of (key, u32 value) pairs by key; returns new arrays."""
    k = np.array(keys, dtype=NP_DTYPE[dt], copy=True, order="C")
    v = np.array(vals, dtype=np.uint32, copy=True, order="C")
    lib().orc_sort_pairs(DTYPES[dt], _ptr(k), _ptr(v), k.size)
    return k, v


def par_argsort(a: np.ndarray, dt: str, threads: int = 0) -> np.ndarray:
    """argsort() on every host thread: sorts (ordered key, index) tuples, so
    the result is the same stable permutation."""
    a = np.ascontiguousarray(a, dtype=NP_DTYPE[dt])
    idx = np.empty(a.size, np.uint32)
    lib().orc_par_argsort(DTYPES[dt], _ptr(a), _ptr(idx), a.size, threads)
    return idx


def par_sort_pairs(keys: np.ndarray, vals: np.ndarray, dt: str, threads: int = 0):
    """sort_pairs() on every host thread (same stable result)."""
    k = np.array(keys, dtype=NP_DTYPE[dt], copy=True, order="C")
    v = np.array(vals, dtype=np.uint32, copy=True, order="C")
    lib().orc_par_sort_pairs(DTYPES[dt], _ptr(k), _ptr(v), k.size, threads)
    return k, v


def radix_sort_pairs(keys: np.ndarray, vals: np.ndarray, dt: str):
    k = np.array(keys, dtype=NP_DTYPE[dt], copy=True, order="C")
    v = np.array(vals, dtype=np.uint32, copy=True, order="C")
    lib().orc_radix_sort(DTYPES[dt], _ptr(k), _ptr(v), k.size)
    return k, v


def max_threads() -> int:
    return int(lib().orc_max_threads())


def to_ordered(x: int, dt: str) -> int:
    L, mode = lib(), DTYPES[dt] % 3
    return int(L.orc_to_ordered64(x, mode) if DTYPES[dt] >= 3 else L.orc_to_ordered32(x, mode))


def from_ordered(y: int, dt: str) -> int:
    L, mode = lib(), DTYPES[dt] % 3
    return int(L.orc_from_ordered64(y, mode) if DTYPES[dt] >= 3 else L.orc_from_ordered32(y, mode))
