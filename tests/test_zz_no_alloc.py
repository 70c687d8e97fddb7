"""GPU test of fs_sort_keys_noalloc, the entry point that allocates nothing.

Some callers cannot allocate device memory when they sort: code running
under a fixed memory budget, or under a caching allocator that owns all
device memory, and plugins whose host runtime forbids allocation at call
time.  fs_sort_keys_noalloc serves them from one fixed device array inside
the library (4 MiB of keys: 2^20 four-byte or 2^19 eight-byte keys).

Checked through the C ABI, for all six key types at the size limit and one
below it:
  - the result is bit-exact against the CPU oracle's sort and against the
    ordinary entry point (fs_sort_keys, which grows its own scratch);
  - two calls in a row of the same type on fresh data both come out right
    (the shared array keeps the previous call's contents);
  - sizes beyond the limit are refused with a clear error.
The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LIMIT_BYTES = 4 << 20  # the fixed scratch covers 4 MiB of keys

CASES = [("u32", "u32"), ("i32", "i32"), ("f32", "f32_mix"), ("u64", "u64"), ("i64", "i64"), ("f64", "f64_logu")]


def _noalloc(lib, dtype_code, tensor, stream):
    return lib.fs_sort_keys_noalloc(dtype_code, ctypes.c_void_p(tensor.data_ptr()), tensor.numel(),
                                    ctypes.c_void_p(stream.cuda_stream))


@pytest.mark.parametrize("dt,dist", CASES, ids=[d for d, _ in CASES])
def test_noalloc_matches_oracle_and_allocating_entry_point(dt, dist):
    import torch
    from forge_sort import GpuSorter, _lib

    lib = _lib.load()
    code = orc.DTYPES[dt]
    kb = 8 if code >= 3 else 4
    bits = orc.BITS_DTYPE[dt]
    sdt = np.int32 if kb == 4 else np.int64
    limit = LIMIT_BYTES // kb
    stream = torch.cuda.Stream()
    sorter = GpuSorter.with_context(0, stream)
    try:
        # limit, then limit - 1, then limit again on fresh data: consecutive
        # calls of the same type over the one shared array
        for call, n in enumerate([limit, limit - 1, limit]):
            host = np.ascontiguousarray(orc.gen(dist, n, seed=500 + 31 * call)).view(bits)
            a = torch.from_numpy(host.view(sdt)).to("cuda")
            b = a.clone()
            torch.cuda.synchronize()
            rc = _noalloc(lib, code, a, stream)
            assert rc == _lib.OK, lib.fs_last_error(None).decode()
            sorter.sort_device(dt, b.data_ptr(), n, sync=True)
            got = a.cpu().numpy().view(bits)
            want = orc.par_sort_keys(host.view(orc.NP_DTYPE[dt]), dt).view(bits)
            assert np.array_equal(got, want), f"call {call}, n={n}: differs from the oracle"
            assert np.array_equal(got, b.cpu().numpy().view(bits)), f"call {call}: differs from fs_sort_keys"
    finally:
        sorter.close()


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch():
    import torch
    from forge_sort import _lib

    lib = _lib.load()
    stream = torch.cuda.Stream()
    too_big = torch.zeros(LIMIT_BYTES // 4 + 1, dtype=torch.int32, device="cuda")
    rc = _noalloc(lib, _lib.U32, too_big, stream)
    assert rc == _lib.E_INVALID
    assert "allocation-free limit" in lib.fs_last_error(None).decode()
    too_big64 = torch.zeros(LIMIT_BYTES // 8 + 1, dtype=torch.int64, device="cuda")
    assert _noalloc(lib, _lib.F64, too_big64, stream) == _lib.E_INVALID
    assert _noalloc(lib, _lib.U32, too_big[:1], stream) == _lib.OK  # n <= 1: nothing to do
    # a size so large that n * key bytes wraps 64 bits still gets the limit error
    rc = lib.fs_sort_keys_noalloc(_lib.U64, ctypes.c_void_p(too_big.data_ptr()), (1 << 61) + 1,
                                  ctypes.c_void_p(stream.cuda_stream))
    assert rc == _lib.E_INVALID and "allocation-free limit" in lib.fs_last_error(None).decode()
