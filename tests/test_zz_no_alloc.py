"""GPU test of fs_sort_keys_noalloc, the entry point that allocates nothing.

Some callers cannot allocate device memory when they sort: code running
under a fixed memory budget, or under a caching allocator that owns all
device memory, and plugins whose host runtime forbids allocation at call
time.  fs_sort_keys_noalloc serves them from one fixed device array inside
the library.  This file checks, through the C ABI, that it returns exactly
what the ordinary entry point (fs_sort_keys, which grows its own scratch)
returns, on two calls in a row, and that it refuses sizes beyond its fixed
limit.  The file name sorts last so that a run stopping at the first failure
has already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIMIT_BYTES = 4 << 20  # the fixed scratch covers 4 MiB of keys


def _noalloc(lib, dtype_code, tensor, stream):
    return lib.fs_sort_keys_noalloc(dtype_code, ctypes.c_void_p(tensor.data_ptr()), tensor.numel(),
                                    ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_matches_allocating_entry_point_twice():
    import torch
    from forge_sort import GpuSorter, _lib
    from oracle import oracle as orc

    lib = _lib.load()
    stream = torch.cuda.Stream()
    sorter = GpuSorter.with_context(0, stream)
    cases = [  # (fs dtype, oracle distribution, numpy bits dtype, torch dtype, n)
        (_lib.U32, "u32", np.uint32, torch.int32, (1 << 20) - 3),
        (_lib.F64, "f64_logu", np.uint64, torch.int64, 300_001),
    ]
    for code, dist, bits, tdt, n in cases:
        host = np.ascontiguousarray(orc.gen(dist, n, seed=77 + n)).view(bits)
        a = torch.from_numpy(host.view(np.int32 if bits is np.uint32 else np.int64)).to("cuda")
        b = a.clone()
        torch.cuda.synchronize()
        rc = _noalloc(lib, code, a, stream)
        assert rc == _lib.OK, lib.fs_last_error(None).decode()
        name = {_lib.U32: "u32", _lib.F64: "f64"}[code]
        sorter.sort_device(name, b.data_ptr(), n, sync=True)
        got = a.cpu().numpy().view(bits)
        want = b.cpu().numpy().view(bits)
        assert np.array_equal(got, want)  # bit-exact: integer / bit-pattern work
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
    assert _noalloc(lib, _lib.U32, too_big[:1], stream) == _lib.OK  # n <= 1: nothing to do
