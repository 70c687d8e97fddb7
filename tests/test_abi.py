"""CPU tests of the C-ABI boundary and the host-side API mirror: the library
loads and exports every symbol include/*.h declares, error strings and
SortKey constants match the reference, and the no-device error path."""
import ctypes
import glob
import os
import re

import pytest

import _cases
import forge_sort
from forge_sort import _lib
from forge_sort.errors import DeviceNotFound, GpuExecution, LengthMismatch, ShaderCompilation

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols(header):
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fs_[a-z0-9_]+)\s*\(", text)))


HEADERS = {"forgesort.h": "SIGNATURES", "forgesort_bench.h": "BENCH_SIGNATURES"}


@pytest.mark.parametrize("header", sorted(HEADERS))
def test_library_exports_every_declared_symbol(header):
    L = _lib.load()
    syms = declared_symbols(os.path.join(ROOT, "include", header))
    assert syms
    for s in syms:
        assert hasattr(L, s), f"{s} declared in {header} but not exported"
    # the ctypes signature table covers exactly the declared surface
    assert sorted(getattr(_lib, HEADERS[header])) == syms


def test_every_header_is_covered():
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        assert os.path.basename(h) in HEADERS, h


def test_abi_version():
    assert _lib.load().fs_abi_version() == 1


def test_sort_error_display_strings():
    e = _cases.load()["errors"]
    assert str(DeviceNotFound()) == e["device_not_found"]
    assert str(ShaderCompilation("test")) == e["shader_compilation_test"]
    assert str(GpuExecution("timeout")) == e["gpu_execution_timeout"]
    assert str(LengthMismatch(10, 5)) == e["length_mismatch_10_5"]
    lm = LengthMismatch(**e["length_mismatch_fields"])
    assert (lm.keys, lm.values) == (3, 2)


def test_sort_key_constants():
    consts = _cases.load()["sort_key_consts"]
    for dt in ("u32", "i32", "f32", "u64", "i64", "f64"):
        assert list(forge_sort.SORT_KEY[dt]) == consts[dt]


def test_dtype_name_rejects_non_sort_keys():
    import numpy as np
    assert forge_sort.dtype_name(np.float32) == "f32"
    assert forge_sort.dtype_name("u64") == "u64"
    for bad in (np.int16, np.uint8, "str", object):
        with pytest.raises(TypeError):
            forge_sort.dtype_name(bad)


def _has_cuda():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_cuda(), reason="checks the no-device path")
def test_no_device_maps_to_device_not_found():
    with pytest.raises(DeviceNotFound) as ei:
        forge_sort.GpuSorter.new()
    assert str(ei.value) == "no Metal GPU device found"
    # the C layer reports the reason text without a sorter handle
    assert _lib.load().fs_last_error(None).decode() == "no CUDA device"


def test_null_arguments_are_rejected_without_a_device():
    L = _lib.load()
    assert L.fs_create(0, None, None) == _lib.E_INVALID
    assert L.fs_sort_keys(None, 0, None, 10, 1) == _lib.E_INVALID
    assert L.fs_destroy(None) == _lib.OK
    assert L.fs_scratch_bytes(None) == 0


def test_stream_handles():
    """None and 0 select the sorter's own stream (NULL in the C ABI); a
    stream object reporting handle 0 (torch's default stream) is the legacy
    default stream, cudaStreamLegacy = 1; other handles pass through."""
    from forge_sort.sorter import _stream_handle

    class S:
        def __init__(self, h):
            self.cuda_stream = h

    assert _stream_handle(None) is None
    assert _stream_handle(0) is None
    assert _stream_handle(0x1234) == 0x1234
    assert _stream_handle(S(0)) == 1
    assert _stream_handle(S(0x5678)) == 0x5678
    with pytest.raises(TypeError):
        _stream_handle(object())
