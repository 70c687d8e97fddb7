"""The Rust crate (gpu-forge_b200/rust/forge-sort) cannot be compiled on this
image (no cargo / rustc).  These CPU checks keep its source consistent with
the C ABI it binds: every `extern "C"` function in src/ffi.rs is declared in
include/*.h and exported by libforgesort.so, and the SortKey constants and
SortError strings in src/lib.rs are the reference's (src/lib.rs:29-104)."""
import os
import re

import _cases
from forge_sort import _lib
from forge_sort.sorter import SORT_KEY

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CRATE = os.path.join(ROOT, "gpu-forge_b200", "rust", "forge-sort")


def _header_symbols():
    syms = set()
    for h in ("forgesort.h", "forgesort_bench.h"):
        text = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", h)).read(), flags=re.S)
        syms |= set(re.findall(r"\b(fs_[a-z0-9_]+)\s*\(", text))
    return syms


def test_ffi_functions_are_declared_and_exported():
    ffi = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    fns = re.findall(r"pub fn (fs_[a-z0-9_]+)\s*\(", ffi)
    assert len(fns) > 40
    declared = _header_symbols()
    L = _lib.load()
    for f in fns:
        assert f in declared, f"{f} bound in ffi.rs but not declared in include/*.h"
        assert hasattr(L, f), f"{f} bound in ffi.rs but not exported"


def test_sort_key_constants_and_error_strings():
    lib = open(os.path.join(CRATE, "src", "lib.rs")).read()
    rows = re.findall(r"sort_key!\((\w+), ffi::FS_\w+, (\d), (\w+), (\w+), (\d), (\d)\);", lib)
    got = {t: (int(a), b == "true", c == "true", int(d), int(e)) for t, a, b, c, d, e in rows}
    assert got == SORT_KEY
    e = _cases.load()["errors"]
    for s in (e["device_not_found"], "shader compilation failed: {m}", "GPU execution failed: {m}",
              "length mismatch: keys={keys}, values={values}"):
        assert s in lib, s


def test_crate_layout_and_label():
    for f in ("Cargo.toml", "build.rs", "src/ffi.rs", "src/lib.rs"):
        text = open(os.path.join(CRATE, f)).read()
        assert "NOT COMPILED" in text, f
