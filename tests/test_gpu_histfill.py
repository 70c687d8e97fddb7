"""Parity of the histogram-fill form of keys-only 32-bit sorts with the CPU
oracle (bit-exact).

Keys-only u32 / i32 / f32 sorts of many keys run the radix passes of the top
two digits only, which group the keys by their top 16 bits, and then sort
every group by counting its low 16 bits (csrc/fs_histfill.cuh).  The sorters
here lower the size at which that form starts (FORGESORT_H16_MIN_KEYS) and
switch the single-launch form off, so modest inputs reach every branch:
  - groups of 0, 1, a few and up to 126975 keys (one CTA each), and larger
    groups spread over CTAs, including one group holding every key;
  - a low value seen 2^16 times or more inside a one-CTA group (the counter
    field wraps and is repaired), on an even and on an odd value;
  - 0, 1 and 2 executed passes (top byte constant, second byte constant,
    top 16 bits constant), in place and out of place;
  - all keys equal, IEEE specials and NaN payloads, signed extremes.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def hsorter():
    from forge_sort import GpuSorter

    saved = {k: os.environ.get(k) for k in ("FORGESORT_H16_MIN_KEYS", "FORGESORT_COOP_MAX_BYTES")}
    os.environ["FORGESORT_H16_MIN_KEYS"] = "4096"
    os.environ["FORGESORT_COOP_MAX_BYTES"] = "0"
    try:
        s = GpuSorter.new()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    yield s
    s.close()


def bits(a, dt):
    return np.ascontiguousarray(a).view(orc.BITS_DTYPE[dt])


def check_both(sorter, x, dt):
    """In place through the host-slice call, and out of place on the device
    (the input must stay untouched)."""
    import torch

    want = bits(orc.par_sort_keys(x, dt), dt)
    a = x.copy()
    getattr(sorter, f"sort_{dt}")(a)
    assert np.array_equal(bits(a, dt), want), "in place"
    src = torch.from_numpy(bits(x, dt).view(np.int32).copy()).to("cuda")
    dst = torch.empty_like(src)
    torch.cuda.synchronize()
    sorter.sort_device_copy(dt, src.data_ptr(), dst.data_ptr(), x.size, sync=True)
    assert np.array_equal(dst.cpu().numpy().view(np.uint32), want), "out of place"
    assert np.array_equal(src.cpu().numpy().view(np.uint32), bits(x, dt)), "input changed"


@pytest.mark.parametrize("n", [4096, 100_003, 1_000_003, 3 << 20])
@pytest.mark.parametrize("dt,dist", [("u32", "u32"), ("i32", "i32"), ("f32", "f32_mix")])
def test_histfill_uniform_and_ieee(hsorter, dt, dist, n):
    check_both(hsorter, orc.gen(dist, n, seed=41 + n), dt)


@pytest.mark.parametrize("mask,name", [(0x00FFFFFF, "top byte constant: one pass"),
                                       (0xFF00FFFF, "second byte constant: one pass"),
                                       (0x0000FFFF, "top 16 bits constant: no pass, one group")])
@pytest.mark.parametrize("n", [150_001, 2_000_000])
def test_histfill_executed_passes(hsorter, mask, name, n):
    x = orc.gen("u32", n, seed=7) & np.uint32(mask)
    check_both(hsorter, x, "u32")


def test_histfill_zipf_one_large_group(hsorter):
    check_both(hsorter, orc.gen("zipf_u32", 1_500_000, seed=3), "u32")


def test_histfill_skewed(hsorter):
    check_both(hsorter, orc.gen("skew_u32", 4_000_000, seed=11), "u32")


@pytest.mark.parametrize("even_first", [True, False])
def test_histfill_counter_wrap_in_one_cta_group(hsorter, even_first):
    # one group of 120,000 keys (<= 126975): 66,000 of one low value and
    # 54,000 of its neighbour sharing the same counter word, plus scattered
    # keys elsewhere
    a, b = (0x12345678, 0x12345679) if even_first else (0x12345679, 0x12345678)
    rng = np.random.default_rng(5)
    x = np.concatenate([np.full(66_000, a, np.uint32), np.full(54_000, b, np.uint32),
                        rng.integers(0, 1 << 32, 30_000, dtype=np.uint64).astype(np.uint32)])
    rng.shuffle(x)
    check_both(hsorter, x, "u32")


@pytest.mark.parametrize("size", [126_975, 126_976, 2 * 61_440, 2 * 61_440 + 1, 400_000])
def test_histfill_group_size_edges(hsorter, size):
    # one group of exactly `size` keys with uniform low 16 bits, among small ones
    rng = np.random.default_rng(size)
    big = (np.uint32(0xABCD0000) | rng.integers(0, 1 << 16, size, dtype=np.uint32)).astype(np.uint32)
    rest = rng.integers(0, 1 << 32, 50_000, dtype=np.uint64).astype(np.uint32)
    rest = rest[(rest >> 16) != 0xABCD]
    x = np.concatenate([big, rest])
    rng.shuffle(x)
    check_both(hsorter, x, "u32")


def test_histfill_large_group_of_one_value_and_neighbours(hsorter):
    # a large group whose keys are nearly all one value (runs far longer than
    # a chunk) with a few neighbours on both sides
    x = np.concatenate([np.full(300_000, 0x40000010, np.uint32), np.arange(0x40000000, 0x40000020, dtype=np.uint32),
                        np.full(70_000, 0x4000FFFF, np.uint32)])
    np.random.default_rng(2).shuffle(x)
    check_both(hsorter, x, "u32")


def test_histfill_one_key_groups(hsorter):
    # 65536 groups of exactly one key
    rng = np.random.default_rng(9)
    x = ((np.arange(1 << 16, dtype=np.uint32) << 16) | rng.integers(0, 1 << 16, 1 << 16, dtype=np.uint32)).astype(
        np.uint32)
    rng.shuffle(x)
    check_both(hsorter, x, "u32")


def test_histfill_all_equal(hsorter):
    check_both(hsorter, np.full(200_000, 0xDEADBEEF, np.uint32), "u32")
    check_both(hsorter, np.full(200_000, -0.0, np.float32), "f32")


def test_histfill_ieee_specials_and_nan_payloads(hsorter):
    rng = np.random.default_rng(13)
    specials = np.array([0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001,
                         0xFF800001, 0x7FFFFFFF, 0xFFFFFFFF, 0x00000001, 0x80000001, 0x007FFFFF, 0x807FFFFF],
                        np.uint32)
    x = np.concatenate([rng.choice(specials, 300_000), orc.gen("f32_mix", 300_000, seed=4).view(np.uint32)])
    rng.shuffle(x)
    check_both(hsorter, x.view(np.float32), "f32")


def test_histfill_signed_extremes(hsorter):
    rng = np.random.default_rng(17)
    ext = np.array([-(1 << 31), (1 << 31) - 1, -1, 0, 1], np.int32)
    x = np.concatenate([rng.choice(ext, 200_000), orc.gen("i32", 200_000, seed=8)])
    rng.shuffle(x)
    check_both(hsorter, x, "i32")


def test_histfill_repeat_calls_reuse_scratch(hsorter):
    # the scratch (group table, pool) keeps the previous call's contents
    for seed, dist in [(1, "zipf_u32"), (2, "u32"), (3, "skew_u32"), (4, "u32")]:
        check_both(hsorter, orc.gen(dist, 700_001, seed=seed), "u32")


def test_histfill_2e27_generated_on_device(hsorter):
    """A 2^27-key u32 sort in the histogram-fill form (15 launches) matches
    the oracle."""
    import torch

    from forge_sort import _lib

    n = 1 << 27
    L = _lib.load()
    x = torch.empty(n, dtype=torch.int32, device="cuda")
    assert L.fs_generate(_lib.GEN_U32, 42, 0, n, x.data_ptr(), 0) == 0
    torch.cuda.synchronize()
    host = x.cpu().numpy().view(np.uint32).copy()
    y = torch.empty_like(x)
    hsorter.sort_device_copy("u32", x.data_ptr(), y.data_ptr(), n, sync=True)
    assert hsorter.last_launch_count() == 15
    assert np.array_equal(y.cpu().numpy().view(np.uint32), orc.par_sort_keys(host, "u32"))
