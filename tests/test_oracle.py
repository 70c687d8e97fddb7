"""CPU tests of the oracle itself: pinned against the reference's known-answer
vectors (tests/golden/known_answers.json), against an independent pure-Python
restatement of Rust's sort / total_cmp, and its two algorithms (comparison
sort, LSD radix) against each other.  No GPU."""
import json
import os

import numpy as np
import pytest

import _cases
from oracle import oracle as orc

CASES = _cases.load()["cases"]
INPUTS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "inputs.json")


@pytest.mark.parametrize("c", CASES, ids=[c["id"] for c in CASES])
def test_oracle_matches_known_answers(c):
    dt = c["dtype"]
    x = _cases.case_input(c)
    keys, idx, vals = _cases.expected(c)
    if c["op"] == "sort":
        got = orc.sort_keys(x, dt)
        assert _cases.as_bits(got, dt) == keys
        assert _cases.as_bits(orc.radix_sort_keys(x, dt), dt) == keys
    elif c["op"] == "argsort":
        assert [int(i) for i in orc.argsort(x, dt)] == idx
    else:
        k, v = orc.sort_pairs(x, _cases.case_values(c), dt)
        assert _cases.as_bits(k, dt) == keys
        assert [int(t) for t in v] == vals
        k2, v2 = orc.radix_sort_pairs(x, _cases.case_values(c), dt)
        assert _cases.as_bits(k2, dt) == keys and [int(t) for t in v2] == vals


def test_xorshift_jump_ahead_matches_sequential():
    # element i = state after i+1 Marsaglia steps from the seed
    x, seq = 42, []
    for _ in range(300):
        x ^= (x << 13) & (2**64 - 1)
        x ^= x >> 7
        x ^= (x << 17) & (2**64 - 1)
        seq.append(x)
    assert [int(v) for v in orc.gen("u64", 300)] == seq
    assert [int(v) for v in orc.gen("u64", 100, start=200)] == seq[200:]
    assert [int(v) for v in orc.gen("u32", 300)] == [v >> 32 for v in seq]


@pytest.mark.parametrize("dt,dist", [("u32", "u32"), ("i32", "i32"), ("f32", "f32_mix"),
                                     ("u64", "u64"), ("i64", "i64"), ("f64", "f64_logu"),
                                     ("u32", "zipf_u32"), ("u32", "skew_u32")])
def test_radix_restatement_agrees_with_comparison_sort(dt, dist):
    x = orc.gen(dist, 200_003, seed=7)
    a = orc.sort_keys(x, dt)
    assert np.array_equal(a.view(orc.BITS_DTYPE[dt]), orc.radix_sort_keys(x, dt).view(orc.BITS_DTYPE[dt]))
    assert np.array_equal(a.view(orc.BITS_DTYPE[dt]), orc.par_sort_keys(x, dt).view(orc.BITS_DTYPE[dt]))
    v = np.arange(x.size, dtype=np.uint32)
    k1, v1 = orc.sort_pairs(x, v, dt)
    k2, v2 = orc.radix_sort_pairs(x, v, dt)
    assert np.array_equal(v1, v2)
    assert np.array_equal(orc.argsort(x, dt), v1)
    # the parallel stable forms (full-size GPU checks use them) agree too
    assert np.array_equal(orc.par_argsort(x, dt), v1)
    k3, v3 = orc.par_sort_pairs(x, v, dt)
    assert np.array_equal(v3, v1)
    assert np.array_equal(k3.view(orc.BITS_DTYPE[dt]), k1.view(orc.BITS_DTYPE[dt]))


@pytest.mark.parametrize("dt,dist", [("f32", "f32_mix"), ("f64", "f64_logu"), ("i32", "i32"), ("i64", "i64")])
def test_oracle_order_is_total_cmp(dt, dist):
    x = orc.gen(dist, 5000, seed=3)
    got = _cases.as_bits(orc.sort_keys(x, dt), dt)
    bits = _cases.as_bits(x, dt)
    assert got == sorted(bits, key=_cases.order_key(dt))


def test_transforms_round_trip_and_order():
    # FloatFlip round trips (reference tests correctness_f32.rs:214-238, f64:183-207)
    for dt, vals in (("f32", [0, 0x80000000, 0x3F800000, 0xBF800000, 0x7F800000, 0xFF800000,
                              0x7FC00000, 0xFFC00000, 0x00000001, 0x80000001]),
                     ("f64", [0, 1 << 63, 0x3FF0000000000000, 0xFFF8000000000000, 1, (1 << 63) | 1])):
        for v in vals:
            assert orc.from_ordered(orc.to_ordered(v, dt), dt) == v
    assert orc.to_ordered(0x80000000, "i32") == 0  # i32::MIN -> smallest
    assert orc.to_ordered(0xFFFFFFFF, "f32") == 0  # most negative NaN -> smallest


def test_generated_input_checksums_are_pinned():
    """FNV-1a 64 of the seeded inputs and of the oracle's outputs, recorded by
    tests/golden/make_golden.py; guards the generators and the oracle against
    silent drift."""
    with open(INPUTS) as f:
        rec = json.load(f)
    for r in rec["inputs"]:
        x = orc.gen(r["dist"], r["n"], seed=r["seed"])
        assert orc.fnv1a64(x) == int(r["fnv1a64"], 16), r
        s = orc.sort_keys(x, r["dtype"])
        assert orc.fnv1a64(s) == int(r["sorted_fnv1a64"], 16), r
