"""Materialise tests/golden/known_answers.json cases, and an independent
pure-Python restatement of the orders the reference's tests use:
Rust `sort()` (integers) and `sort_by(total_cmp)` (floats; the published
algorithm of core::f32::total_cmp: flip the non-sign bits of negative values,
compare as signed integers)."""
from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "known_answers.json")
NP = {"u32": np.uint32, "i32": np.int32, "f32": np.float32,
      "u64": np.uint64, "i64": np.int64, "f64": np.float64}
BITS = {"f32": np.uint32, "f64": np.uint64}
WIDTH = {"u32": 32, "i32": 32, "f32": 32, "u64": 64, "i64": 64, "f64": 64}


def load():
    with open(GOLDEN) as f:
        return json.load(f)


def total_cmp_key(bits: int, width: int) -> int:
    sign = (bits >> (width - 1)) & 1
    s = bits ^ (sign * ((1 << (width - 1)) - 1))
    return s - (1 << width) if s >> (width - 1) else s


def order_key(dt: str):
    """Key function on the *bit pattern* (for floats) or value (ints)."""
    if dt in ("f32", "f64"):
        w = WIDTH[dt]
        return lambda b: total_cmp_key(int(b), w)
    return lambda v: int(v)


def _gen(name: str):
    if name == "f32_nan_variants":
        return [0x7FC00000 | i for i in range(1, 11)] + [0xFFC00000 | i for i in range(1, 11)]
    if name == "f32_denormals":
        return ([i for i in range(1, 101)] + [0x80000000 | i for i in range(1, 101)]
                + [0x00000000, 0x80000000, 0x00800000, 0x80800000])
    if name == "f64_nan_variants":
        return ([0x7FF8000000000000 | i for i in range(1, 11)]
                + [0xFFF8000000000000 | i for i in range(1, 11)])
    if name == "f64_per_byte":
        return [v << (8 * b) for b in range(8) for v in (0x01, 0x80, 0xFF)]
    if name == "u64_byte_boundary":
        return [0xFF << (8 * b) for b in range(8)] + [0x01 << (8 * b) for b in range(8)] + [0, 2**64 - 1]
    if name == "u64_powers_of_two":
        return [1 << i for i in range(64)] + [0, 2**64 - 1]
    if name == "i64_sign_boundary":
        return list(range(-1000, 1001)) + [-(2**63), 2**63 - 1]
    if name == "lcg_1000":
        rng, out = 42, []
        for _ in range(1000):
            rng = (rng * 6364136223846793005 + 1442695040888963407) % 2**64
            out.append(rng >> 33)
        return out
    raise KeyError(name)


def case_input(c) -> np.ndarray:
    dt = c["dtype"]
    if "input_fill" in c:
        return np.full(c["input_fill"]["n"], c["input_fill"]["value"], NP[dt])
    if "input_bits" in c:
        return np.array([int(b, 16) for b in c["input_bits"]], BITS[dt]).view(NP[dt])
    if "input_gen" in c:
        vals = _gen(c["input_gen"])
        if dt in BITS:
            return np.array(vals, BITS[dt]).view(NP[dt])
        return np.array(vals, NP[dt])
    return np.array(c["input"], NP[dt])


def as_bits(a: np.ndarray, dt: str):
    if dt in BITS:
        return [int(x) for x in np.ascontiguousarray(a).view(BITS[dt])]
    return [int(x) for x in a]


def case_values(c):
    if "values_iota" in c:
        return np.arange(c["values_iota"], dtype=np.uint32)
    return np.array(c["values"], np.uint32)


def expected(c):
    """(expected keys as bit-ints/ints, expected argsort idx, expected values)."""
    dt = c["dtype"]
    x = case_input(c)
    bits = as_bits(x, dt)
    key = order_key(dt)
    perm = sorted(range(len(bits)), key=lambda i: key(bits[i]))  # stable
    if "expected_bits" in c:
        keys = [int(b, 16) for b in c["expected_bits"]]
    elif "expected" in c and c["op"] != "argsort":
        keys = [int(v) for v in c["expected"]]
    else:
        keys = [bits[i] for i in perm]
    idx = c.get("expected") if c["op"] == "argsort" else None
    if c.get("expected_iota"):
        idx = list(range(c["expected_iota"]))
    if idx is None:
        idx = perm
    vals = None
    if c["op"] == "pairs":
        if "expected_values" in c:
            vals = c["expected_values"]
        elif c.get("expected_values_iota"):
            vals = list(range(c["expected_values_iota"]))
        else:
            v = case_values(c)
            vals = [int(v[i]) for i in perm]
    return keys, list(idx), vals
