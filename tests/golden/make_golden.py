"""Regenerate tests/golden/inputs.json: FNV-1a-64 checksums of the seeded
synthetic inputs (oracle generators) and of their oracle-sorted outputs.

    python tests/golden/make_golden.py

known_answers.json is NOT generated: it is transcribed by hand from the
reference's tests (file:line in each case)."""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as orc  # noqa: E402

SPECS = [
    ("u32", "u32", 1 << 20, 42),      # config D1
    ("u32", "u32", 1 << 16, 42),
    ("i32", "i32", 1 << 16, 42),
    ("f32", "f32_mix", 1 << 16, 42),
    ("u64", "u64", 1 << 16, 42),
    ("i64", "i64", 1 << 16, 42),
    ("f64", "f64_logu", 1 << 16, 42),
    ("u32", "zipf_u32", 1 << 16, 42),
    ("u32", "skew_u32", 1 << 16, 42),
]


def main():
    out = {"about": __doc__.strip().splitlines()[0], "inputs": []}
    for dt, dist, n, seed in SPECS:
        x = orc.gen(dist, n, seed=seed)
        s = orc.sort_keys(x, dt)
        out["inputs"].append({"dtype": dt, "dist": dist, "n": n, "seed": seed,
                              "fnv1a64": f"{orc.fnv1a64(x):016x}",
                              "sorted_fnv1a64": f"{orc.fnv1a64(s):016x}"})
    with open(os.path.join(HERE, "inputs.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
