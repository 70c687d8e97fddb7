"""Performance floors, the B200 counterpart of forge-sort's CI perf gate
(tests/performance.rs:17-207): 16M keys, one warm-up then the median of 10
timed calls, Mkeys/s against a floor.

Two tiers:
  - host-slice calls (sort_u32(&mut [u32]) and kin, host memory in and out,
    the copies inside the timed call): the reference's own floors, which it
    sets for its M4 Pro GPU -- a drop-in must not be slower than them;
  - device-resident sorts (keys already in HBM, CUDA events on the sorter's
    stream): B200 floors at about two thirds of what this build measured on
    one B200, so a regression in the chained launches or the scatter fails.
Inputs: the reference draws uniform values from a seeded ChaCha RNG
(`rand_chacha`, absent here); the seeded xorshift stream stands in, with the
reference's value ranges (f32/f64 uniform in [-1000, 1000))."""
import time

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

N = 16_000_000


def _median(ts):
    ts = sorted(ts)
    return ts[len(ts) // 2]


def _data(kind, seed):
    if kind in ("u32", "i32", "u64", "i64"):
        return orc.gen(kind, N, seed=seed)
    u = orc.gen("u64", N, seed=seed).astype(np.float64) / 2.0 ** 64  # uniform [0, 1)
    x = u * 2000.0 - 1000.0
    return x.astype(np.float32) if kind == "f32" else x


# (name, call, reference floor Mk/s at performance.rs line)
HOST_CASES = [
    ("sort_u32", "u32", 2000.0),        # performance.rs:37
    ("sort_i32", "i32", 1900.0),        # :60
    ("sort_f32", "f32", 500.0),         # :83
    ("argsort_u32", "u32", 750.0),      # :107
    ("sort_pairs_f32", "f32", 250.0),   # :136
    ("sort_u64", "u64", 600.0),         # :161
    ("sort_i64", "i64", 550.0),         # :184
    ("sort_f64", "f64", 100.0),         # :207
]


@pytest.mark.parametrize("name,dt,floor", HOST_CASES, ids=[c[0] for c in HOST_CASES])
def test_host_slice_floor(sorter, name, dt, floor):
    x = _data(dt, 42)
    v = orc.gen("u32", N, seed=7)

    def call():
        if name.startswith("argsort"):
            getattr(sorter, name)(x)
        elif name.startswith("sort_pairs"):
            getattr(sorter, name)(x.copy(), v.copy())
        else:
            getattr(sorter, name)(x.copy())

    call()
    ts = []
    for _ in range(10):
        a = x.copy()
        vv = v.copy()
        t0 = time.perf_counter()
        if name.startswith("argsort"):
            getattr(sorter, name)(a)
        elif name.startswith("sort_pairs"):
            getattr(sorter, name)(a, vv)
        else:
            getattr(sorter, name)(a)
        ts.append(time.perf_counter() - t0)
    mks = N / _median(ts) / 1e6
    print(f"{name} host slice 16M: {mks:.0f} Mk/s ({_median(ts) * 1e3:.2f} ms)")
    assert mks >= floor, f"{name}: {mks:.0f} Mk/s < {floor:.0f}"


# device-resident: (op, dtype, floor Mk/s on one B200)
DEVICE_CASES = [  # measured on one B200 (16M keys): keys u32 42.3, u64 16.1, argsort 30.3, pairs u32 29.5 / u64 9.9 Gk/s
    ("keys", "u32", 28000.0),
    ("keys", "i32", 28000.0),
    ("keys", "f32", 28000.0),
    ("keys", "u64", 10500.0),
    ("keys", "i64", 10500.0),
    ("keys", "f64", 10500.0),
    ("argsort", "u32", 20000.0),
    ("argsort", "f32", 20000.0),
    ("pairs", "u32", 19500.0),
    ("pairs", "u64", 6500.0),
]


@pytest.mark.parametrize("op,dt,floor", DEVICE_CASES, ids=[f"{o}_{d}" for o, d, _ in DEVICE_CASES])
def test_device_resident_floor(sorter, op, dt, floor):
    import torch
    kb = 8 if dt in ("u64", "i64", "f64") else 4
    x = _data(dt, 42)
    kin = torch.from_numpy(np.ascontiguousarray(x).view(np.int32 if kb == 4 else np.int64)).cuda()
    kout = torch.empty_like(kin)
    vin = torch.arange(N, dtype=torch.int32, device="cuda")
    vout = torch.empty_like(vin)
    stream = torch.cuda.Stream()
    sorter.set_stream(stream)

    def call():
        if op == "keys":
            sorter.sort_device_copy(dt, kin.data_ptr(), kout.data_ptr(), N, sync=False)
        elif op == "argsort":
            sorter.argsort_device(dt, kin.data_ptr(), vout.data_ptr(), N, sync=False)
        else:
            sorter.sort_pairs_device_copy(dt, kin.data_ptr(), vin.data_ptr(), kout.data_ptr(), vout.data_ptr(), N,
                                          sync=False)

    try:
        with torch.cuda.stream(stream):
            for _ in range(3):
                call()
            sorter.synchronize()
            ts = []
            for _ in range(10):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                call()
                e1.record(stream)
                e1.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e-3)
            sorter.synchronize()
    finally:
        sorter.set_stream(None)
    mks = N / _median(ts) / 1e6
    print(f"{op} {dt} device 16M: {mks:.0f} Mk/s ({_median(ts) * 1e3:.3f} ms)")
    assert mks >= floor, f"{op} {dt}: {mks:.0f} Mk/s < {floor:.0f}"
