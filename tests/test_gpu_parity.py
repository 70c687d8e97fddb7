"""Parity of the CUDA path with the CPU oracle on seeded inputs: every key
type, argsort and pairs, sizes around the tile edges, skewed and degenerate
distributions.  Bit-exact (integer and bit-pattern work)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

DT_DIST = [("u32", "u32"), ("i32", "i32"), ("f32", "f32_mix"),
           ("u64", "u64"), ("i64", "i64"), ("f64", "f64_logu")]
SIZES = [2, 3, 31, 32, 33, 1000, 4095, 4096, 4097, 8192 + 17, 65536, 100_003, 1 << 20]


def bits(a, dt):
    return np.ascontiguousarray(a).view(orc.BITS_DTYPE[dt])


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("dt,dist", DT_DIST, ids=[d for d, _ in DT_DIST])
def test_sort_keys(sorter, dt, dist, n):
    x = orc.gen(dist, n, seed=1000 + n)
    want = orc.sort_keys(x, dt)
    a = x.copy()
    getattr(sorter, f"sort_{dt}")(a)
    assert np.array_equal(bits(a, dt), bits(want, dt))


@pytest.mark.parametrize("n", [2, 33, 4097, 100_003, 1 << 20])
@pytest.mark.parametrize("dt,dist", DT_DIST, ids=[d for d, _ in DT_DIST])
def test_argsort_stable(sorter, dt, dist, n):
    x = orc.gen(dist, n, seed=2000 + n)
    got = getattr(sorter, f"argsort_{dt}")(x)
    assert np.array_equal(got, orc.argsort(x, dt))


@pytest.mark.parametrize("n", [2, 33, 4097, 100_003, 1 << 20])
@pytest.mark.parametrize("dt,dist", DT_DIST, ids=[d for d, _ in DT_DIST])
def test_pairs_stable(sorter, dt, dist, n):
    x = orc.gen(dist, n, seed=3000 + n)
    v = orc.gen("u32", n, seed=9)
    wk, wv = orc.sort_pairs(x, v, dt)
    k = x.copy()
    vv = v.copy()
    getattr(sorter, f"sort_pairs_{dt}")(k, vv)
    assert np.array_equal(bits(k, dt), bits(wk, dt))
    assert np.array_equal(vv, wv)


def _edge_inputs(dt, n):
    npdt = orc.NP_DTYPE[dt]
    rng = np.random.default_rng(n)
    b = orc.BITS_DTYPE[dt]
    yield "zeros", np.zeros(n, npdt)
    yield "all_same", np.full(n, 7, npdt)
    base = orc.gen(dt if dt in ("u32", "i32", "u64", "i64") else ("f32_mix" if dt == "f32" else "f64_logu"), n, seed=5)
    s = orc.sort_keys(base, dt)
    yield "presorted", s
    yield "reverse", s[::-1].copy()
    # keys that vary in only some digits: exercises skipped passes with odd
    # and even counts of executed passes (result must still land in place)
    width = 8 * np.dtype(b).itemsize
    for mask_bits in (8, 16, 24, width - 8):
        m = (1 << mask_bits) - 1
        r = rng.integers(0, 2**63, n, dtype=np.uint64).astype(b) & b(m)
        yield f"low{mask_bits}", r.view(npdt)
    hi = (rng.integers(0, 256, n, dtype=np.uint64).astype(b) << b(width - 8))
    yield "top_byte_only", hi.view(npdt)
    one_hot = np.zeros(n, b)
    one_hot[n // 2] = b(1) << b(width - 1)
    yield "one_hot", one_hot.view(npdt)


@pytest.mark.parametrize("n", [5, 4096, 4097, 70_000])
@pytest.mark.parametrize("dt", ["u32", "i32", "f32", "u64", "i64", "f64"])
def test_edge_distributions(sorter, dt, n):
    for name, x in _edge_inputs(dt, n):
        a = x.copy()
        getattr(sorter, f"sort_{dt}")(a)
        assert np.array_equal(bits(a, dt), bits(orc.sort_keys(x, dt), dt)), name
        idx = getattr(sorter, f"argsort_{dt}")(x)
        assert np.array_equal(idx, orc.argsort(x, dt)), name
        k, v = x.copy(), np.arange(n, dtype=np.uint32)
        getattr(sorter, f"sort_pairs_{dt}")(k, v)
        wk, wv = orc.sort_pairs(x, np.arange(n, dtype=np.uint32), dt)
        assert np.array_equal(bits(k, dt), bits(wk, dt)) and np.array_equal(v, wv), name


@pytest.mark.parametrize("dist", ["zipf_u32", "skew_u32"])
def test_skewed_u32(sorter, dist):
    n = 1 << 20
    x = orc.gen(dist, n, seed=11)
    a = x.copy()
    sorter.sort_u32(a)
    assert np.array_equal(a, orc.sort_keys(x, "u32"))
    assert np.array_equal(sorter.argsort_u32(x), orc.argsort(x, "u32"))


def test_deterministic_repeat(sorter):
    x = orc.gen("zipf_u32", 300_000, seed=4)
    a = sorter.argsort_u32(x)
    b = sorter.argsort_u32(x)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("n", [8193, 65_537, 300_001, 500_000, 1 << 20, (1 << 21) - 5])
@pytest.mark.parametrize("dt,dist", DT_DIST, ids=[d for d, _ in DT_DIST])
def test_single_launch_matches_chain_and_oracle(dt, dist, n):
    """Keys-only 32-bit sorts run as one cooperative launch (k_resident_sort,
    forced here up to 8 MiB): bit-exact against the oracle and the chained
    kernels, in place and out of place, including inputs with skipped passes.
    The sizes reach every keys-per-thread shape (2, 4, 7, 14 on 148 SMs) with a
    partial last CTA.  64-bit keys always take the chain."""
    import torch
    from forge_sort import GpuSorter
    kb = 8 if dt in ("u64", "i64", "f64") else 4
    if n * kb > (8 << 20):
        n = (8 << 20) // kb - 3
    x = orc.gen(dist, n, seed=4000 + n)
    xb = bits(x, dt)
    want = bits(orc.sort_keys(x, dt), dt)
    iv = np.int32 if kb == 4 else np.int64
    one = GpuSorter.new()
    one.set_single_launch_max(8 << 20)
    chain = GpuSorter.new()
    chain.set_single_launch_max(0)
    try:
        for s in (one, chain):
            a = torch.from_numpy(xb.view(iv).copy()).cuda()
            s.sort_device(dt, a.data_ptr(), n)  # in place
            assert np.array_equal(a.cpu().numpy().view(xb.dtype), want)
            b = torch.from_numpy(xb.view(iv).copy()).cuda()
            out = torch.empty_like(b)
            s.sort_device_copy(dt, b.data_ptr(), out.data_ptr(), n)
            assert np.array_equal(out.cpu().numpy().view(xb.dtype), want)
            assert np.array_equal(b.cpu().numpy().view(xb.dtype), xb)  # input untouched
        assert one.last_launch_count() == (1 if kb == 4 else 2 + 3 * kb)
        # low bits only vary: odd and even numbers of executed passes (and,
        # for 32-bit keys, a top digit that never varies: the single launch
        # falls back from the top-digit partition to the LSD passes)
        for mask_bits in (8, 16, 24):
            y = (xb & xb.dtype.type((1 << mask_bits) - 1)).view(orc.NP_DTYPE[dt])
            a = torch.from_numpy(np.ascontiguousarray(y).view(iv).copy()).cuda()
            one.sort_device(dt, a.data_ptr(), n)
            assert np.array_equal(a.cpu().numpy().view(xb.dtype), bits(orc.sort_keys(y, dt), dt)), mask_bits
        # 32-bit keys: only the top byte varies (the partition alone orders
        # them); two top-digit buckets (each larger than a tile: fallback);
        # the top byte and the low byte vary
        if kb == 4:
            for mask in (0xFF000000, 0x100000FF):
                y = (xb & xb.dtype.type(mask)).view(orc.NP_DTYPE[dt])
                a = torch.from_numpy(np.ascontiguousarray(y).view(iv).copy()).cuda()
                one.sort_device(dt, a.data_ptr(), n)
                assert np.array_equal(a.cpu().numpy().view(xb.dtype), bits(orc.sort_keys(y, dt), dt)), hex(mask)
            y = (xb & xb.dtype.type(0xFF0000FF)).view(orc.NP_DTYPE[dt])
            a = torch.from_numpy(np.ascontiguousarray(y).view(iv).copy()).cuda()
            out = torch.empty_like(a)
            one.sort_device_copy(dt, a.data_ptr(), out.data_ptr(), n)
            assert np.array_equal(out.cpu().numpy().view(xb.dtype), bits(orc.sort_keys(y, dt), dt))
        z = np.full(n, 7, orc.NP_DTYPE[dt])  # nothing varies
        a = torch.from_numpy(np.ascontiguousarray(z).view(iv).copy()).cuda()
        out = torch.empty_like(a)
        one.sort_device_copy(dt, a.data_ptr(), out.data_ptr(), n)
        assert np.array_equal(out.cpu().numpy().view(xb.dtype), bits(z, dt))
    finally:
        one.close()
        chain.close()


def test_single_launch_alternating_sizes():
    """Launches of k_resident_sort alternate two accumulator sets, each launch
    clearing the one the next uses: calls of different sizes and grids, back
    to back without a wait between them, must each be bit-exact."""
    import torch
    from forge_sort import GpuSorter
    s = GpuSorter.new()
    s.set_single_launch_max(8 << 20)
    try:
        sizes = [1 << 20, 8193, (1 << 21) - 5, 300_001, 65_537, 1 << 20, 500_000, 20_000, 150_000]
        cases = []
        for i, n in enumerate(sizes * 2):
            dt, dist = DT_DIST[i % len(DT_DIST)]
            if dt in ("u64", "i64", "f64"):
                dt, dist = "u32", "zipf_u32"
            x = orc.gen(dist, n, seed=77 + i)
            xb = bits(x, dt)
            a = torch.from_numpy(xb.view(np.int32).copy()).cuda()
            s.sort_device(dt, a.data_ptr(), n, sync=False)
            assert s.last_launch_count() == 1
            cases.append((a, bits(orc.sort_keys(x, dt), dt)))
        s.synchronize()
        for a, want in cases:
            assert np.array_equal(a.cpu().numpy().view(want.dtype), want)
    finally:
        s.close()
