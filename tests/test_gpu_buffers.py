"""SortBuffer (zero-copy), encode_sort on a caller stream, scratch reuse and
cross-type interleaving -- the reference's correctness.rs:86-239 and
regression.rs:8-193 behaviours."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_sort_buffer_basic_and_direct_write(sorter):
    buf = sorter.alloc_sort_buffer("u32", 1000)
    assert buf.capacity() == 1000 and buf.len() == 0 and buf.is_empty()
    x = orc.gen("u32", 1000, seed=1)
    buf.as_mut_slice()[:1000] = x
    buf.set_len(1000)
    sorter.sort_buffer(buf)
    assert np.array_equal(buf.as_slice(), np.sort(x))
    out = np.zeros(1000, np.uint32)
    buf.copy_to_slice(out)
    assert np.array_equal(out, np.sort(x))
    with pytest.raises(AssertionError):
        buf.set_len(1001)


@pytest.mark.parametrize("dt,dist", [("i32", "i32"), ("f32", "f32_mix"), ("u64", "u64"),
                                     ("i64", "i64"), ("f64", "f64_logu")])
def test_typed_buffers(sorter, dt, dist):
    x = orc.gen(dist, 50_001, seed=2)
    buf = sorter.alloc_sort_buffer(dt, x.size)
    buf.copy_from_slice(x)
    getattr(sorter, f"sort_{dt}_buffer")(buf)
    want = orc.sort_keys(x, dt)
    assert np.array_equal(buf.as_slice().view(orc.BITS_DTYPE[dt]), want.view(orc.BITS_DTYPE[dt]))
    with pytest.raises(TypeError):
        sorter.sort_buffer(buf)  # SortBuffer<u32> required


def test_sort_buffer_reuse_and_grow_only_scratch(sorter):
    buf = sorter.alloc_sort_buffer("u32", 1 << 20)
    sizes = [1 << 20, 1000, 4097, 1 << 18]
    peak = 0
    for i, n in enumerate(sizes):
        x = orc.gen("u32", n, seed=10 + i)
        buf.copy_from_slice(x)
        sorter.sort_buffer(buf)
        assert np.array_equal(buf.as_slice(), np.sort(x))
        s = sorter.scratch_bytes()
        assert s >= peak
        peak = s


def test_sort_pairs_buffer(sorter):
    n = 100_000
    k = orc.gen("zipf_u32", n, seed=5)
    kb = sorter.alloc_sort_buffer("u32", n)
    vb = sorter.alloc_sort_buffer("u32", n)
    kb.copy_from_slice(k)
    vb.copy_from_slice(np.arange(n, dtype=np.uint32))
    sorter.sort_pairs_buffer(kb, vb)
    wk, wv = orc.sort_pairs(k, np.arange(n, dtype=np.uint32), "u32")
    assert np.array_equal(kb.as_slice(), wk) and np.array_equal(vb.as_slice(), wv)


def test_encode_sort_on_caller_stream(sorter):
    import torch
    s = torch.cuda.Stream()
    buf = sorter.alloc_sort_buffer("u32", 1024)
    data = np.array([50, 10, 90, 30, 70, 20, 80, 40, 60, 100], np.uint32)
    buf.copy_from_slice(data)
    sorter.encode_sort(s, buf)
    s.synchronize()
    assert list(buf.as_slice()) == sorted(data.tolist())
    one = sorter.alloc_sort_buffer("u32", 1)
    one.copy_from_slice(np.array([42], np.uint32))
    sorter.encode_sort(s, one)  # n <= 1: nothing enqueued
    assert list(one.as_slice()) == [42]
    sorter.set_stream(None)


def test_with_context_shares_caller_stream():
    import torch
    from forge_sort import GpuSorter
    st = torch.cuda.Stream()
    s = GpuSorter.with_context(0, st)
    t = torch.from_numpy(orc.gen("u32", 1 << 16, seed=3).view(np.int32)).cuda()
    with torch.cuda.stream(st):
        s.sort_device("u32", t.data_ptr(), t.numel(), sync=False)
    st.synchronize()
    got = t.cpu().numpy().view(np.uint32)
    assert np.array_equal(got, np.sort(orc.gen("u32", 1 << 16, seed=3)))
    s.close()


def test_cross_type_interleave(sorter):
    for i in range(3):
        for dt, dist in (("u32", "u32"), ("f64", "f64_logu"), ("i32", "i32"), ("u64", "u64"), ("f32", "f32_mix")):
            x = orc.gen(dist, 10_000 + i, seed=i)
            a = x.copy()
            getattr(sorter, f"sort_{dt}")(a)
            assert np.array_equal(a.view(orc.BITS_DTYPE[dt]), orc.sort_keys(x, dt).view(orc.BITS_DTYPE[dt]))
            assert np.array_equal(getattr(sorter, f"argsort_{dt}")(x), orc.argsort(x, dt))


def test_device_pointer_checks(sorter):
    host = np.zeros(16, np.uint32)
    with pytest.raises(ValueError):
        sorter.sort_device("u32", host.ctypes.data, 16)


def test_launch_count(sorter):
    x = orc.gen("u32", 100_000, seed=1)
    sorter.sort_u32(x.copy())
    assert sorter.last_launch_count() == 1  # keys-only 32-bit up to 8 MiB: one cooperative launch
    sorter.set_single_launch_max(0)
    try:
        sorter.sort_u32(x.copy())
    finally:
        sorter.set_single_launch_max(8 << 20)
    # first count, plan, per pass (count -- pass 0 is counted by the first
    # count --, scan, scatter -- pass 0 ranks unstably, the others stably),
    # finalize
    assert sorter.last_launch_count() == 2 + 3 * 4
    y = orc.gen("u64", 100_000, seed=1)
    sorter.sort_u64(y.copy())
    assert sorter.last_launch_count() == 2 + 3 * 8
    k, v = orc.gen("u32", 10_000, seed=2), np.arange(10_000, dtype=np.uint32)
    sorter.sort_pairs_u32(k, v)  # payload: every pass ranks stably, one scatter each
    assert sorter.last_launch_count() == 2 + 3 * 4
    # up to 4096 keys with a payload, 8192 without: one single-CTA launch
    for dt in ("u32", "f64"):
        getattr(sorter, f"argsort_{dt}")(orc.gen("u32" if dt == "u32" else "f64_logu", 4096, seed=3))
        assert sorter.last_launch_count() == 1
        getattr(sorter, f"sort_{dt}")(orc.gen("u32" if dt == "u32" else "f64_logu", 8192, seed=3))
        assert sorter.last_launch_count() == 1
    sorter.argsort_u32(orc.gen("u32", 4097, seed=3))
    assert sorter.last_launch_count() == 2 + 3 * 4


@pytest.mark.parametrize("dt,dist", [("u32", "u32"), ("i32", "i32"), ("f32", "f32_mix"),
                                     ("u64", "u64"), ("i64", "i64"), ("f64", "f64_logu")])
def test_small_sort_matches_radix_path(sorter, monkeypatch, dt, dist):
    """The single-CTA path (n <= 8192 keys alone, <= 4096 with a payload;
    6000 and 8192 below cover both sides) and the radix passes
    (FORGESORT_SMALL_SORT=0) give the same keys, the same stable argsort and
    the same pairs, on inputs full of ties, and sort device memory in place."""
    import torch
    from forge_sort import GpuSorter
    monkeypatch.setenv("FORGESORT_SMALL_SORT", "0")
    radix = GpuSorter()
    rng = np.random.default_rng(17)
    for n in (1, 2, 3, 255, 1000, 2049, 4096, 6000, 8192):
        x = orc.gen(dist, n, seed=n)
        x[rng.integers(0, n, n // 2)] = x[0]  # ties
        for srt in (sorter, radix):
            a = x.copy()
            getattr(srt, f"sort_{dt}")(a)
            assert np.array_equal(a.view(orc.BITS_DTYPE[dt]), orc.sort_keys(x, dt).view(orc.BITS_DTYPE[dt]))
            assert np.array_equal(getattr(srt, f"argsort_{dt}")(x), orc.argsort(x, dt))
            k, v = x.copy(), orc.gen("u32", n, seed=5)
            wk, wv = orc.sort_pairs(x, v, dt)
            getattr(srt, f"sort_pairs_{dt}")(k, v)
            assert np.array_equal(k.view(orc.BITS_DTYPE[dt]), wk.view(orc.BITS_DTYPE[dt]))
            assert np.array_equal(v, wv)
        # in place on the device
        t = torch.from_numpy(x.view(orc.BITS_DTYPE[dt]).view(np.int32 if x.itemsize == 4 else np.int64)).cuda()
        sorter.sort_device(dt, t.data_ptr(), n)
        got = t.cpu().numpy().view(orc.BITS_DTYPE[dt])
        assert np.array_equal(got, orc.sort_keys(x, dt).view(orc.BITS_DTYPE[dt]))
    radix.close()


def test_async_host_sorts_overlap_and_match(sorter):
    """fs_host_sort_keys_copy_async: a stream of calls (mixed types, sizes
    that grow the two device buffers, n = 0 and 1), one synchronize, every
    output bit-exact; inputs untouched."""
    import torch
    cases = [("u32", "u32", 1 << 20), ("f32", "f32_mix", 300_001), ("u64", "u64", 1 << 19),
             ("u32", "skew_u32", 3 << 20), ("i64", "i64", 1), ("i32", "i32", 0), ("f64", "f64_logu", 77_777),
             ("u32", "zipf_u32", 2 << 20)]
    ins, outs, keep = [], [], []
    for dt, dist, n in cases:
        x = orc.gen(dist, n, seed=n + 3)
        tdt = torch.int32 if x.itemsize == 4 else torch.int64
        h_in = torch.from_numpy(np.ascontiguousarray(x).view(np.int32 if x.itemsize == 4 else np.int64)).pin_memory()
        h_out = torch.zeros(n, dtype=tdt).pin_memory()
        sorter.host_sort_copy_async_ptr(dt, h_in.data_ptr(), h_out.data_ptr(), n)
        ins.append(h_in)
        outs.append(h_out)
        keep.append((dt, x))
    sorter.synchronize()
    for (dt, x), h_in, h_out in zip(keep, ins, outs):
        bits = orc.BITS_DTYPE[dt]
        assert np.array_equal(h_in.numpy().view(bits), np.ascontiguousarray(x).view(bits))
        assert np.array_equal(h_out.numpy().view(bits), orc.sort_keys(x, dt).view(bits)), dt


@pytest.mark.parametrize("width", [4, 8])
def test_gather_applies_argsort_permutation(sorter, width):
    """fs_gather: dst[i] = src[idx[i]] (forge-runtime GpuGather): applying the
    argsort of keys to a payload equals the payload of a stable pairs sort;
    an out-of-range index is an error, not a wild read."""
    import torch
    from forge_sort import GpuExecution
    n = 1_000_003
    keys = orc.gen("zipf_u32", n, seed=5)
    payload = orc.gen("u64" if width == 8 else "u32", n, seed=6)
    tdt = torch.int64 if width == 8 else torch.int32
    idx = torch.from_numpy(sorter.argsort_u32(keys).view(np.int32)).cuda()
    src = torch.from_numpy(np.ascontiguousarray(payload).view(np.int64 if width == 8 else np.int32)).cuda()
    dst = torch.empty_like(src)
    sorter.gather_device(width, src.data_ptr(), n, idx.data_ptr(), dst.data_ptr(), n)
    want = payload[orc.argsort(keys, "u32")]
    assert np.array_equal(dst.cpu().numpy().view(want.dtype), want)
    # unaligned index pointer (scalar path) and a tail shorter than 4
    sorter.gather_device(width, src.data_ptr(), n, idx.data_ptr() + 4, dst.data_ptr(), 7)
    assert np.array_equal(dst[:7].cpu().numpy().view(want.dtype), want[1:8])
    bad = idx.clone()
    bad[123] = n
    with pytest.raises(GpuExecution):
        sorter.gather_device(width, src.data_ptr(), n, bad.data_ptr(), dst.data_ptr(), n)


def test_sort_buffer_coherence_between_host_and_device(sorter):
    """The device copy and the host mirror of a SortBuffer stay coherent
    through every access pattern of the reference's shared buffer: sorts
    without host access in between, host writes after a sort (partial, then
    a longer len), reads after writes."""
    n = 1 << 16
    buf = sorter.alloc_sort_buffer("u32", n)
    x = orc.gen("u32", n // 2, seed=31)
    buf.copy_from_slice(x)
    sorter.sort_buffer(buf)
    sorter.sort_buffer(buf)  # again with no host access: stays on the device
    assert np.array_equal(buf.as_slice(), np.sort(x))
    # write the second half through a fresh as_mut_slice session, sort all n
    y = orc.gen("u32", n // 2, seed=32)
    w = buf.as_mut_slice()
    w[n // 2:] = y
    buf.set_len(n)
    sorter.sort_buffer(buf)
    assert np.array_equal(buf.as_slice(), np.sort(np.concatenate([x, y])))
    # overwrite a few leading elements after the sort, sort again
    w = buf.as_mut_slice()
    w[:3] = [7, 5, 6]
    sorter.sort_buffer(buf)
    want = np.sort(np.concatenate([[7, 5, 6], np.sort(np.concatenate([x, y]))[3:]]).astype(np.uint32))
    assert np.array_equal(buf.as_slice(), want)
    # a shorter len sorts only its prefix; the rest keeps its values
    before = buf.as_slice().copy()
    z = np.arange(100, 0, -1, dtype=np.uint32)
    buf.as_mut_slice()[:100] = z
    buf.set_len(100)
    sorter.sort_buffer(buf)
    buf.set_len(n)
    got = buf.as_slice()
    assert np.array_equal(got[:100], np.sort(z)) and np.array_equal(got[100:], before[100:])
    buf.free()


def test_sort_buffer_raw_parts_device_use_and_lifetime():
    """into_raw_parts / from_raw_parts round trip; device code reading and
    writing a SortBuffer through device_ptr() (here the library's gather);
    the buffer outliving the sorter that created it."""
    import torch
    from forge_sort import GpuSorter, SortBuffer
    s = GpuSorter.new()
    g = GpuSorter.new()
    x = orc.gen("f64_logu", 30_000, seed=4)
    n = x.size
    buf = s.alloc_sort_buffer("f64", n)
    buf.copy_from_slice(x)
    h, ln, cap = buf.into_raw_parts()
    buf2 = SortBuffer.from_raw_parts(s, "f64", h, ln, cap)
    s.sort_f64_buffer(buf2)
    want = orc.sort_keys(x, "f64")
    ident = torch.arange(n, dtype=torch.int32, device="cuda")
    out = torch.empty(n, dtype=torch.int64, device="cuda")
    g.gather_device(8, buf2.device_ptr(), n, ident.data_ptr(), out.data_ptr(), n)  # device reads the buffer
    assert np.array_equal(out.cpu().numpy().view(np.uint64), want.view(np.uint64))
    neg = torch.from_numpy(np.ascontiguousarray(-want).view(np.int64)).cuda()
    g.gather_device(8, neg.data_ptr(), n, ident.data_ptr(), buf2.device_ptr(), n)  # device writes it
    s.close()  # the buffer outlives its sorter
    g.close()
    assert np.array_equal(buf2.as_slice().view(np.uint64), np.ascontiguousarray(-want).view(np.uint64))
    buf2.free()
