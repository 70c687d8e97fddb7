"""Failure paths on the GPU, made without faulting or hanging it.

The reference maps a failed command buffer to SortError::GpuExecution
(forge-sort src/lib.rs:396-406) and panics when a buffer allocation fails
(src/metal_helpers.rs:194-202).  Here:
  - a bounded device wait that runs out: one bulk copy is left un-issued
    (fs_test_inject FS_TEST_WITHHOLD_COPY), the scatter's mbarrier wait gives
    up after the sorter's wait bound (10 ms here), the kernels stop early and
    the call fails with a timeout (GpuExecution);
  - a grid barrier that never completes: CTA 0 of the single-launch sort
    leaves before the first barrier (FS_TEST_SKIP_ARRIVAL), the other CTAs'
    bounded waits run out and the call fails with a timeout;
  - a device allocation that fails (FS_TEST_FAIL_ALLOC): the call fails with
    an out-of-memory GpuExecution, nothing leaks into the next call.
After each, the same sorter must sort correctly again (bit-exact against the
oracle)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_then_sorter_recovers():
    from forge_sort import GpuSorter, _lib
    from forge_sort.errors import GpuExecution

    s = GpuSorter.new()
    try:
        s.set_wait_timeout_ms(10)
        x = orc.gen("u32", 1 << 20, seed=123)
        a = x.copy()
        s._test_inject(_lib.TEST_WITHHOLD_COPY)
        with pytest.raises(GpuExecution) as ei:
            s.sort_u32(a)
        assert "timeout" in str(ei.value)
        # the injection is one-shot; the control block and error word re-arm
        for dt, dist in (("u32", "u32"), ("f64", "f64_logu")):
            y = orc.gen(dist, 300_001, seed=7)
            b = y.copy()
            getattr(s, f"sort_{dt}")(b)
            assert np.array_equal(b.view(orc.BITS_DTYPE[dt]), orc.sort_keys(y, dt).view(orc.BITS_DTYPE[dt]))
        idx = s.argsort_f32(orc.gen("f32_mix", 100_000, seed=3))
        assert np.array_equal(idx, orc.argsort(orc.gen("f32_mix", 100_000, seed=3), "f32"))
    finally:
        s.close()


def test_grid_barrier_wait_runs_out_then_sorter_recovers():
    from forge_sort import GpuSorter, _lib
    from forge_sort.errors import GpuExecution

    s = GpuSorter.new()
    try:
        s.set_single_launch_max(8 << 20)
        s.set_wait_timeout_ms(10)
        x = orc.gen("u32", 1 << 20, seed=321)
        s._test_inject(_lib.TEST_SKIP_ARRIVAL)
        with pytest.raises(GpuExecution) as ei:
            s.sort_u32(x.copy())
        assert "timeout" in str(ei.value)
        # the barrier count and error word are cleared before the next sort
        for dt, dist, n in (("u32", "u32", 1 << 20), ("f32", "f32_mix", 300_001), ("i32", "i32", 8193),
                            ("u64", "u64", 200_000)):
            y = orc.gen(dist, n, seed=9)
            b = y.copy()
            getattr(s, f"sort_{dt}")(b)
            assert np.array_equal(b.view(orc.BITS_DTYPE[dt]), orc.sort_keys(y, dt).view(orc.BITS_DTYPE[dt])), dt
    finally:
        s.close()


def test_bounded_wait_on_pairs_path():
    from forge_sort import GpuSorter, _lib
    from forge_sort.errors import GpuExecution

    s = GpuSorter.new()
    try:
        s.set_wait_timeout_ms(10)
        k = orc.gen("u64", 200_000, seed=5)
        v = np.arange(k.size, dtype=np.uint32)
        s._test_inject(_lib.TEST_WITHHOLD_COPY)
        with pytest.raises(GpuExecution):
            s.sort_pairs_u64(k.copy(), v.copy())
        kk, vv = k.copy(), v.copy()
        s.sort_pairs_u64(kk, vv)
        wk, wv = orc.sort_pairs(k, v, "u64")
        assert np.array_equal(kk, wk) and np.array_equal(vv, wv)
    finally:
        s.close()


@pytest.mark.parametrize("nth", [1, 2])
def test_injected_out_of_memory_then_sorter_recovers(nth):
    from forge_sort import GpuSorter, _lib
    from forge_sort.errors import GpuExecution

    s = GpuSorter.new()  # fresh: every scratch slot still has to grow
    try:
        x = orc.gen("i32", 1 << 20, seed=11)
        s._test_inject(_lib.TEST_FAIL_ALLOC, nth)
        with pytest.raises(GpuExecution) as ei:
            s.sort_i32(x.copy())
        assert "out of memory" in str(ei.value)
        a = x.copy()
        s.sort_i32(a)
        assert np.array_equal(a, orc.sort_keys(x, "i32"))
        idx = s.argsort_i32(x)
        assert np.array_equal(idx, orc.argsort(x, "i32"))
    finally:
        s.close()


def test_inject_rejects_bad_arguments():
    from forge_sort import GpuSorter, _lib

    s = GpuSorter.new()
    try:
        with pytest.raises(ValueError):
            s._test_inject(99)
        with pytest.raises(ValueError):
            s._test_inject(_lib.TEST_FAIL_ALLOC, 0)
        with pytest.raises(ValueError):
            s.set_wait_timeout_ms(0)
        s._test_inject(0)  # disarm: a plain sort works
        x = orc.gen("u32", 50_000, seed=1)
        a = x.copy()
        s.sort_u32(a)
        assert np.array_equal(a, orc.sort_keys(x, "u32"))
    finally:
        s.close()
