"""Every single-GPU BASELINE config, bit-exact against the CPU oracle at its
own size, through the public host API (the call a user of forge-sort makes):

  configs[0]  sort_u32, 2^20 uniform keys
  configs[1]  sort_u32 / sort_i32 / sort_f32, 2^24 keys (f32: the IEEE mix)
  configs[2]  sort_u64 / sort_i64 / sort_f64, 2^26 keys; argsort_f32 2^24;
              argsort_u32 / argsort_u64 2^24 (stable)
  configs[3]  sort_pairs_buffer, 2^28 Zipf(1.1) keys over 2^16 values with
              values = original index, through the zero-copy SortBuffer path
  1G u32      the north-star size, 2^30 uniform u32 keys

At these sizes a slice of the array holds many scatter tiles, so the
running per-digit offsets carried from tile to tile within a slice are
compared bit for bit, as are the unstable first pass of a keys-only sort and
every skipped-pass route.  Keys: the oracle's parallel sort of the
order-transformed bits (Rust sort_unstable / total_cmp order; equal keys have
equal bits, so the answer is unique).  argsort / pairs: the oracle's stable
order (ties by input position), i.e. Rust's stable sort_by_key
(forge-sort tests/correctness_argsort.rs:42-56,
tests/correctness_sort_pairs.rs:35-45).  Mirrors the reference's own
full-size correctness tests (tests/correctness.rs:28-35, which go to 16M,
and tests/correctness_u64.rs)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def bits(a, dt):
    return np.ascontiguousarray(a).view(orc.BITS_DTYPE[dt])


def test_configs0_sort_u32_2e20(sorter):
    x = orc.gen("u32", 1 << 20, seed=42)
    a = x.copy()
    sorter.sort_u32(a)
    assert np.array_equal(a, orc.par_sort_keys(x, "u32"))


@pytest.mark.parametrize("dt,dist", [("u32", "u32"), ("i32", "i32"), ("f32", "f32_mix")])
def test_configs1_sort_2e24(sorter, dt, dist):
    x = orc.gen(dist, 1 << 24, seed=42)
    want = orc.par_sort_keys(x, dt)
    a = x.copy()
    getattr(sorter, f"sort_{dt}")(a)
    assert np.array_equal(bits(a, dt), bits(want, dt))


@pytest.mark.slow
@pytest.mark.parametrize("dt,dist", [("u64", "u64"), ("i64", "i64"), ("f64", "f64_logu")])
def test_configs2_sort_2e26(sorter, dt, dist):
    x = orc.gen(dist, 1 << 26, seed=42)
    want = orc.par_sort_keys(x, dt)
    a = x.copy()
    getattr(sorter, f"sort_{dt}")(a)
    assert np.array_equal(bits(a, dt), bits(want, dt))


@pytest.mark.slow
@pytest.mark.parametrize("dt,dist", [("f32", "f32_mix"), ("u32", "zipf_u32"), ("u64", "u64"), ("i64", "i64")])
def test_configs2_argsort_2e24(sorter, dt, dist):
    x = orc.gen(dist, 1 << 24, seed=42)
    x0 = x.copy()
    got = getattr(sorter, f"argsort_{dt}")(x)
    assert np.array_equal(bits(x, dt), bits(x0, dt)), "argsort modified its input"
    assert np.array_equal(got, orc.par_argsort(x, dt))


@pytest.mark.slow
def test_configs3_sort_pairs_buffer_2e28_zipf(sorter):
    n = 1 << 28
    keys = orc.gen("zipf_u32", n, seed=42)
    vals = np.arange(n, dtype=np.uint32)
    want_k, want_v = orc.par_sort_pairs(keys, vals, "u32")
    kb = sorter.alloc_sort_buffer("u32", n)
    vb = sorter.alloc_sort_buffer("u32", n)
    try:
        kb.copy_from_slice(keys)
        vb.copy_from_slice(vals)
        sorter.sort_pairs_buffer(kb, vb)
        assert np.array_equal(kb.as_slice(), want_k)
        assert np.array_equal(vb.as_slice(), want_v)
    finally:
        kb.free()
        vb.free()


@pytest.mark.slow
def test_1g_u32_device_generated_matches_oracle(sorter):
    """2^30 u32 keys generated on the device by fs_generate (the bench's
    input), sorted out of place, copied back and compared with the oracle's
    sort of the same stream generated on the host."""
    import torch
    from forge_sort import _lib
    n = 1 << 30
    L = _lib.load()
    kin = torch.empty(n, dtype=torch.int32, device="cuda")
    assert L.fs_generate(_lib.GEN_U32, 42, 0, n, kin.data_ptr(), None) == 0
    kout = torch.empty_like(kin)
    sorter.sort_device_copy("u32", kin.data_ptr(), kout.data_ptr(), n)
    host_in = orc.gen("u32", n, seed=42)
    assert np.array_equal(kin[: 1 << 20].cpu().numpy().view(np.uint32), host_in[: 1 << 20]), "generator mismatch"
    del kin
    got = kout.cpu().numpy().view(np.uint32)
    del kout
    torch.cuda.empty_cache()
    want = orc.par_sort_keys(host_in, "u32")
    assert np.array_equal(got, want)
