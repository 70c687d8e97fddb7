"""Full BASELINE sizes, checked through size-independent properties on the
device (the oracle cannot sort 2^32 keys in test time):
  - the output is sorted (unsigned order of the order-transformed bits);
  - it is a permutation of the input: equal wrapping sums of x, x^2 and x^3
    (64-bit) before and after;
  - pairs / argsort: stable -- within equal keys the original positions are
    ascending -- and every (key, value) pair is an input pair.
Inputs come from the library's own seed-42 generators (fs_generate)."""
import pytest

pytestmark = [pytest.mark.gpu]

CH = 1 << 27  # keys per checking chunk (bounds the int64 temporaries)


def _unsigned(t):
    """int64 view of raw 32-bit bits as unsigned values, or 64-bit bits with
    the sign flipped so that signed int64 order is the unsigned order."""
    import torch
    if t.dtype == torch.int32:
        return t.to(torch.int64) & 0xFFFFFFFF
    return t ^ torch.iinfo(torch.int64).min


def _moments(t):
    import torch
    s1 = s2 = s3 = torch.zeros((), dtype=torch.int64, device=t.device)
    for i in range(0, t.numel(), CH):
        x = t[i:i + CH].to(torch.int64)
        s1 = s1 + x.sum()
        s2 = s2 + (x * x).sum()
        s3 = s3 + (x * x * x).sum()
    return int(s1), int(s2), int(s3)


def _assert_sorted(t):
    prev = None
    for i in range(0, t.numel(), CH):
        c = _unsigned(t[i:i + CH])
        assert bool((c[1:] >= c[:-1]).all()), f"not sorted in chunk at {i}"
        if prev is not None:
            assert int(c[0]) >= prev, f"not sorted across the chunk boundary at {i}"
        prev = int(c[-1])


def _generate(n, dist, dtype):
    import torch
    from forge_sort import _lib
    L = _lib.load()
    t = torch.empty(n, dtype=dtype, device="cuda")
    assert L.fs_generate(dist, 42, 0, n, t.data_ptr(), None) == 0
    torch.cuda.synchronize()
    return t


@pytest.mark.slow
@pytest.mark.parametrize("log2n,dist", [(32, "uniform"), (32, "skew")])
def test_u32_2e32_sorted_permutation(sorter, log2n, dist):
    """configs[4] on one GPU: 2^32 u32 keys (16 GiB), uniform and 70% in one
    2^20-wide range."""
    import torch
    from forge_sort import _lib
    n = 1 << log2n
    x = _generate(n, _lib.GEN_U32 if dist == "uniform" else _lib.GEN_SKEW_U32, torch.int32)
    want = _moments(x)
    out = torch.empty_like(x)
    sorter.sort_device_copy("u32", x.data_ptr(), out.data_ptr(), n)
    _assert_sorted(out)
    assert _moments(out) == want
    del x, out
    torch.cuda.empty_cache()


@pytest.mark.slow
def test_u64_2e30_in_place(sorter):
    """configs[4] u64 on one GPU: 2^30 u64 keys sorted in place."""
    import torch
    from forge_sort import _lib
    n = 1 << 30
    x = _generate(n, _lib.GEN_U64, torch.int64)
    want = _moments(x)
    sorter.sort_device("u64", x.data_ptr(), n)
    _assert_sorted(x)
    assert _moments(x) == want
    del x
    torch.cuda.empty_cache()


@pytest.mark.slow
def test_pairs_2e28_zipf_stable(sorter):
    """2^28 (key, original index) pairs with Zipf keys over 2^16
    values (two digit passes trivial): keys sorted, every pair kept, indices
    ascending within equal keys (stability)."""
    import numpy as np
    import torch
    from oracle import oracle as orc
    n = 1 << 28
    keys_h = orc.gen("zipf_u32", n, seed=42)
    k = torch.from_numpy(keys_h.view(np.int32)).to("cuda")
    v = torch.arange(n, dtype=torch.int32, device="cuda")
    k0 = k.clone()
    sorter.sort_pairs_device("u32", k.data_ptr(), v.data_ptr(), n)
    _assert_sorted(k)
    # every output pair is an input pair: key == original key at that index
    for i in range(0, n, CH):
        assert bool((k0[v[i:i + CH].to(torch.int64)] == k[i:i + CH]).all())
    # stability: within a run of equal keys the original indices ascend
    for i in range(0, n, CH):
        kk, vv = k[i:i + CH + 1], v[i:i + CH + 1]
        same = kk[1:] == kk[:-1]
        assert bool(((vv[1:] > vv[:-1]) | ~same).all())
    # the indices are a permutation of 0..n-1
    assert int(torch.bincount(v.to(torch.int64), minlength=n).max()) == 1


@pytest.mark.slow
def test_argsort_f32_2e24_matches_oracle(sorter):
    """configs[2] argsort_f32 at its full size (16M): bit-exact against the
    oracle's stable sort (small enough for the oracle)."""
    import numpy as np
    from oracle import oracle as orc
    x = orc.gen("f32_mix", 1 << 24, seed=42)
    got = sorter.argsort_f32(x)
    assert np.array_equal(got, orc.argsort(x, "f32"))
