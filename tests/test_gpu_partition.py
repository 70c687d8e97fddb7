"""fs_partition (the sample sort's bucket pass) against a numpy stable
partition by (ordered key, global position) -- bit-exact, including keys
equal to a splitter (duplicate-heavy Zipf input)."""
import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def ref_partition(x, dt, gpos_base, spl_raw, spl_gpos):
    from forge_sort.samplesort import ordered_bits
    o = ordered_bits(x, dt)
    g = np.arange(x.size, dtype=np.uint64) + np.uint64(gpos_base)
    so = ordered_bits(spl_raw, dt)
    b = np.zeros(x.size, np.int64)
    for j in range(len(spl_gpos)):
        b += ((o > so[j]) | ((o == so[j]) & (g >= spl_gpos[j]))).astype(np.int64)
    idx = np.argsort(b, kind="stable")
    return x[idx], np.bincount(b, minlength=len(spl_gpos) + 1)


@pytest.mark.parametrize("dt,dist,nspl", [("u32", "u32", 7), ("u32", "zipf_u32", 3), ("f32", "f32_mix", 1),
                                         ("u64", "u64", 15), ("i64", "i64", 2), ("u32", "u32", 0),
                                         ("i32", "i32", 255)])
def test_partition_matches_stable_reference(sorter, dt, dist, nspl):
    import torch
    from forge_sort.samplesort import choose_splitters, ordered_bits
    n, base = 200_003, 1_000_000
    x = orc.gen(dist, n, seed=31 + nspl)
    bits = orc.BITS_DTYPE[dt]
    xb = np.ascontiguousarray(x).view(bits)
    # splitters from regular samples, as the sample sort picks them
    per = 64
    pos = ((np.arange(per * (nspl + 1)) + 0.5) * (n / (per * (nspl + 1)))).astype(np.int64)
    samp_raw, samp_gpos = xb[pos], (pos + base).astype(np.uint64)
    picks = choose_splitters(ordered_bits(samp_raw, dt), samp_gpos, nspl + 1, per)
    spl_raw, spl_gpos = samp_raw[picks], samp_gpos[picks]
    tdt = torch.int32 if bits is np.uint32 else torch.int64
    keys = torch.from_numpy(xb.view(np.int32 if bits is np.uint32 else np.int64).copy()).cuda()
    out = torch.empty_like(keys)
    counts = torch.zeros(nspl + 1, dtype=torch.int64, device="cuda")
    sk = torch.from_numpy(spl_raw.view(np.int32 if bits is np.uint32 else np.int64).copy()).cuda() if nspl else None
    sg = torch.from_numpy(spl_gpos.view(np.int64).copy()).cuda() if nspl else None
    sorter.partition_device(dt, keys.data_ptr(), n, base, sk.data_ptr() if nspl else 0,
                            sg.data_ptr() if nspl else 0, nspl, out.data_ptr(), counts.data_ptr())
    want, wcounts = ref_partition(xb, dt, base, spl_raw, spl_gpos)
    assert np.array_equal(out.cpu().numpy().view(bits), want)
    assert counts.cpu().numpy().tolist() == wcounts.tolist()
    del tdt


def test_single_rank_sample_sort_is_the_local_sort(sorter):
    import torch
    import torch.distributed as dist
    from forge_sort.samplesort import CudaOps, SampleSorter
    import os
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        x = orc.gen("u32", 100_000, seed=3)
        keys = torch.from_numpy(x.view(np.int32).copy()).cuda()
        out = SampleSorter(CudaOps(sorter, torch), dtype="u32").sort(keys)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), np.sort(x))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dt,dist,nspl,with_vals", [("u32", "zipf_u32", 3, True), ("f32", "f32_mix", 7, False),
                                                    ("u64", "u64", 1, True), ("i64", "i64", 12, False),
                                                    ("i32", "i32", 0, True)])
def test_dispatch_pairs_matches_stable_reference(sorter, dt, dist, nspl, with_vals):
    """fs_partition_count + fs_partition_dispatch_pairs with every bucket's
    destination a region of one local buffer (the single-GPU shape of the
    peers' inboxes): keys and their values (given, or the global positions)
    land bucket by bucket in stable order."""
    import torch
    from forge_sort.samplesort import choose_splitters, ordered_bits
    n, base = 300_007, 5_000_000
    x = orc.gen(dist, n, seed=7 + nspl)
    bits = orc.BITS_DTYPE[dt]
    iv = np.int32 if bits is np.uint32 else np.int64
    xb = np.ascontiguousarray(x).view(bits)
    per = 64
    pos = ((np.arange(per * (nspl + 1)) + 0.5) * (n / (per * (nspl + 1)))).astype(np.int64)
    samp_raw, samp_gpos = xb[pos], (pos + base).astype(np.uint64)
    picks = choose_splitters(ordered_bits(samp_raw, dt), samp_gpos, nspl + 1, per)
    spl_raw, spl_gpos = samp_raw[picks], samp_gpos[picks]
    keys = torch.from_numpy(xb.view(iv).copy()).cuda()
    vals_h = orc.gen("u32", n, seed=99)
    vals = torch.from_numpy(vals_h.view(np.int32).copy()).cuda()
    sk = torch.from_numpy(spl_raw.view(iv).copy()).cuda() if nspl else None
    sg = torch.from_numpy(spl_gpos.view(np.int64).copy()).cuda() if nspl else None
    skp, sgp = (sk.data_ptr(), sg.data_ptr()) if nspl else (0, 0)
    counts = sorter.partition_count(dt, keys.data_ptr(), n, base, skp, sgp, nspl)
    want_k, wcounts = ref_partition(xb, dt, base, spl_raw, spl_gpos)
    assert counts == wcounts.tolist()
    # the same stable order applied to the values
    o = ordered_bits(xb, dt)
    g = np.arange(n, dtype=np.uint64) + np.uint64(base)
    so = ordered_bits(spl_raw, dt)
    b = np.zeros(n, np.int64)
    for j in range(nspl):
        b += ((o > so[j]) | ((o == so[j]) & (g >= spl_gpos[j]))).astype(np.int64)
    order = np.argsort(b, kind="stable")
    want_v = vals_h[order] if with_vals else (order + base).astype(np.uint32)
    out_k = torch.full((n + 64,), -1, dtype=keys.dtype, device="cuda")
    out_v = torch.full((n + 64,), -1, dtype=torch.int32, device="cuda")
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    kb = keys.element_size()
    dst = [out_k.data_ptr() + int(st) * kb for st in starts]
    vdst = [out_v.data_ptr() + int(st) * 4 for st in starts]
    sorter.partition_dispatch_pairs(dt, keys.data_ptr(), vals.data_ptr() if with_vals else 0, n, base, skp, sgp,
                                    nspl, dst, vdst, sync=True)
    assert np.array_equal(out_k[:n].cpu().numpy().view(bits), want_k)
    assert np.array_equal(out_v[:n].cpu().numpy().view(np.uint32), want_v)
    assert bool((out_k[n:] == -1).all()) and bool((out_v[n:] == -1).all())  # nothing past the regions


@pytest.mark.parametrize("n", [1, 2, 4096, 100_003])
@pytest.mark.parametrize("dt,dist", [("u32", "zipf_u32"), ("i32", "i32"), ("f32", "f32_mix"), ("u64", "u64"),
                                     ("i64", "i64"), ("f64", "f64_logu")])
def test_sort_pairs_copy_matches_oracle(sorter, dt, dist, n):
    """fs_sort_pairs_copy: stable, inputs untouched; vals_in NULL gives the
    input positions."""
    import torch
    x = orc.gen(dist, n, seed=n + 3)
    bits = orc.BITS_DTYPE[dt]
    iv = np.int32 if bits is np.uint32 else np.int64
    v = orc.gen("u32", n, seed=n + 4)
    kin = torch.from_numpy(np.ascontiguousarray(x).view(iv).copy()).cuda()
    vin = torch.from_numpy(v.view(np.int32).copy()).cuda()
    kin0, vin0 = kin.clone(), vin.clone()
    order = orc.argsort(x, dt)
    for with_vals in (True, False):
        kout = torch.empty_like(kin)
        vout = torch.empty_like(vin)
        sorter.sort_pairs_device_copy(dt, kin.data_ptr(), vin.data_ptr() if with_vals else 0, kout.data_ptr(),
                                      vout.data_ptr(), n)
        assert np.array_equal(kout.cpu().numpy().view(bits), np.ascontiguousarray(x).view(bits)[order])
        want_v = v[order] if with_vals else order.astype(np.uint32)
        assert np.array_equal(vout.cpu().numpy().view(np.uint32), want_v)
    assert torch.equal(kin, kin0) and torch.equal(vin, vin0)


def test_single_rank_argsort_and_pairs(sorter):
    import os
    import socket
    import torch
    import torch.distributed as dist
    from forge_sort.samplesort import CudaOps, SampleSorter
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        x = orc.gen("zipf_u32", 50_000, seed=3)
        keys = torch.from_numpy(x.view(np.int32).copy()).cuda()
        ss = SampleSorter(CudaOps(sorter, torch), dtype="u32")
        idx = ss.argsort(keys, gpos_base=1000)
        assert np.array_equal(idx.cpu().numpy().view(np.uint32), orc.argsort(x, "u32").astype(np.uint32) + 1000)
        v = np.arange(50_000, dtype=np.uint32)[::-1].copy()
        k2, v2 = ss.sort_pairs(keys, torch.from_numpy(v.view(np.int32)).cuda())
        order = orc.argsort(x, "u32")
        assert np.array_equal(k2.cpu().numpy().view(np.uint32), x[order])
        assert np.array_equal(v2.cpu().numpy().view(np.uint32), v[order])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dt,dist,nspl,payload,with_vals", [("u32", "u32", 7, False, False),
                                                             ("f32", "f32_mix", 3, True, True),
                                                             ("u64", "u64", 1, True, False),
                                                             ("i64", "i64", 5, False, False)])
def test_async_count_and_matrix_dispatch(sorter, dt, dist, nspl, payload, with_vals):
    """fs_partition_count_async + fs_partition_dispatch_matrix, the host-wait-
    free form of the sample sort's exchange, as rank r of G ranks on one GPU:
    the counts land in device memory, and bucket b's keys (and values) land in
    inbox b after what the lower ranks send there (rows of the send matrix
    other than r are made up); nothing else in the inboxes is touched.  With
    a payload a bucket keeps the input order; keys alone may arrive in any
    order within their bucket (compared as multisets)."""
    import torch
    from forge_sort.samplesort import choose_splitters, ordered_bits
    G = nspl + 1
    rank = G // 2
    n, base = 250_003, 3_000_000
    x = orc.gen(dist, n, seed=11 + nspl)
    bits = orc.BITS_DTYPE[dt]
    iv = np.int32 if bits is np.uint32 else np.int64
    xb = np.ascontiguousarray(x).view(bits)
    per = 64
    pos = ((np.arange(per * G) + 0.5) * (n / (per * G))).astype(np.int64)
    samp_raw, samp_gpos = xb[pos], (pos + base).astype(np.uint64)
    picks = choose_splitters(ordered_bits(samp_raw, dt), samp_gpos, G, per)
    spl_raw, spl_gpos = samp_raw[picks], samp_gpos[picks]
    keys = torch.from_numpy(xb.view(iv).copy()).cuda()
    vals_h = orc.gen("u32", n, seed=5)
    vals = torch.from_numpy(vals_h.view(np.int32).copy()).cuda()
    sk = torch.from_numpy(spl_raw.view(iv).copy()).cuda()
    sg = torch.from_numpy(spl_gpos.view(np.int64).copy()).cuda()
    counts = torch.zeros(G, dtype=torch.int64, device="cuda")
    sorter.partition_count_async(dt, keys.data_ptr(), n, base, sk.data_ptr(), sg.data_ptr(), nspl, counts.data_ptr())
    want_k, wcounts = ref_partition(xb, dt, base, spl_raw, spl_gpos)
    assert counts.cpu().numpy().tolist() == wcounts.tolist()
    rng = np.random.default_rng(nspl)
    M = rng.integers(0, 5000, (G, G)).astype(np.int64)
    M[rank] = wcounts
    Mdev = torch.from_numpy(M).cuda()
    col = M.sum(axis=0)
    kb = keys.element_size()
    inbox_k = [torch.full((int(col[b]) + 16,), -1, dtype=keys.dtype, device="cuda") for b in range(G)]
    inbox_v = [torch.full((int(col[b]) + 16,), -1, dtype=torch.int32, device="cuda") for b in range(G)]
    sorter.partition_dispatch_matrix(dt, keys.data_ptr(), n, base, sk.data_ptr(), sg.data_ptr(), nspl,
                                     Mdev.data_ptr(), rank, [t.data_ptr() for t in inbox_k],
                                     [t.data_ptr() for t in inbox_v] if payload else None,
                                     vals_ptr=vals.data_ptr() if with_vals else 0, payload=payload, sync=True)
    o = ordered_bits(xb, dt)
    g = np.arange(n, dtype=np.uint64) + np.uint64(base)
    so = ordered_bits(spl_raw, dt)
    bk = np.zeros(n, np.int64)
    for j in range(nspl):
        bk += ((o > so[j]) | ((o == so[j]) & (g >= spl_gpos[j]))).astype(np.int64)
    order = np.argsort(bk, kind="stable")
    want_v = vals_h[order] if with_vals else (order + base).astype(np.uint32)
    starts = np.concatenate([[0], np.cumsum(wcounts)[:-1]])
    for b in range(G):
        lo = int(M[:rank, b].sum())
        c = int(wcounts[b])
        got = inbox_k[b].cpu().numpy().view(bits)
        if payload:
            assert np.array_equal(got[lo:lo + c], want_k[starts[b]:starts[b] + c]), b
        else:
            assert np.array_equal(np.sort(got[lo:lo + c]), np.sort(want_k[starts[b]:starts[b] + c])), b
        assert bool((inbox_k[b][:lo] == -1).all()) and bool((inbox_k[b][lo + c:] == -1).all()), b
        if payload:
            gv = inbox_v[b].cpu().numpy().view(np.uint32)
            assert np.array_equal(gv[lo:lo + c], want_v[starts[b]:starts[b] + c]), b
            assert bool((inbox_v[b][:lo] == -1).all()) and bool((inbox_v[b][lo + c:] == -1).all()), b
