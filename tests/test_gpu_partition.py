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
