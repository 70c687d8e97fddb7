"""Multi-GPU sample-sort host logic on CPU ranks (gloo, world sizes 2 and 3).

The orchestration in forge_sort.samplesort (sampling, splitter choice with
the (key, global position) tie-break, size exchange, all-to-all) runs for
real; the two GPU steps (partition, local sort) are replaced by a numpy
stand-in and the result is checked against the oracle's sort of the whole
input.  No GPU."""
import os
import socket

import numpy as np
import pytest

N_PER_RANK = 20_000


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class CpuOps:
    """Host stand-in for CudaOps (test only)."""

    def __init__(self, torch):
        self.torch = torch

    def partition(self, dt, keys, gpos_base, spl_raw, spl_gpos):
        from forge_sort.samplesort import ordered_bits
        x = keys.numpy()
        o = ordered_bits(x, dt)
        g = np.arange(x.size, dtype=np.uint64) + np.uint64(gpos_base)
        so = ordered_bits(spl_raw, dt)
        bucket = np.zeros(x.size, np.int64)
        for j in range(len(spl_gpos)):
            bucket += ((o > so[j]) | ((o == so[j]) & (g >= spl_gpos[j]))).astype(np.int64)
        idx = np.argsort(bucket, kind="stable")
        counts = np.bincount(bucket, minlength=len(spl_gpos) + 1)
        return self.torch.from_numpy(x[idx].copy()), [int(c) for c in counts]

    def partition_pairs(self, dt, keys, vals, gpos_base, spl_raw, spl_gpos):
        from forge_sort.samplesort import ordered_bits
        x = keys.numpy()
        o = ordered_bits(x, dt)
        g = np.arange(x.size, dtype=np.uint64) + np.uint64(gpos_base)
        so = ordered_bits(spl_raw, dt)
        bucket = np.zeros(x.size, np.int64)
        for j in range(len(spl_gpos)):
            bucket += ((o > so[j]) | ((o == so[j]) & (g >= spl_gpos[j]))).astype(np.int64)
        idx = np.argsort(bucket, kind="stable")
        counts = np.bincount(bucket, minlength=len(spl_gpos) + 1)
        return (self.torch.from_numpy(x[idx].copy()), self.torch.from_numpy(vals.numpy()[idx].copy()),
                [int(c) for c in counts])

    def sort(self, dt, keys):
        from oracle import oracle as orc
        x = keys.numpy()
        bits = np.uint32 if x.dtype.itemsize == 4 else np.uint64
        npdt = orc.NP_DTYPE[dt]
        s = orc.sort_keys(x.view(bits).view(npdt), dt)
        return self.torch.from_numpy(s.view(x.dtype).copy())

    def sort_pairs(self, dt, keys, vals):
        from oracle import oracle as orc
        x = keys.numpy()
        bits = np.uint32 if x.dtype.itemsize == 4 else np.uint64
        order = orc.argsort(x.view(bits).view(orc.NP_DTYPE[dt]), dt)  # stable
        v = vals.numpy() if vals is not None else np.arange(x.size, dtype=np.int32)
        return self.torch.from_numpy(x[order].copy()), self.torch.from_numpy(v[order].copy())


def _worker(rank, world, port, dist_name, dt, result_path, per_rank_sizes, mode="keys"):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "gpu-forge_b200"), root]
    import torch
    import torch.distributed as tdist
    from forge_sort.samplesort import SampleSorter
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start = sum(per_rank_sizes[:rank])
        m = per_rank_sizes[rank]
        x = orc.gen(dist_name, sum(per_rank_sizes), seed=5)[start:start + m]
        bits = np.uint32 if x.dtype.itemsize == 4 else np.uint64
        t = torch.from_numpy(np.ascontiguousarray(x).view(bits).view(np.int32 if bits is np.uint32 else np.int64))
        ss = SampleSorter(CpuOps(torch), dtype=dt, samples_per_rank=512)
        if mode == "keys":
            out = ss.sort(t)
        elif mode == "argsort":
            np.save(f"{result_path}.{rank}.v.npy", ss.argsort(t).numpy())
            out = t[:0]
        else:  # pairs: value = a scrambled global position
            v = ((np.arange(start, start + m, dtype=np.uint64) * 2654435761) & 0xFFFFFFFF).astype(np.uint32)
            out, vout = ss.sort_pairs(t, torch.from_numpy(v.view(np.int32)))
            np.save(f"{result_path}.{rank}.v.npy", vout.numpy())
        np.save(f"{result_path}.{rank}.npy", out.numpy())
    finally:
        tdist.destroy_process_group()


def _run(world, dist_name, dt, tmp_path, per_rank_sizes=None, mode="keys"):
    import torch.multiprocessing as mp
    sizes = per_rank_sizes or [N_PER_RANK] * world
    path = str(tmp_path / "out")
    mp.start_processes(_worker, args=(world, _free_port(), dist_name, dt, path, sizes, mode), nprocs=world,
                       start_method="spawn")
    from oracle import oracle as orc
    x = orc.gen(dist_name, sum(sizes), seed=5)
    bits = np.uint32 if x.dtype.itemsize == 4 else np.uint64
    if mode != "keys":
        order = orc.argsort(x, dt)  # the stable global order
        vals = [np.load(f"{path}.{r}.v.npy").view(np.uint32) for r in range(world)]
        got_v = np.concatenate(vals)
        if mode == "argsort":
            assert np.array_equal(got_v, order.astype(np.uint32))
            return [p.size for p in vals]
        v_all = ((np.arange(x.size, dtype=np.uint64) * 2654435761) & 0xFFFFFFFF).astype(np.uint32)
        assert np.array_equal(got_v, v_all[order])
    want = orc.sort_keys(x, dt)
    pieces = [np.load(f"{path}.{r}.npy").view(bits) for r in range(world)]
    got = np.concatenate(pieces)
    assert np.array_equal(got, want.view(bits))
    return [p.size for p in pieces]


@pytest.mark.parametrize("world", [2, 3])
def test_uniform_u32(world, tmp_path):
    sizes = _run(world, "u32", "u32", tmp_path)
    assert max(sizes) < 1.25 * N_PER_RANK  # regular sampling keeps buckets near n/G


def test_skewed_u32_70pct_in_one_range(tmp_path):
    sizes = _run(2, "skew_u32", "u32", tmp_path)
    assert max(sizes) < 1.25 * N_PER_RANK


def test_all_duplicates_still_split_by_position(tmp_path):
    # zipf keys: most mass on a few values; the (key, position) tie-break
    # still divides equal keys between ranks
    sizes = _run(2, "zipf_u32", "u32", tmp_path)
    assert max(sizes) < 1.25 * N_PER_RANK


@pytest.mark.parametrize("dt,dist_name", [("f64", "f64_logu"), ("i64", "i64"), ("f32", "f32_mix")])
def test_other_key_types(dt, dist_name, tmp_path):
    _run(2, dist_name, dt, tmp_path)


def test_uneven_and_empty_shards(tmp_path):
    _run(3, "u32", "u32", tmp_path, per_rank_sizes=[25_000, 0, 7_000])


@pytest.mark.parametrize("mode", ["argsort", "pairs"])
@pytest.mark.parametrize("dist_name,dt", [("zipf_u32", "u32"), ("f32_mix", "f32"), ("i64", "i64")])
def test_argsort_and_pairs_globally_stable(mode, dist_name, dt, tmp_path):
    """Multi-rank argsort / sort_pairs equal the stable sort_by_key of the
    whole input: heavy duplicates (zipf) split across ranks keep their global
    input order."""
    _run(2, dist_name, dt, tmp_path, mode=mode)


def test_argsort_uneven_and_empty_shards(tmp_path):
    _run(3, "zipf_u32", "u32", tmp_path, per_rank_sizes=[25_000, 0, 7_000], mode="argsort")


@pytest.mark.parametrize("distinct", [7, 1000, 1 << 40])
def test_choose_splitters_matches_lexicographic_order(distinct):
    """Splitter picks equal the per_rank-th tuples of a full (key, position)
    lexicographic sort, with heavy, light and no key duplication."""
    from forge_sort.samplesort import choose_splitters
    rng = np.random.default_rng(distinct % 97)
    G, S = 8, 512
    keys = rng.integers(0, distinct, G * S, dtype=np.uint64)
    gpos = rng.permutation(G * S * 3)[: G * S].astype(np.uint64)
    order = np.lexsort((gpos, keys))
    want = [order[j * S] for j in range(1, G)]
    got = choose_splitters(keys, gpos, G, S)
    assert [(keys[i], gpos[i]) for i in got] == [(keys[i], gpos[i]) for i in want]


@pytest.mark.parametrize("dt", ["u32", "i32", "f32", "u64", "i64", "f64"])
def test_sample_sort_keys_order_matches_ordered_bits(dt):
    """The device-side sample keys (signed int64 order) sort like the
    oracle's order transform."""
    import torch
    from forge_sort.samplesort import ordered_bits, sample_sort_keys
    from oracle import oracle as orc
    gen = {"u32": "u32", "i32": "i32", "f32": "f32_mix", "u64": "u64", "i64": "i64", "f64": "f64_logu"}[dt]
    x = orc.gen(gen, 5000, seed=11)
    iv = np.int32 if x.itemsize == 4 else np.int64
    k = sample_sort_keys(torch, torch.from_numpy(np.ascontiguousarray(x).view(iv)), dt).numpy()
    o = ordered_bits(x, dt)
    assert np.array_equal(np.argsort(k, kind="stable"), np.argsort(o, kind="stable"))
