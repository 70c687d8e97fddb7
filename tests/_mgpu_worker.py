"""Worker of tests/test_gpu_multi.py: one process per GPU (torchrun), NCCL.

Every rank builds the whole seeded input with the oracle's generators, takes
its shard (ragged sizes, one rank possibly empty), runs the sample sort
(fs_partition_count + fs_partition_dispatch into the peers' inboxes, local
radix sort), and rank 0 checks the concatenated pieces bit for bit against the
oracle's sort of the whole input.  The payload cases (argsort, sort_pairs)
carry a u32 per key through fs_partition_dispatch_pairs and a stable local
pairs sort, and are checked against the oracle's stable order of the whole
input.  Exit code 0 = every case matched."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "gpu-forge_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import forge_sort  # noqa: E402
from forge_sort.samplesort import CudaOps, SampleSorter  # noqa: E402
from oracle import oracle as orc  # noqa: E402

CASES = [  # (generator, dtype, total keys, shard weights)
    ("u32", "u32", 1 << 22, None),
    ("skew_u32", "u32", 1 << 22, None),
    ("zipf_u32", "u32", 3_000_017, None),
    ("f32_mix", "f32", 1 << 21, None),
    ("i32", "i32", 1_000_003, "ragged"),
    ("u64", "u64", 1 << 21, None),
    ("f64_logu", "f64", 1 << 20, None),
    ("i64", "i64", 777_777, "one_empty"),
]
PAYLOAD_CASES = [  # (generator, dtype, total keys, shard weights, "argsort" | "pairs")
    ("zipf_u32", "u32", 3_000_017, None, "argsort"),
    ("f32_mix", "f32", 1 << 21, "ragged", "pairs"),
    ("u64", "u64", 1 << 20, None, "argsort"),
    ("i64", "i64", 777_777, "one_empty", "pairs"),
]


def scrambled_values(lo, hi):
    return ((np.arange(lo, hi, dtype=np.uint64) * 2654435761) & 0xFFFFFFFF).astype(np.uint32)


def shard_bounds(n, world, mode):
    if mode == "ragged":
        w = np.arange(1, world + 1, dtype=np.float64)
    elif mode == "one_empty":
        w = np.ones(world)
        w[-1] = 0.0
    else:
        w = np.ones(world)
    cuts = np.concatenate([[0], np.floor(np.cumsum(w) / w.sum() * n).astype(np.int64)])
    cuts[-1] = n
    return cuts


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    sorter = forge_sort.GpuSorter.with_context(local, torch.cuda.current_stream(dev).cuda_stream)
    bad = []
    ss = None

    def gather_all(piece):
        """Every rank's piece, concatenated in rank order (padded all_gather)."""
        size = torch.tensor([piece.numel()], dtype=torch.int64, device=dev)
        sizes = [torch.empty_like(size) for _ in range(world)]
        dist.all_gather(sizes, size)
        sizes = [int(x.item()) for x in sizes]
        pad = torch.zeros(max(max(sizes), 1), dtype=piece.dtype, device=dev)
        pad[: piece.numel()] = piece
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        return np.concatenate([p[:k].cpu().numpy() for p, k in zip(parts, sizes)]), sizes

    for gen, dt, n, mode, what in PAYLOAD_CASES:
        full = orc.gen(gen, n, seed=42)
        cuts = shard_bounds(n, world, mode)
        lo, hi = int(cuts[rank]), int(cuts[rank + 1])
        iv = np.int32 if full.itemsize == 4 else np.int64
        shard = torch.from_numpy(np.ascontiguousarray(full[lo:hi]).view(iv)).to(dev)
        ss = SampleSorter(CudaOps(sorter, torch), dtype=dt, samples_per_rank=1024)
        order = orc.argsort(full, dt) if rank == 0 else None
        if what == "argsort":
            got_v, sizes = gather_all(ss.argsort(shard, gpos_base=lo))
            ok = rank != 0 or np.array_equal(got_v.view(np.uint32), order.astype(np.uint32))
        else:
            vals = torch.from_numpy(scrambled_values(lo, hi).view(np.int32)).to(dev)
            k, v = ss.sort_pairs(shard, vals, gpos_base=lo)
            got_k, sizes = gather_all(k)
            got_v, _ = gather_all(v)
            ok = rank != 0 or (np.array_equal(got_k.view(orc.BITS_DTYPE[dt]), full[order].view(orc.BITS_DTYPE[dt]))
                               and np.array_equal(got_v.view(np.uint32), scrambled_values(0, n)[order]))
        ss.close()
        if rank == 0:
            print(f"{what} {gen}/{dt} n={n} shards={mode or 'even'} pieces={sizes}: {'ok' if ok else 'MISMATCH'}",
                  flush=True)
            if not ok:
                bad.append(f"{what}/{gen}")

    for gen, dt, n, mode in CASES:
        full = orc.gen(gen, n, seed=42)
        cuts = shard_bounds(n, world, mode)
        lo, hi = int(cuts[rank]), int(cuts[rank + 1])
        tdt = torch.int32 if full.itemsize == 4 else torch.int64
        shard = torch.from_numpy(np.ascontiguousarray(full[lo:hi]).view(
            np.int32 if full.itemsize == 4 else np.int64)).to(dev)
        ss = SampleSorter(CudaOps(sorter, torch), dtype=dt, samples_per_rank=1024)
        piece = ss.sort(shard, gpos_base=lo)
        # gather the pieces on every rank (padded all_gather)
        size = torch.tensor([piece.numel()], dtype=torch.int64, device=dev)
        sizes = [torch.empty_like(size) for _ in range(world)]
        dist.all_gather(sizes, size)
        sizes = [int(x.item()) for x in sizes]
        pad = torch.zeros(max(sizes), dtype=tdt, device=dev)
        pad[: piece.numel()] = piece
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        ss.close()
        if rank == 0:
            got = np.concatenate([p[:k].cpu().numpy() for p, k in zip(parts, sizes)])
            want = orc.sort_keys(full, dt)
            ok = got.size == want.size and np.array_equal(got.view(orc.BITS_DTYPE[dt]), want.view(orc.BITS_DTYPE[dt]))
            print(f"{gen}/{dt} n={n} shards={mode or 'even'} pieces={sizes}: {'ok' if ok else 'MISMATCH'}", flush=True)
            if not ok:
                bad.append(gen)
    flag = torch.tensor([len(bad)], dtype=torch.int32, device=dev)
    dist.broadcast(flag, 0)
    sorter.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(1 if int(flag.item()) else 0)


if __name__ == "__main__":
    main()
