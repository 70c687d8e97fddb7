"""Multi-GPU sample sort, bit-exact against the oracle (needs >= 2 GPUs; one
process per GPU under torchrun, NCCL, dispatch over CUDA IPC peer memory)."""
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sample_sort_matches_oracle(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "_mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "MISMATCH" not in r.stdout


MG_CASES = [("u32", "u32", 1 << 22, None), ("skew_u32", "u32", 1 << 22, None), ("zipf_u32", "u32", 3_000_017, None),
            ("f32_mix", "f32", 1 << 21, None), ("i32", "i32", 1_000_003, "ragged"), ("u64", "u64", 1 << 21, None),
            ("f64_logu", "f64", 1 << 20, None), ("i64", "i64", 777_777, "one_empty")]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_sorter_one_process_matches_oracle(world):
    """fs_mg_sort_keys: the same sample sort driven from one process over
    `world` devices with peer access; pieces concatenated == oracle sort."""
    import numpy as np
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    import forge_sort
    from oracle import oracle as orc
    from tests._mgpu_worker import shard_bounds
    mg = forge_sort.MultiGpuSorter(list(range(world)))
    try:
        for gen, dt, n, mode in MG_CASES:
            full = orc.gen(gen, n, seed=42)
            cuts = shard_bounds(n, world, mode)
            iv = np.int32 if full.itemsize == 4 else np.int64
            shards = [torch.from_numpy(np.ascontiguousarray(full[cuts[i]:cuts[i + 1]]).view(iv)).to(f"cuda:{i}")
                      for i in range(world)]
            pieces = mg.sort(dt, shards) if dt != "u32" else mg.sort_u32(shards)
            got = np.concatenate([p.cpu().numpy() for p in pieces]).view(orc.BITS_DTYPE[dt])
            want = orc.sort_keys(full, dt).view(orc.BITS_DTYPE[dt])
            assert np.array_equal(got, want), (gen, dt, [p.numel() for p in pieces])
            mean = n / world
            if mode is None and gen != "zipf_u32":
                assert max(p.numel() for p in pieces) < 1.1 * mean + 1024  # regular-sampling balance
    finally:
        mg.close()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_sorter_argsort_and_pairs_stable(world):
    """fs_mg_sort_pairs: values (or global positions) travel with the keys;
    the pieces concatenated equal the oracle's stable order of the whole
    input, Zipf duplicates split across devices included."""
    import numpy as np
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs, {torch.cuda.device_count()} visible")
    import forge_sort
    from oracle import oracle as orc
    from tests._mgpu_worker import scrambled_values, shard_bounds
    mg = forge_sort.MultiGpuSorter(list(range(world)))
    try:
        for gen, dt, n, mode in [("zipf_u32", "u32", 2_000_003, None), ("f64_logu", "f64", 1 << 20, "one_empty"),
                                 ("i32", "i32", 1_000_003, "ragged")]:
            full = orc.gen(gen, n, seed=42)
            cuts = shard_bounds(n, world, mode)
            iv = np.int32 if full.itemsize == 4 else np.int64
            shards = [torch.from_numpy(np.ascontiguousarray(full[cuts[i]:cuts[i + 1]]).view(iv)).to(f"cuda:{i}")
                      for i in range(world)]
            order = orc.argsort(full, dt)
            bits = orc.BITS_DTYPE[dt]
            keys, pos = mg.argsort(dt, shards)
            assert np.array_equal(np.concatenate([k.cpu().numpy() for k in keys]).view(bits),
                                  np.ascontiguousarray(full[order]).view(bits)), gen
            assert np.array_equal(np.concatenate([p.cpu().numpy() for p in pos]).view(np.uint32),
                                  order.astype(np.uint32)), gen
            vals = [torch.from_numpy(scrambled_values(int(cuts[i]), int(cuts[i + 1])).view(np.int32)).to(f"cuda:{i}")
                    for i in range(world)]
            keys, vout = mg.sort_pairs(dt, shards, vals)
            assert np.array_equal(np.concatenate([k.cpu().numpy() for k in keys]).view(bits),
                                  np.ascontiguousarray(full[order]).view(bits)), gen
            assert np.array_equal(np.concatenate([v.cpu().numpy() for v in vout]).view(np.uint32),
                                  scrambled_values(0, n)[order]), gen
    finally:
        mg.close()
