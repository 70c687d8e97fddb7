"""Rank failures in the multi-GPU sample sort's host logic, on CPU ranks
(gloo, world size 3, no GPU).

One rank is made to fail on the host -- its local partition step raises,
stalls past the process group's timeout, or the process exits before the
exchange -- and every other rank must come back with SortError::GpuExecution
naming the collective that failed, within a deadline, instead of hanging.
The parent kills anything still alive at the deadline and fails the test."""
import json
import os
import socket
import time

import pytest

from test_samplesort_gloo import CpuOps

WORLD = 3
BAD = 1
PG_TIMEOUT_S = 4
DEADLINE_S = 90


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class FailingOps(CpuOps):
    """CpuOps whose partition step fails in the given way on one rank."""

    def __init__(self, torch, mode):
        super().__init__(torch)
        self.mode = mode

    def partition(self, dt, keys, gpos_base, spl_raw, spl_gpos):
        if self.mode == "raise":
            raise RuntimeError("injected failure in the local partition step")
        if self.mode == "exit":
            os._exit(3)
        if self.mode == "stall":
            time.sleep(3 * PG_TIMEOUT_S)
        return super().partition(dt, keys, gpos_base, spl_raw, spl_gpos)


def _worker(rank, world, port, mode, result_path):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "gpu-forge_b200"), root, os.path.join(root, "tests")]
    import numpy as np
    import torch
    import torch.distributed as tdist
    from forge_sort.errors import GpuExecution
    from forge_sort.samplesort import SampleSorter
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world,
                             timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    rec = {"rank": rank}
    t0 = time.time()
    try:
        x = orc.gen("u32", 3000 * world, seed=5)[rank * 3000:(rank + 1) * 3000]
        t = torch.from_numpy(np.ascontiguousarray(x).view(np.int32))
        ops = FailingOps(torch, mode if rank == BAD else "ok")
        ss = SampleSorter(ops, dtype="u32", samples_per_rank=64)
        ss.sort(t)
        rec["result"] = "ok"
    except GpuExecution as e:
        rec["result"] = "GpuExecution"
        rec["text"] = str(e)
    except Exception as e:  # noqa: BLE001 -- recorded for the parent's assertion
        rec["result"] = type(e).__name__
        rec["text"] = str(e)
    rec["seconds"] = time.time() - t0
    with open(f"{result_path}.{rank}.json", "w") as f:
        json.dump(rec, f)
    try:
        tdist.destroy_process_group()
    except Exception:  # noqa: BLE001 -- the group may already be broken
        pass
    os._exit(0)  # do not wait for peers in interpreter teardown


@pytest.mark.parametrize("mode", ["raise", "stall", "exit"])
def test_other_ranks_fail_fast_when_one_rank_fails(mode, tmp_path):
    import torch.multiprocessing as mp
    path = str(tmp_path / "rec")
    ctx = mp.start_processes(_worker, args=(WORLD, _free_port(), mode, path), nprocs=WORLD,
                             start_method="spawn", join=False)
    end = time.time() + DEADLINE_S
    procs = ctx.processes
    while time.time() < end and any(p.is_alive() for p in procs):
        time.sleep(0.2)
    hung = [i for i, p in enumerate(procs) if p.is_alive()]
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(5)
    assert not hung, f"ranks {hung} still running after {DEADLINE_S} s"
    for r in range(WORLD):
        if r == BAD:
            continue
        with open(f"{path}.{r}.json") as f:
            rec = json.load(f)
        assert rec["result"] == "GpuExecution", rec
        assert "collective" in rec["text"], rec
        assert rec["seconds"] < DEADLINE_S - 10, rec
    if mode == "raise":
        with open(f"{path}.{BAD}.json") as f:
            bad = json.load(f)
        assert bad["result"] == "RuntimeError" and "injected" in bad["text"], bad
