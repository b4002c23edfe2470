"""The benchmark's whole-job figures over several ranks (bench.whole_job): the slowest rank's time
and the sum of every rank's work and bytes, as the multi-GPU bench line reports them. Run here as
world-size-2 gloo ranks on CPU."""
import os
import socket
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, result_path):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        times = [100.0 + 7 * rank, 50.0 - rank]           # rank 1 slower on the first, faster on the second
        work = [1e9 * (rank + 1), 3.0 + rank]
        mx, sm = bench.whole_job(times, work, world, "cpu")
        if rank == 0:
            np.save(result_path, np.array(mx + sm))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_whole_job_over_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "r.npy")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    assert np.load(out).tolist() == [107.0, 50.0, 3e9, 7.0]


def test_whole_job_single_rank_passes_through():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.whole_job([1.5, 2], [3, 4.25], 1, None) == ([1.5, 2.0], [3.0, 4.25])
