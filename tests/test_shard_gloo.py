"""The multi-rank path on CPU: two gloo ranks each bound their shard of the
boxes (with the CPU oracle standing in for the GPU engine) and gather the
final bounds; the result must equal bounding all boxes in one process."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from luna_b200 import abi, workloads as W
from luna_b200.shard import gather_bounds, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 512, 1000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(r, world, n) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        from oracle.lirpa_oracle import LirpaOracle
        g, bx = W.mlp_5_50x6_5(10)
        counts = [b - a for a, b in (shard_range(r, world, bx.n) for r in range(world))]
        a, b = shard_range(rank, world, bx.n)
        lb, ub = LirpaOracle(g).compute_bounds(bx.slice(a, b), abi.METHOD_CROWN)
        glb, gub = gather_bounds(torch.from_numpy(lb), torch.from_numpy(ub), counts)
        if rank == 0:
            np.save(out_path, np.stack([glb.numpy(), gub.numpy()]))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_gloo_ranks_gather_equals_single_process(tmp_path):
    out = str(tmp_path / "gathered.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn", join=True)
    from oracle.lirpa_oracle import LirpaOracle
    g, bx = W.mlp_5_50x6_5(10)
    lb, ub = LirpaOracle(g).compute_bounds(bx, abi.METHOD_CROWN)
    got = np.load(out)
    np.testing.assert_array_equal(got[0], lb)
    np.testing.assert_array_equal(got[1], ub)
