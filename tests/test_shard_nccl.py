"""Native multi-GPU sharding (lb200_shard_run over an NCCL communicator made
by the engine library), on the GPU."""
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

import golden_cases as G
from luna_b200 import abi, workloads as W

pytestmark = pytest.mark.gpu


def _case():
    g, bx = W.small_cnn_case(2, n_boxes=7, big_first=False)
    return g, bx, abi.default_options(alpha_lr=0.1, alpha_iterations=4)


def test_single_rank_shard_run_matches_compute_bounds():
    from luna_b200.build import build
    from luna_b200.engine import Model, NcclComm, nccl_unique_id
    build()
    g, bx, opt = _case()
    m = Model(g, device=0, options=opt)
    ref = m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    comm = NcclComm(nccl_unique_id(), 0, 1, 0)
    try:
        lb, ub = m.shard_run(comm, bx, abi.METHOD_ALPHA_CROWN, timeout_ms=30000)
    finally:
        comm.close()
    assert np.array_equal(lb, ref[0]) and np.array_equal(ub, ref[1])


def _rank(rank, world, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from luna_b200.engine import Model, NcclComm
    g, bx, opt = _case()
    m = Model(g, device=rank, options=opt)
    comm = NcclComm(uid, rank, world, rank)
    try:
        q.put((rank, m.shard_run(comm, bx, abi.METHOD_ALPHA_CROWN, timeout_ms=30000)))
    finally:
        comm.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_gather_every_box():
    """Two processes, one GPU each: every rank ends with the bounds of every
    box, equal to one GPU bounding the whole batch."""
    from luna_b200.build import build
    from luna_b200.engine import Model, nccl_unique_id
    build()
    g, bx, opt = _case()
    ref = Model(g, device=0, options=opt).compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        lb, ub = out[r]
        G.parity(f"shard rank {r}", lb, ub, ref[0], ref[1])


def _rank_absent(rank, world, uid, q, gone):
    """Both ranks bound and gather a first batch; then rank 1 leaves the job
    between steps: it stays alive, with nothing in flight, until rank 0 has
    reported, and never touches the communicator again.  Rank 0's second
    gather must end at its bounded wait."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from luna_b200.engine import EngineError, Model, NcclComm
    g, bx, opt = _case()
    m = Model(g, device=rank, options=opt)
    comm = NcclComm(uid, rank, world, rank)
    first = m.shard_run(comm, bx, abi.METHOD_ALPHA_CROWN, timeout_ms=30000)
    if rank == 0:
        try:
            m.shard_run(comm, bx, abi.METHOD_ALPHA_CROWN, timeout_ms=3000)
            q.put((0, "no error", first, None))
        except EngineError as e:
            # The model stays usable after the aborted gather.
            q.put((0, str(e) + (" | handle released" if comm.handle is None else ""), first,
                   m.compute_bounds(bx, abi.METHOD_ALPHA_CROWN)))
        gone.set()
    else:
        q.put((1, "left", first, None))
        gone.wait(timeout=120)
    os._exit(0)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_absent_rank_times_out_the_gather():
    """A rank that leaves between steps: the other's next gather ends at its
    bounded wait, the communicator is aborted, the call fails with an error,
    and its model still bounds correctly.  NVLS off (NCCL_NVLS_ENABLE=0)."""
    import queue

    from luna_b200.build import build
    from luna_b200.engine import Model, nccl_unique_id
    build()
    g, bx, opt = _case()
    ref = Model(g, device=0, options=opt).compute_bounds(bx, abi.METHOD_ALPHA_CROWN)
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    gone = ctx.Event()
    procs = [ctx.Process(target=_rank_absent, args=(r, 2, uid, q, gone)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in procs:
            r, msg, first, res = q.get(timeout=180)
            out[r] = (msg, first, res)
        for p in procs:
            p.join(timeout=120)
    except queue.Empty:
        pass
    finally:
        # A rank still running here is stuck: end it so the test reports
        # instead of waiting on its process at exit.
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    assert sorted(out) == [0, 1], f"ranks that reported: {sorted(out)}"
    assert all(p.exitcode == 0 for p in procs)
    for r in range(2):
        G.parity(f"first step rank {r}", out[r][1][0], out[r][1][1], ref[0], ref[1])
    msg, _, res = out[0]
    assert "timed out" in msg and "aborted" in msg and "handle released" in msg, msg
    G.parity("after the aborted gather", res[0], res[1], ref[0], ref[1])
