"""Resumable sub-domain sweeps (luna_b200/sweep.py): the on-disk chunk files,
resume after an interruption, refusal of a different sweep, damaged files,
and two ranks sharing one directory.  CPU only: the bounder is a stand-in
whose bounds are a function of the sub-domain, so every check is exact."""
import multiprocessing as mp
import os

import numpy as np
import pytest

from luna_b200 import abi
from luna_b200.sweep import SweepDir, run_sweep
from luna_b200.workloads import SubdomainSplit


def _split(groups=6, n_in=12):
    rng = np.random.default_rng(0)
    lo = rng.uniform(-1, 0, n_in).astype(np.float32)
    hi = (lo + 1).astype(np.float32)
    C = np.zeros((1, 3, 4), np.float32)
    C[0, :, 0] = 1
    C[0, [0, 1, 2], [1, 2, 3]] = -1
    g = np.arange(groups * 2).reshape(groups, 2) % n_in
    return SubdomainSplit(lo, hi, (lo + hi) / 2, C, g)


class FakeModel:
    """Bounds that identify the box: lb row j = sum(lower) + j, ub = sum(upper) + j."""

    def __init__(self):
        self.calls = 0

    def compute_bounds(self, boxes, method):
        self.calls += 1
        nspec = boxes.C.shape[1]
        lb = boxes.lower.sum(1, keepdims=True) + np.arange(nspec, dtype=np.float32)
        ub = boxes.upper.sum(1, keepdims=True) + np.arange(nspec, dtype=np.float32)
        return lb.astype(np.float32), ub.astype(np.float32)


def _expected(split):
    bx = split.boxes(0, split.count)
    return FakeModel().compute_bounds(bx, 0)


def test_resume_after_interruption(tmp_path):
    split = _split()
    m = FakeModel()
    sd = run_sweep(m, split, abi.METHOD_CROWN, str(tmp_path), chunk=10, max_chunks=3)
    assert m.calls == 3 and len(sd.pending()) == sd.n_chunks - 3
    with pytest.raises(RuntimeError):
        sd.collect()
    m2 = FakeModel()
    sd = run_sweep(m2, split, abi.METHOD_CROWN, str(tmp_path), chunk=10)
    assert m2.calls == sd.n_chunks - 3 and sd.pending() == []
    lb, ub, st = sd.collect()
    elb, eub = _expected(split)
    assert np.array_equal(lb, elb) and np.array_equal(ub, eub) and st is None
    # Nothing left: a further call bounds nothing.
    m3 = FakeModel()
    run_sweep(m3, split, abi.METHOD_CROWN, str(tmp_path), chunk=10)
    assert m3.calls == 0


def test_different_sweep_is_refused(tmp_path):
    split = _split()
    run_sweep(FakeModel(), split, abi.METHOD_CROWN, str(tmp_path), chunk=10, max_chunks=1)
    with pytest.raises(ValueError):
        run_sweep(FakeModel(), split, abi.METHOD_CROWN, str(tmp_path), chunk=16)
    with pytest.raises(ValueError):
        run_sweep(FakeModel(), split, abi.METHOD_ALPHA_CROWN, str(tmp_path), chunk=10)


def test_damaged_chunk_is_redone(tmp_path):
    split = _split()
    sd = run_sweep(FakeModel(), split, abi.METHOD_CROWN, str(tmp_path), chunk=10)
    f = os.path.join(str(tmp_path), "chunk_000002.npz")
    with open(f, "r+b") as fh:
        fh.truncate(40)                                       # a torn write
    with open(os.path.join(str(tmp_path), "chunk_000004.npz.tmp123"), "wb") as fh:
        fh.write(b"partial")                                 # a leftover temporary file
    assert sd.pending() == [2]
    m = FakeModel()
    sd = run_sweep(m, split, abi.METHOD_CROWN, str(tmp_path), chunk=10)
    assert m.calls == 1
    lb, ub, _ = sd.collect()
    assert np.array_equal(lb, _expected(split)[0])


def test_chunk_with_wrong_ids_counts_as_missing(tmp_path):
    sd = SweepDir(str(tmp_path), 25, 10, 3)
    sd.write(0, np.zeros((10, 3)), np.ones((10, 3)))
    os.replace(os.path.join(str(tmp_path), "chunk_000000.npz"), os.path.join(str(tmp_path), "chunk_000001.npz"))
    assert not sd.done(1) and sd.pending() == [0, 1, 2]
    with pytest.raises(ValueError):
        sd.write(2, np.zeros((10, 3)), np.zeros((10, 3)))     # the last chunk holds 5 sub-domains


def _rank_worker(rank, world, path):
    split = _split()
    run_sweep(FakeModel(), split, abi.METHOD_CROWN, path, chunk=7, rank=rank, world=world)


def test_two_ranks_share_one_directory(tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    split = _split()
    sd = SweepDir(str(tmp_path), split.count, 7, 3, {"method": abi.METHOD_CROWN, "property": False})
    lb, ub, _ = sd.collect()
    elb, eub = _expected(split)
    assert np.array_equal(lb, elb) and np.array_equal(ub, eub)
    # Each rank took its own chunks: rank 1 alone has nothing left to do.
    assert sd.pending(1, 2) == [] and sd.pending(0, 2) == []


class InjectedFailure(Exception):
    pass


class FailingModel(FakeModel):
    """FakeModel that raises on its call number `fail_at` (1-based)."""

    def __init__(self, fail_at):
        super().__init__()
        self.fail_at = fail_at

    def compute_bounds(self, boxes, method):
        if self.calls + 1 == self.fail_at:
            raise InjectedFailure("injected")
        return super().compute_bounds(boxes, method)


def _gloo_rank(rank, world, port, path, fail_rank, fail_at, out):
    import datetime

    import torch.distributed as dist

    from luna_b200.sweep import finish_ranks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    split = _split()
    model = FailingModel(fail_at) if rank == fail_rank else FakeModel()
    try:
        sd = run_sweep(model, split, abi.METHOD_CROWN, path, chunk=3, rank=rank, world=world)
    except InjectedFailure:
        os._exit(3)  # the rank dies between chunks, before the end-of-sweep barrier
    try:
        missing = finish_ranks(sd, world, timeout_s=5)
        msg = f"ok {len(missing)} {model.calls}"
    except RuntimeError as e:
        msg = f"failed {e}"
    with open(f"{out}.{rank}", "w") as f:
        f.write(msg)
    os._exit(0)


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(world, path, fail_rank, fail_at, out):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, path, fail_rank, fail_at, out))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    return [p.exitcode for p in procs]


@pytest.mark.timeout(300)
def test_failed_gloo_rank_is_resumed(tmp_path):
    """Rank 1 of two gloo ranks raises after one chunk: it exits, rank 0
    finishes its own chunks and learns of the failure at the end-of-sweep
    barrier, with the lost chunks named.  A rerun of the sweep bounds only
    those chunks (rank 0 has none left), and the collected result equals one
    uninterrupted sweep."""
    path = str(tmp_path / "sweep")
    out = str(tmp_path / "msg")
    codes = _launch(2, path, fail_rank=1, fail_at=2, out=out)
    assert codes == [0, 3]
    with open(out + ".0") as f:
        msg = f.read()
    assert msg.startswith("failed a rank did not reach the end of the sweep"), msg
    split = _split()
    sd = SweepDir(path, split.count, 3, 3, {"method": abi.METHOD_CROWN, "property": False})
    lost = sd.pending(1, 2)
    assert sd.pending(0, 2) == [] and len(lost) == len(range(1, sd.n_chunks, 2)) - 1
    assert f"{len(lost)} of {sd.n_chunks} chunks pending" in msg
    codes = _launch(2, path, fail_rank=-1, fail_at=0, out=out)
    assert codes == [0, 0]
    for r, calls in ((0, 0), (1, len(lost))):
        with open(f"{out}.{r}") as f:
            assert f.read() == f"ok 0 {calls}"
    lb, ub, _ = sd.collect()
    elb, eub = _expected(split)
    assert np.array_equal(lb, elb) and np.array_equal(ub, eub)
