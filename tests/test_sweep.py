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
