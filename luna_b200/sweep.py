"""Resumable sub-domain sweeps: bound every sub-domain of a split box in
chunks, one result file per chunk, so an interrupted sweep picks up where it
stopped.

Luna keeps branch-and-bound state in memory only (TorchModel::getState /
loadState, src/engine/TorchModel.cpp:975-1084) and writes nothing to disk.
A sweep here is a directory:

    manifest.json          what is being swept: sub-domain count, chunk size,
                           rows per sub-domain, method and the caller's
                           description; a resume with a different manifest
                           is refused
    chunk_000123.npz       sub-domains [123*chunk, min(124*chunk, n)): ids,
                           lb, ub [rows], and the verdicts when a property
                           is swept

Each chunk file is written to a temporary name and renamed into place, so a
process killed mid-write leaves either the whole file or none; a file that
does not read back with the expected ids and shapes counts as missing and is
bounded again.  With several ranks (one process per GPU) rank r takes the
chunks k with k % world == r; ranks share nothing but the directory.
"""
from __future__ import annotations

import json
import os
import zipfile

import numpy as np


class SweepDir:
    """The on-disk state of one sweep."""

    def __init__(self, path: str, n: int, chunk: int, rows: int, meta: dict | None = None):
        if n <= 0 or chunk <= 0 or rows <= 0:
            raise ValueError("n, chunk and rows must be positive")
        self.path, self.n, self.chunk, self.rows = path, int(n), int(chunk), int(rows)
        self.manifest = {"n": self.n, "chunk": self.chunk, "rows": self.rows, "meta": meta or {}}
        os.makedirs(path, exist_ok=True)
        mpath = os.path.join(path, "manifest.json")
        if os.path.exists(mpath):
            with open(mpath) as f:
                old = json.load(f)
            if old != json.loads(json.dumps(self.manifest)):
                raise ValueError(f"{path} holds a different sweep: {old} (this one: {self.manifest})")
        else:
            self._atomic_write(mpath, json.dumps(self.manifest, indent=1).encode())

    @property
    def n_chunks(self) -> int:
        return (self.n + self.chunk - 1) // self.chunk

    def ids(self, k: int) -> np.ndarray:
        return np.arange(k * self.chunk, min((k + 1) * self.chunk, self.n), dtype=np.int64)

    def _file(self, k: int) -> str:
        return os.path.join(self.path, f"chunk_{k:06d}.npz")

    @staticmethod
    def _atomic_write(path: str, data: bytes):
        tmp = f"{path}.tmp{os.getpid()}"
        with open(tmp, "wb") as f:
            f.write(data)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)

    def load(self, k: int):
        """(lb, ub, status or None) of chunk k, or None when it is missing or
        does not read back whole."""
        try:
            with np.load(self._file(k)) as z:
                ids, lb, ub = z["ids"], z["lb"], z["ub"]
                st = z["status"] if "status" in z else None
        except (OSError, ValueError, KeyError, EOFError, zipfile.BadZipFile):
            return None
        m = len(self.ids(k))
        if not np.array_equal(ids, self.ids(k)) or lb.shape != (m, self.rows) or ub.shape != (m, self.rows):
            return None
        if st is not None and st.shape != (m,):
            return None
        return lb, ub, st

    def done(self, k: int) -> bool:
        return self.load(k) is not None

    def pending(self, rank: int = 0, world: int = 1) -> list[int]:
        """This rank's chunks that have no valid result file yet."""
        if world <= 0 or not 0 <= rank < world:
            raise ValueError("bad rank")
        return [k for k in range(rank, self.n_chunks, world) if not self.done(k)]

    def write(self, k: int, lb, ub, status=None):
        import io
        m = len(self.ids(k))
        lb = np.ascontiguousarray(lb, np.float32).reshape(m, self.rows)
        ub = np.ascontiguousarray(ub, np.float32).reshape(m, self.rows)
        arrays = {"ids": self.ids(k), "lb": lb, "ub": ub}
        if status is not None:
            arrays["status"] = np.ascontiguousarray(status, np.int32).reshape(m)
        buf = io.BytesIO()
        np.savez(buf, **arrays)
        self._atomic_write(self._file(k), buf.getvalue())

    def collect(self):
        """(lb, ub, status) of the whole sweep, [n, rows] and [n] (status None
        unless every chunk has verdicts); raises while chunks are missing."""
        lb = np.empty((self.n, self.rows), np.float32)
        ub = np.empty((self.n, self.rows), np.float32)
        st = np.empty(self.n, np.int32)
        have_status = True
        missing = []
        for k in range(self.n_chunks):
            r = self.load(k)
            if r is None:
                missing.append(k)
                continue
            ids = self.ids(k)
            lb[ids], ub[ids] = r[0], r[1]
            if r[2] is None:
                have_status = False
            else:
                st[ids] = r[2]
        if missing:
            raise RuntimeError(f"{len(missing)} of {self.n_chunks} chunks are not done (first: {missing[0]})")
        return lb, ub, (st if have_status else None)


def run_sweep(model, split, method: int, path: str, chunk: int = 256, prop=None, rank: int = 0, world: int = 1,
              max_chunks: int | None = None, meta: dict | None = None) -> SweepDir:
    """Bound this rank's pending chunks of `split` (a workloads.SubdomainSplit)
    with `model` (engine.Model), writing each chunk's file as it completes.
    With `prop` (vnnlib.Property) every chunk goes through
    Model.compute_property (its thresholds stop verified sub-domains early and
    verdicts are stored); otherwise through Model.compute_bounds with the
    split's specification.  `max_chunks` bounds the work of this call (the
    rest stays pending for a later call).  Returns the SweepDir."""
    rows = prop.nspec if (prop is not None and prop.nspec) else (
        prop.n_out if prop is not None else split.C.shape[1])
    info = {"method": int(method), "property": prop is not None}
    info.update(meta or {})
    sd = SweepDir(path, split.count, chunk, rows, info)
    todo = sd.pending(rank, world)
    if max_chunks is not None:
        todo = todo[:max_chunks]
    for k in todo:
        ids = sd.ids(k)
        boxes = split.boxes(int(ids[0]), len(ids))
        if prop is not None:
            lb, ub, st = model.compute_property(prop, method, boxes.lower, boxes.upper)
            sd.write(k, lb, ub, st)
        else:
            lb, ub = model.compute_bounds(boxes, method)
            sd.write(k, lb, ub)
    return sd



def finish_ranks(sd: SweepDir, world: int, timeout_s: float | None = None) -> list[int]:
    """End of a multi-rank sweep (torch.distributed initialised, one process
    per rank): wait for every rank at a barrier, then return the chunks that
    are still pending over all ranks (empty when the sweep is complete).

    A rank that died before the barrier makes the wait fail on the others:
    the peer's closed connection or the group's timeout (`timeout_s`, with
    gloo's monitored barrier; otherwise the process group's own) raises.  This
    function then raises RuntimeError naming the chunks left pending, which a
    rerun of the same sweep, at any world size, bounds without redoing the
    chunks already written."""
    import datetime

    import torch.distributed as dist
    try:
        if timeout_s is not None and dist.get_backend() == "gloo":
            dist.monitored_barrier(timeout=datetime.timedelta(seconds=timeout_s))
        else:
            dist.barrier()
    except RuntimeError as e:
        missing = sd.pending(0, 1)
        raise RuntimeError(f"a rank did not reach the end of the sweep ({e}); "
                           f"{len(missing)} of {sd.n_chunks} chunks pending: rerun to resume") from e
    return sd.pending(0, 1)
