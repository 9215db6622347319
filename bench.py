"""Throughput of alpha-CROWN bounding on B200: input boxes per second.

Workload (per GPU): the MLP 784->256->256->256->256->10 with ReLU (He-normal
weights, seed 1), 512 L-inf boxes (centres U[0,1]^784, eps 0.02 clipped to
[0,1]), 9 margin rows y_t - y_j per box, alpha-CROWN with 20 Adam iterations
at lr 0.1, lower bounds optimised and upper bounds by CROWN, all as Luna's
TorchModel::compute_bounds(..., AlphaCROWN) does for each box.

A step bounds one batch of 512 boxes per GPU.  With N GPUs (torchrun) each
rank bounds its own 512 boxes (weak scaling) and the final bounds are
all-gathered over NCCL inside the step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload mlp|cnn|resnet|sweep|property]

`--impl reference` times Luna's own CPU implementation (oracle/_ref) on the
host cores for the same workload and metric.  `--workload cnn` measures the
CIFAR-shaped CNN instead (3x32x32 -> conv32 k3 -> conv64 k4s2 -> conv64 k4s2
-> 512 -> 10, He-normal weights, seed 2; 256 boxes per GPU, eps 2/255, 9
margin rows; alpha-CROWN 30 iterations at Luna's default lr 0.5).  `--workload
resnet` measures the small CIFAR ResNet (stem conv3->16 k3, residual blocks
16, 16, 32 s2 with a 1x1 projection skip, 32, BatchNorm with running mean 0,
flatten 8192 -> 100 -> Sigmoid -> 10, seed 3; 128 boxes per GPU, eps 1/255;
alpha-CROWN 50 iterations at lr 0.5).  `--workload property` bounds 512
sub-domains of one VNN-LIB robustness property on the MLP through
lb200_compute_property, with the property's thresholds stopping verified
boxes early (one GPU; see the workload's description).
"""
from __future__ import annotations

import argparse
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from luna_b200 import abi, workloads as W  # noqa: E402

METRIC = "alpha_crown_boxes_per_sec"
UNIT = "boxes/s"
L2_FLUSH_BYTES = 256 << 20

# Workloads: the MLP (the default) and the CIFAR-shaped CNN.
WORKLOADS = {
    "mlp": dict(name="mlp", gen=W.mlp_784_256x4_10, boxes=512, iters=20, lr=0.1, input_dim=784,
                desc="mlp_784_256x4_10 alpha-CROWN (20 Adam iterations, lr 0.1), {b} boxes per GPU, "
                     "eps 0.02, 9 margin specs"),
    "cnn": dict(name="cnn", gen=W.cnn_cifar, boxes=256, iters=30, lr=0.5, input_dim=3072,
                desc="cnn_cifar 3x32x32 conv32-conv64s2-conv64s2-fc512-fc10 alpha-CROWN (30 Adam "
                     "iterations, lr 0.5), {b} boxes per GPU, eps 2/255, 9 margin specs"),
    "sweep": dict(name="sweep", gen=W.convt_sweep_boxes, boxes=256, iters=50, lr=0.5, input_dim=3072,
                  desc="cnn_convt_cifar sub-domain sweep (one eps 8/255 box split into 65,536 sub-domains along "
                       "16 groups of 4 widest-gradient pixels), {b} sub-domains per GPU, alpha-CROWN (50 Adam "
                       "iterations, lr 0.5), 9 margin specs"),
    "property": dict(name="property", gen=W.mlp_property_boxes, boxes=512, iters=20, lr=0.1, input_dim=784,
                     property=True,
                     desc="VNN-LIB robustness property on mlp_784_256x4_10 (one eps 0.00317 box around a seeded "
                          "point, OR over the 9 margins of the predicted label), split into {b} sub-domains along "
                          "9 groups of 8 widest-gradient pixels; alpha-CROWN (20 Adam iterations, lr 0.1) with "
                          "the property's thresholds, so boxes stop when verified (STOP_CROWN/ALPHA_ON_VERIFIED); "
                          "bounds and verdicts through lb200_compute_property_device (e2e: "
                          "lb200_compute_property with host buffers)"),
    "resnet": dict(name="resnet", gen=W.resnet_cifar, boxes=128, iters=50, lr=0.5, input_dim=3072,
                   desc="resnet_cifar 3x32x32 stem16 + 4 residual blocks (16,16,32s2+proj,32) with BatchNorm, "
                        "fc100-Sigmoid-fc10 alpha-CROWN (50 Adam iterations, lr 0.5), {b} boxes per GPU, "
                        "eps 1/255, 9 margin specs",
                   ref_unavailable="Luna's alpha-CROWN throws on any graph with a Sigmoid node "
                                   "(AlphaCROWNAnalysis::ensureAlphaFor writes its 8 tangent slots along the "
                                   "neuron axis: shape error), so its CPU path has no alpha-CROWN result here"),
}
WL = dict(WORKLOADS["mlp"])
BOXES_PER_GPU = WL["boxes"]


def options():
    return abi.default_options(alpha_lr=WL["lr"], alpha_iterations=WL["iters"])


def config(n_gpus):
    return {"workload": WL["desc"].format(b=BOXES_PER_GPU), "boxes_per_gpu": BOXES_PER_GPU,
            "global_boxes": BOXES_PER_GPU * n_gpus, "input_dim": WL["input_dim"], "nspec": 9,
            "alpha_iterations": WL["iters"], "alpha_lr": WL["lr"],
            "parallelism": f"box-sharded x{n_gpus}", "l2": "flushed between timed steps (256 MiB write)"}


def global_boxes(n_gpus):
    """The seeded global box set of an n_gpus job."""
    return WL["gen"](BOXES_PER_GPU * n_gpus)[1]


def rank_boxes(rank, n_gpus):
    """This rank's slice of one seeded global box set (same weights on every rank)."""
    from luna_b200.shard import shard_range
    g, bx = WL["gen"](BOXES_PER_GPU * n_gpus)
    a, b = shard_range(rank, n_gpus, bx.n)
    return g, bx.slice(a, b)


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- peaks
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def traffic_per_launch(workload):
    """DRAM bytes per contraction launch of `workload` from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "contraction_traffic.json")) as f:
            return json.load(f).get(workload)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- engine arm
def run_engine(args):
    import torch
    import torch.distributed as dist

    from luna_b200.build import build
    from luna_b200.engine import Model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if rank == 0:
        build()
    if world > 1:
        dist.barrier()
    g, bx = rank_boxes(rank, world)
    model = Model(g, device=local, options=options())
    dev = torch.device("cuda", local)
    xl = torch.from_numpy(bx.lower).to(dev)
    xu = torch.from_numpy(bx.upper).to(dev)
    Cm = torch.from_numpy(bx.C).to(dev)
    B, nspec = bx.n, bx.C.shape[1]
    lb = torch.empty((B, nspec), device=dev)
    ub = torch.empty((B, nspec), device=dev)
    from luna_b200.shard import gather_bounds
    counts = [BOXES_PER_GPU] * world
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        model.compute_bounds_ptr(abi.METHOD_ALPHA_CROWN, xl.data_ptr(), xu.data_ptr(), B, Cm.data_ptr(),
                                 Cm.shape[0], nspec, lb.data_ptr(), ub.data_ptr(), stream.cuda_stream)
        if world > 1:
            gather_bounds(lb, ub, counts)  # NCCL all-gather of the final bounds
        return model.last_stats

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timing: per-step CUDA events, L2 flushed between steps
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    total_ms, launches, flops = 0.0, 0, 0.0
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        st = step()
        e1.record(stream)
        e1.synchronize()
        total_ms += e0.elapsed_time(e1)
        launches += st.kernel_launches
        flops += st.algorithmic_flops
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t = torch.tensor([total_ms], device=dev)
    rank_ms = [total_ms / args.steps]
    if world > 1:
        parts = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        rank_ms = [float(x.item()) / args.steps for x in parts]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps

    # ---- contraction kernels: CUDA events around every contraction launch,
    # on the engine's stream, in a separate pass of the same step (events
    # recorded inside the timed steps above would slow them)
    model.set_profiling(True)
    contr_ms, contr_flops, contr_launches, prof_ms = 0.0, 0.0, 0, 0.0
    for _ in range(max(1, min(args.steps, 2))):
        flush.zero_()
        st = step()
        contr_ms += st.ms_contractions
        contr_flops += st.contraction_flops
        contr_launches += st.contraction_launches
        prof_ms += st.ms_device
    model.set_profiling(False)

    # ---- end to end through the public C ABI with host buffers (pinned):
    # one GPU: lb200_compute_bounds; N GPUs: lb200_shard_run over the
    # library's own NCCL communicator (each rank copies its share in, bounds
    # it, all-gathers every rank's bounds and copies them all out).
    e2e_steps = max(1, args.steps)
    if world == 1:
        hxl = torch.from_numpy(bx.lower).pin_memory()
        hxu = torch.from_numpy(bx.upper).pin_memory()
        hC = torch.from_numpy(bx.C).pin_memory()
        hlb = torch.empty((B, nspec)).pin_memory()
        hub = torch.empty((B, nspec)).pin_memory()
        model.compute_bounds_host_ptr(abi.METHOD_ALPHA_CROWN, hxl.data_ptr(), hxu.data_ptr(), B, hC.data_ptr(),
                                      hC.shape[0], nspec, hlb.data_ptr(), hub.data_ptr())
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            model.compute_bounds_host_ptr(abi.METHOD_ALPHA_CROWN, hxl.data_ptr(), hxu.data_ptr(), B,
                                          hC.data_ptr(), hC.shape[0], nspec, hlb.data_ptr(), hub.data_ptr())
        e2e_s = (time.perf_counter() - t0) / e2e_steps
        h2d = int(hxl.numel() * 4 + hxu.numel() * 4 + hC.numel() * 4)
        d2h = int(hlb.numel() * 4 + hub.numel() * 4)
    else:
        from luna_b200.engine import NcclComm, nccl_unique_id
        uid = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = NcclComm(bytes(uid.cpu().numpy().tobytes()), rank, world, local)
        gbx = global_boxes(world)
        pinned = [torch.from_numpy(a).pin_memory() for a in (gbx.lower, gbx.upper, gbx.C)]
        hbx = W.Boxes(*(p.numpy() for p in pinned))
        model.shard_run(comm, hbx, abi.METHOD_ALPHA_CROWN, timeout_ms=120000)
        dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            model.shard_run(comm, hbx, abi.METHOD_ALPHA_CROWN, timeout_ms=120000)
        e2e_s = (time.perf_counter() - t0) / e2e_steps
        comm.close()
        h2d = int((bx.lower.size + bx.upper.size + bx.C.size) * 4)  # this rank's share
        d2h = int(2 * gbx.n * nspec * 4)  # every rank's bounds
    te = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())

    if rank == 0:
        pk, pk_src = peaks()
        # 3xTF32 split fp32 contractions: TF32 dense is half the bf16 rate and
        # the split issues three MMAs per product.
        peak = pk["bf16_tflops_sustained"] / 2.0 / 3.0
        achieved = (contr_flops / contr_launches) / (contr_ms / contr_launches) / 1e9 if contr_launches else 0.0
        tr = traffic_per_launch(WL["name"])
        line = {
            "metric": METRIC, "value": world * B / (ms_per_step / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded He-normal weights, uniform box centres)",
            "config": config(world),
            "e2e": {"value": world * B / e2e_s, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": "lb200_compute_bounds" if world == 1 else "lb200_shard_run (NCCL all-gather inside)"},
            "rank_ms_per_step": rank_ms,
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak if peak else None,
                         "traffic": tr.get("bytes_per_launch") if tr else None,
                         "kernel": "A.W contraction (GEMM + fused relaxation / concretisation / adjoint epilogue)",
                         "peak_source": f"{pk_src}: bf16_tflops_sustained / 2 (TF32) / 3 (3-pass split)",
                         "timing": "CUDA events around each contraction launch on the engine's stream, "
                                   "in a separate pass of the same step after the timed steps",
                         "contraction_share_of_step": contr_ms / prof_ms if prof_ms else None,
                         "algorithmic_tflops_step": flops / (total_ms / 1e3) / 1e12 if total_ms else None},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            if WL.get("ref_unavailable"):
                line["cpu_baseline"] = {"unavailable": WL["ref_unavailable"]}
            else:
                line["cpu_baseline"] = cpu_baseline(args.cpu_boxes)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_property(args):
    """The property workload on one GPU: `value` times
    lb200_compute_property_device on device-resident sub-domains with CUDA
    events (L2 flushed between steps); `e2e` times lb200_compute_property
    with host buffers in and out."""
    import torch

    from luna_b200.build import build
    from luna_b200.engine import Model
    from luna_b200.vnnlib import Property

    if int(os.environ.get("WORLD_SIZE", "1")) != 1 or args.gpus != 1:
        raise SystemExit("--workload property runs on one GPU")
    torch.cuda.set_device(0)
    build()
    g, bx = WL["gen"](BOXES_PER_GPU)
    _, _, text = W.mlp_property_split()
    prop = Property(text, WL["input_dim"], 10)
    model = Model(g, device=0, options=options())
    dev = torch.device("cuda", 0)
    B, rows = bx.n, prop.nspec
    xl = torch.from_numpy(bx.lower).to(dev)
    xu = torch.from_numpy(bx.upper).to(dev)
    lb = torch.empty((B, rows), device=dev)
    ub = torch.empty((B, rows), device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return model.compute_property_ptr(prop, abi.METHOD_ALPHA_CROWN, xl.data_ptr(), xu.data_ptr(), B,
                                          lb.data_ptr(), ub.data_ptr(), status.data_ptr(), stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    total_ms, launches, iters = 0.0, 0, 0
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        st = step()
        e1.record(stream)
        e1.synchronize()
        total_ms += e0.elapsed_time(e1)
        launches += st.kernel_launches
        iters = max(iters, st.alpha_iterations_run)
    clocks = sampler.stop()
    # Contraction timing in a separate pass (see run_engine).
    model.set_profiling(True)
    contr_ms, contr_flops, contr_launches, prof_ms = 0.0, 0.0, 0, 0.0
    for _ in range(max(1, min(args.steps, 2))):
        flush.zero_()
        st = step()
        contr_ms += st.ms_contractions
        contr_flops += st.contraction_flops
        contr_launches += st.contraction_launches
        prof_ms += st.ms_device
    model.set_profiling(False)
    ms_per_step = total_ms / args.steps
    st_host = status.cpu().numpy()

    # End to end: host buffers in and out (lb200_compute_property).
    hxl, hxu = np.ascontiguousarray(bx.lower), np.ascontiguousarray(bx.upper)
    hlb, hub, hst = model.compute_property(prop, abi.METHOD_ALPHA_CROWN, hxl, hxu)
    e2e_steps = max(1, min(args.steps, 3))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        hlb, hub, hst = model.compute_property(prop, abi.METHOD_ALPHA_CROWN, hxl, hxu)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    assert (hst == st_host).all()

    pk, pk_src = peaks()
    peak = pk["bf16_tflops_sustained"] / 2.0 / 3.0
    achieved = (contr_flops / contr_launches) / (contr_ms / contr_launches) / 1e9 if contr_launches else 0.0
    counts = {abi.STATUS_NAMES[k]: int((st_host == k).sum()) for k in abi.STATUS_NAMES}
    cfg = config(1)
    cfg.update(nspec=rows, or_branches=prop.n_branches, verdicts=counts, alpha_iterations_run=iters)
    line = {
        "metric": METRIC, "value": B / (ms_per_step / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded He-normal weights, seeded box centre)",
        "config": cfg,
        "e2e": {"value": B / e2e_s, "unit": UNIT, "h2d_bytes_per_step": int(hxl.nbytes + hxu.nbytes),
                "d2h_bytes_per_step": int(hlb.nbytes + hub.nbytes + hst.nbytes)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if peak else None, "traffic": None,
                     "kernel": "A.W contraction (GEMM + fused relaxation / concretisation / adjoint epilogue)",
                     "peak_source": f"{pk_src}: bf16_tflops_sustained / 2 (TF32) / 3 (3-pass split)",
                     "contraction_share_of_step": contr_ms / prof_ms if prof_ms else None},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_boxes)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- reference arm
_REF = {}


def _ref_worker(task):
    """One host process: bound boxes [a, b) of workload `name` with Luna's CPU
    path on one thread.  The reference library and the workload are loaded
    once per process."""
    name, n_boxes, a, b = task
    if _REF.get("key") != (name, n_boxes):
        os.environ["CUDA_VISIBLE_DEVICES"] = ""
        for var in ("OMP_NUM_THREADS", "MKL_NUM_THREADS", "OPENBLAS_NUM_THREADS"):
            os.environ[var] = "1"
        from oracle import luna_ref
        WL.clear()
        WL.update(WORKLOADS[name])
        _REF["lib"] = luna_ref
        _REF["work"] = WL["gen"](n_boxes)
        _REF["key"] = (name, n_boxes)
    if b <= a:
        return 0.0
    g, bx = _REF["work"]
    if WL.get("property"):
        # Luna's CLI flow: the property's constraints set on the model, so
        # its thresholds stop verified boxes early.
        if "spec" not in _REF:
            _, _, text = W.mlp_property_split()
            _REF["spec"] = _REF["lib"].vnnlib_parse(text, WL["input_dim"], 10)
        sub = bx.slice(a, b)
        t0 = time.perf_counter()
        _REF["lib"].compute_property(g, _REF["spec"], sub.lower, sub.upper, abi.METHOD_ALPHA_CROWN, options(),
                                     num_threads=1)
        return time.perf_counter() - t0
    t0 = time.perf_counter()
    _REF["lib"].compute_bounds(g, bx.slice(a, b), abi.METHOD_ALPHA_CROWN, options(), num_threads=1)
    return time.perf_counter() - t0


class CpuBaseline:
    """Luna's CPU implementation (oracle/_ref) on the host cores: one process
    per core, one thread each; a sample bounds `boxes_per_proc` boxes per
    process."""

    def __init__(self, procs=None):
        self.procs = procs or min(os.cpu_count() or 1, BOXES_PER_GPU)
        self.pool = mp.get_context("spawn").Pool(self.procs)
        self.name = WL["name"]
        # Load the library and the workload in every worker.
        self.pool.map(_ref_worker, [(self.name, BOXES_PER_GPU, 0, 0)] * self.procs)

    def sample(self, boxes_per_proc=1):
        work = [(self.name, BOXES_PER_GPU, (i * boxes_per_proc) % BOXES_PER_GPU,
                 (i * boxes_per_proc) % BOXES_PER_GPU + boxes_per_proc) for i in range(self.procs)]
        t0 = time.perf_counter()
        self.pool.map(_ref_worker, work, chunksize=1)
        wall = time.perf_counter() - t0
        n = self.procs * boxes_per_proc
        return {"value": n / wall, "unit": UNIT, "cores": self.procs, "kind": "reference",
                "sample": f"{n} of the {BOXES_PER_GPU} boxes ({boxes_per_proc} per process, {self.procs} processes x 1 "
                          f"thread), wall {wall:.2f} s", "wall_s": wall, "boxes": n}

    def close(self):
        self.pool.close()
        self.pool.join()


def cpu_baseline(boxes_per_proc=1):
    """One warm-up sample (first boxes pay Luna's one-time set-up in every
    process), then the measured sample: the same sampler as the reference arm."""
    cb = CpuBaseline()
    try:
        cb.sample(1)
        return cb.sample(boxes_per_proc)
    finally:
        cb.close()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import luna_ref
    if not luna_ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libluna_ref.so not built"}))
        return
    if WL.get("ref_unavailable"):
        print(json.dumps({"impl": "reference", "unavailable": WL["ref_unavailable"]}))
        return
    cb = CpuBaseline()
    try:
        for _ in range(args.warmup):
            cb.sample(1)
        vals = [cb.sample(args.cpu_boxes) for _ in range(args.steps)]
    finally:
        cb.close()
    boxes = sum(x["boxes"] for x in vals)
    wall = sum(x["wall_s"] for x in vals)
    v = boxes / wall
    base = dict(vals[0])
    base["value"] = v
    base["sample"] = f"{args.steps} samples of {vals[0]['boxes']} boxes ({args.cpu_boxes} per process, " \
                     f"{cb.procs} processes x 1 thread)"
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * wall / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded He-normal weights, uniform box centres)", "config": config(args.gpus),
            "impl": "reference", "cpu_baseline": base,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--cpu-boxes", type=int, default=1, help="boxes per host process in the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--boxes", type=int, default=0,
                    help="boxes per GPU (default: the workload's; smaller cases are for profiling only)")
    ap.add_argument("--workload", default="mlp", choices=sorted(WORKLOADS))
    args = ap.parse_args()
    WL.clear()
    WL.update(WORKLOADS[args.workload])
    globals()["BOXES_PER_GPU"] = args.boxes if args.boxes else WL["boxes"]
    if args.impl == "reference":
        run_reference(args)
    elif WL.get("property"):
        run_property(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
