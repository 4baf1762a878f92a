#!/usr/bin/env python
"""Benchmark of the cufk reconstruction hot path on B200: fwd+bwd atoms/s (B=4096, N=768, fp32).

One step = the block forward plus the block backward over this rank's chains of config 1
(B = 4096 chains per rank by default, N = 768 atoms, float32).  Prints ONE JSON line on rank 0.

* ``value``: atoms of all ranks / (max over ranks of the device time per step).  Inputs are
  resident in HBM.  Each step replays a CUDA graph holding the two kernel launches for one of
  several input sets; the sets rotate so that the data of a step was last touched several steps
  earlier (total footprint > 3x the 126 MB L2), i.e. every step reads its inputs from HBM.
* ``roofline``: algorithmic bytes per launch (forward 24 B/atom, backward 36 B/atom in fp32, from
  the minimum reads and writes) / the average launch duration of that kernel, timed with CUDA
  events in a second region of single-kernel graphs; ``peak`` from MEASURED_PEAKS.json.
* ``e2e``: the same metric through the public API (``cufk_b200.reconstruct`` + autograd) with
  pinned host buffers: every step copies its inputs host->device and its outputs device->host.
* ``cpu_baseline``: the float64 torch restatement (oracle/nerf64.py) on the host cores, on a
  bounded sample of the same workload (rank 0, single-GPU runs only).
* ``--impl reference``: the reference arm.  The reference's path exists only as CUDA kernels, so
  the CPU implementation timed is the float64 restatement of its algorithm on all host cores.

Multi-GPU: ``python -m torch.distributed.run --nproc-per-node N bench.py --gpus N``.  Chains are
independent, so there is no collective on the hot path.  ``--scaling strong`` (the default, config
1's own split) divides the fixed B = 4096 over the ranks (2048 / 1024 / 512 chains per GPU at
2 / 4 / 8); the line also carries the weak figure (every rank a full B = 4096 of its own chains)
under ``weak``.  ``--scaling weak`` makes weak the headline instead.  An NCCL all-gather of xyz is
timed separately and reported under ``allgather``.

Timing: every timed region is repeated (``--repeats``, default 5) and the median is reported, with
the spread beside it; ``unflushed`` is the same step replayed on one resident input set.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "fwd+bwd atoms/s (B=4096,N=768 fp32)"
GLOBAL_BATCH = 4096
POINTS = 768
L2_BYTES = 126 * 1024 * 1024
# chains longer than this take the one-slot-per-step kernels for float64 and for every backward
VEC_MAX_POINTS_LONG = 1024
HBM_FALLBACK_GBS = 6650.0


# The other configurations of the path (one JSON line each, not the headline): kind, chains,
# points, dtype, anchors.
WORKLOADS = {
    "cfg2-f32": ("block", 2048, 2051, torch.float32, True),
    "cfg2-f64": ("block", 2048, 2051, torch.float64, True),
    "cfg3-f32": ("torsion", 16384, 768, torch.float32, False),
    "cfg3-bf16": ("torsion", 16384, 768, torch.bfloat16, False),
    "cfg4-f16": ("block", 8192, 1026, torch.float16, False),
    "cfg4-bf16": ("block", 8192, 1026, torch.bfloat16, False),
    # the fused consumer (reconstruct_mse) on the config-1 shape, beside the unfused sequence
    "mse-cfg1": ("mse", 4096, 768, torch.float32, False),
}
BACKBONE_LENGTHS = (0.14685231, 0.15365194, 0.13405086)
BACKBONE_ANGLES = (1.9676635, 2.062335, 2.164016)


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH, help="chains per rank (weak) or in total (strong)")
    ap.add_argument(
        "--scaling",
        choices=["weak", "strong"],
        default="strong",
        help="strong (config 1's split): the batch is split over the ranks; weak: every rank runs the whole batch on its own chains",
    )
    ap.add_argument("--repeats", type=int, default=5, help="timed regions per figure (median reported)")
    ap.add_argument("--per-graph", type=int, default=10, help="steps captured per CUDA graph (consecutive input sets)")
    ap.add_argument("--no-ref-kernels", action="store_true", help="skip timing the reference's own kernels (oracle/_ref)")
    ap.add_argument("--points", type=int, default=POINTS)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument(
        "--workload",
        choices=["cfg1", *WORKLOADS],
        default="cfg1",
        help="cfg1 (default) is the headline line; the others time the remaining configurations of the path",
    )
    return ap.parse_args(argv)


# ------------------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------------------
class Dist:
    def __init__(self, gpus: int, device_needed: bool = True):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus and self.world > 1:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.pg = None
        self.device = torch.device("cuda") if device_needed else torch.device("cpu")
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            if device_needed:
                torch.cuda.set_device(self.local_rank)
            dist.init_process_group(
                "nccl" if device_needed else "gloo",
                timeout=datetime.timedelta(seconds=120),
                device_id=torch.device("cuda", self.local_rank) if device_needed else None,
            )
            self.pg = dist
        elif device_needed:
            torch.cuda.set_device(0)

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def gather(self, values: list[float]) -> list[list[float]]:
        """Every rank's `values` (same length on all ranks), indexed by rank."""
        if self.pg is None:
            return [list(values)]
        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        out = torch.empty(self.world * len(values), dtype=torch.float64, device=self.device)
        self.pg.all_gather_into_tensor(out, t)
        return out.view(self.world, len(values)).tolist()

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def make_inputs(batch: int, points: int, seed: int = 0) -> dict:
    """Seeded synthetic config-1 inputs (float64 on the CPU, cast to float32).

    lengths cycle the backbone bond lengths (0.14685231, 0.15365194, 0.13405086) nm + N(0, 0.002);
    angles cycle (1.9676635, 2.062335, 2.164016) rad + N(0, 0.03); dihedrals ~ U(-pi, pi);
    grad_out ~ N(0, 1).  No public dataset exists for this path; these are the benchmark inputs.
    """
    g = torch.Generator().manual_seed(seed)
    f64 = torch.float64
    i1 = torch.arange(points - 1)
    i2 = torch.arange(points - 2)
    L = torch.tensor((0.14685231, 0.15365194, 0.13405086), dtype=f64)[i1 % 3] + 0.002 * torch.randn(batch, points - 1, generator=g, dtype=f64)
    A = torch.tensor((1.9676635, 2.062335, 2.164016), dtype=f64)[i2 % 3] + 0.03 * torch.randn(batch, points - 2, generator=g, dtype=f64)
    D = (torch.rand(batch, points - 3, generator=g, dtype=f64) * 2.0 - 1.0) * math.pi
    G = torch.randn(batch, points, 3, generator=g, dtype=f64)
    return {"lengths": L.float(), "angles": A.float(), "dihedrals": D.float(), "grad": G.float()}


def shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous chain range [lo, hi) of this rank (chains are independent: no exchange)."""
    per, extra = divmod(batch, world)
    lo = rank * per + min(rank, extra)
    return lo, lo + per + (1 if rank < extra else 0)


def rank_inputs(make, batch: int, scaling: str, world: int, rank: int) -> tuple[dict, int]:
    """This rank's inputs and the job's total chain count.  Weak scaling: a whole `batch` of the
    rank's own chains (generated from seed = rank).  Strong: the rank's slice of one `batch`
    generated from seed 0 (identically on every rank).  `make(batch, seed)` builds the inputs."""
    if scaling == "weak" or world == 1:
        return make(batch, rank), batch * world
    lo, hi = shard(batch, world, rank)
    host = make(batch, 0)
    return {k: (v[lo:hi].contiguous() if v.dim() > 1 else v) for k, v in host.items()}, batch


# ------------------------------------------------------------------------------------------------
# clocks: NVML sampling during the timed region (read-only queries)
# ------------------------------------------------------------------------------------------------
REASON_BITS = {
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
    0x2: "applications_clocks_setting",
    0x10: "sync_boost",
}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self.handle = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
        except Exception as exc:  # noqa: BLE001 - clocks are reported as unavailable
            self.error = repr(exc)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self.handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "error", "nvml unavailable")}
        names = sorted(name for bit, name in REASON_BITS.items() if self.reasons & bit)
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": names,
            "samples": len(self.samples),
        }


# ------------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------------
def bytes_per_atom(points: int, elem: int = 4) -> tuple[float, float]:
    """Algorithmic bytes per chain / N: forward reads 3N-6, writes 3N; backward reads 3N-6 + 3N,
    writes 3N-6 elements."""
    fwd = (6 * points - 6) * elem / points
    bwd = (9 * points - 12) * elem / points
    return fwd, bwd


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        if data.get("hbm_gbs"):
            return float(data["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


def profiled_traffic_per_atom(kernel: str):
    """DRAM bytes per atom of one launch from the committed ncu summary (profiles/traffic.json)."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    data = json.loads(path.read_text())
    entry = data.get(kernel)
    return None if entry is None else float(entry["dram_bytes_per_atom"])


def time_graphs(graphs, steps: int, warmup: int, dist: Dist, stream, repeats: int = 1) -> list[float]:
    """Replays graphs[k % len] for `warmup` then, `repeats` times, `steps` iterations bracketed by
    a barrier and a device synchronisation; returns the max-over-ranks ms of each repeat."""
    for k in range(warmup):
        graphs[k % len(graphs)].replay()
    out = []
    for _ in range(max(1, repeats)):
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for k in range(steps):
            graphs[k % len(graphs)].replay()
        end.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        out.append(dist.max(start.elapsed_time(end)))
    return out


def spread(ms_per_step: list[float]) -> dict:
    """Median, min and max of per-step times (ms) over the repeats."""
    return {
        "median_ms": statistics.median(ms_per_step),
        "min_ms": min(ms_per_step),
        "max_ms": max(ms_per_step),
        "repeats": len(ms_per_step),
    }


class StepGraphs:
    """Device-resident input sets of one rank and CUDA graphs of `per_graph` consecutive steps (each
    step the forward then the backward that reads the forward's xyz, the kernels autograd runs), and
    of each kernel alone.  A graph's steps take consecutive input sets, which rotate (total footprint
    > 3x the 126 MB L2) so that every step reads from HBM.  Several steps per graph keep the
    per-replay launch gap of the device (several microseconds) out of the per-step time."""

    def __init__(self, C, host: dict, n: int, dev, stream, per_graph: int = 1):
        b_local = host["lengths"].shape[0]
        self.b_local = b_local
        self.per_graph = max(1, per_graph)
        self.set_bytes = 4 * b_local * ((n - 1) + (n - 2) + (n - 3) + 3 * n) * 2  # inputs + outputs of a step
        self.n_sets = max(2, min(64, math.ceil(3 * L2_BYTES / max(self.set_bytes, 1))))
        self.sets = []
        for i in range(self.n_sets):
            # each set a distinct copy (perturbed dihedrals) so no two sets alias
            d = {k: v.to(dev) for k, v in host.items()}
            d["dihedrals"] = d["dihedrals"] + 1e-3 * i
            self.sets.append(d)
        torch.cuda.synchronize()

        def fwd(d):
            return C.block_forward(d["lengths"], d["angles"], d["dihedrals"], None, None, None)

        def bwd(d, xyz):
            C.block_backward_from_xyz(d["lengths"], d["angles"], d["dihedrals"], None, None, None, xyz, d["grad"])

        def capture(body):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                body()
            return g

        self.step, self.fwd, self.bwd = [], [], []
        with torch.cuda.stream(stream):
            for d in self.sets:  # eager warm-up of both kernels (first-call attribute setup happens here)
                d["xyz"] = fwd(d)
                bwd(d, d["xyz"])
            stream.synchronize()
            for i in range(self.n_sets):
                group = [self.sets[(i + r) % self.n_sets] for r in range(self.per_graph)]
                self.step.append(capture(lambda group=group: [bwd(d, fwd(d)) for d in group]))
                self.fwd.append(capture(lambda group=group: [fwd(d) for d in group]))
                self.bwd.append(capture(lambda group=group: [bwd(d, d["xyz"]) for d in group]))
            # the unflushed figure: every step of the graph on the first set (its data may stay in L2)
            first = self.sets[0]
            self.unflushed = [capture(lambda: [bwd(first, fwd(first)) for _ in range(self.per_graph)])]
        torch.cuda.synchronize()

    def time(self, graphs, steps: int, warmup: int, dist: "Dist", stream, repeats: int) -> list[float]:
        """ms per step of each repeat (max over ranks), `steps` steps per repeat."""
        replays = max(1, steps // self.per_graph)
        return [t / (replays * self.per_graph) for t in time_graphs(graphs, replays, max(1, warmup // self.per_graph), dist, stream, repeats)]


def run_ours(args, dist: Dist) -> dict | None:
    sys.path.insert(0, str(ROOT))
    import cufk_b200 as cufk
    from cufk_b200 import _native

    C = _native._C
    dev = torch.device("cuda", torch.cuda.current_device())
    n = args.points
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    # synthetic config-1 inputs of this rank: the headline split, and (several ranks) the other one
    host, global_batch = rank_inputs(lambda b, seed: make_inputs(b, n, seed=seed), args.batch, args.scaling, dist.world, dist.rank)
    per_graph = max(1, min(args.per_graph, args.steps))
    sg = StepGraphs(C, host, n, dev, stream, per_graph)
    b_local = sg.b_local

    sampler = ClockSampler(dev.index)
    with torch.cuda.stream(stream):
        with sampler:
            step_ms = sg.time(sg.step, args.steps, args.warmup, dist, stream, args.repeats)
        fwd_ms = sg.time(sg.fwd, args.steps, args.warmup, dist, stream, args.repeats)
        bwd_ms = sg.time(sg.bwd, args.steps, args.warmup, dist, stream, args.repeats)
        unflushed_ms = sg.time(sg.unflushed, args.steps, args.warmup, dist, stream, args.repeats)
    ms_step = statistics.median(step_ms)
    ms_fwd, ms_bwd = statistics.median(fwd_ms), statistics.median(bwd_ms)
    atoms_total = global_batch * n
    value = atoms_total / (ms_step * 1e-3)

    # the other scaling mode on several ranks (weak beside a strong headline, or strong beside weak)
    other = None
    if dist.world > 1:
        other_mode = "weak" if args.scaling == "strong" else "strong"
        host_o, global_o = rank_inputs(lambda b, seed: make_inputs(b, n, seed=seed), args.batch, other_mode, dist.world, dist.rank)
        sg_o = StepGraphs(C, host_o, n, dev, stream, per_graph)
        with torch.cuda.stream(stream):
            o_ms = sg_o.time(sg_o.step, args.steps, args.warmup, dist, stream, args.repeats)
        other = {
            "scaling": other_mode,
            "value": global_o * n / (statistics.median(o_ms) * 1e-3),
            "ms_per_step": statistics.median(o_ms),
            "global_batch": global_o,
            "per_gpu_batch": sg_o.b_local,
            "spread": spread(o_ms),
        }
        del sg_o
        torch.cuda.synchronize()

    # roofline of the dominant kernel
    peak, peak_kind = measured_peak()
    fwd_bpa, bwd_bpa = bytes_per_atom(n)
    atoms_local = b_local * n
    per_kernel = {
        "block_forward_vec_kernel": (ms_fwd, fwd_bpa),
        "block_backward_xyz_vec_kernel": (ms_bwd, bwd_bpa),
    }
    # bytes the kernels move: the backward reads the forward's xyz (3N) in place of the three input
    # rows (3N - 6) and only three scalars of the inputs
    moved_bpa = {"block_forward_vec_kernel": fwd_bpa, "block_backward_xyz_vec_kernel": (9 * n - 6) * 4 / n}
    dom = max(per_kernel, key=lambda k: per_kernel[k][0])
    ms_dom, bpa_dom = per_kernel[dom]
    achieved = bpa_dom * atoms_local / (ms_dom * 1e-3) / 1e9
    traffic_pa = profiled_traffic_per_atom(dom)
    roofline = {
        "kernel": dom,
        "bound": "hbm",
        "achieved": round(achieved, 1),
        "peak": peak,
        "unit": "GB/s",
        "frac": round(achieved / peak, 4),
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
        "traffic": None if traffic_pa is None else round(traffic_pa * atoms_local),
        "algorithmic_bytes": round(bpa_dom * atoms_local),
        "launch_ms": round(ms_dom, 5),
        "per_kernel": {
            k: {
                "launch_ms": round(t, 5),
                "bytes_per_atom": round(b, 3),
                "achieved_gbs": round(b * atoms_local / (t * 1e-3) / 1e9, 1),
                "frac": round(b * atoms_local / (t * 1e-3) / 1e9 / peak, 4),
                "moved_bytes_per_atom": round(moved_bpa[k], 3),
                "moved_gbs": round(moved_bpa[k] * atoms_local / (t * 1e-3) / 1e9, 1),
                "spread": spread(ms),
            }
            for (k, (t, b)), ms in zip(per_kernel.items(), (fwd_ms, bwd_ms))
        },
        "step_frac": round((fwd_bpa + bwd_bpa) * atoms_local / (ms_step * 1e-3) / 1e9 / peak, 4),
    }

    # optional NCCL all-gather of xyz (not part of the step), timed separately
    allgather = None
    if dist.world > 1:
        xyz = torch.empty(b_local, n, 3, device=dev)
        full = torch.empty(b_local * dist.world, n, 3, device=dev)
        for _ in range(3):
            dist.pg.all_gather_into_tensor(full, xyz)
        torch.cuda.synchronize()
        dist.barrier()
        reps = 20
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(reps):
            dist.pg.all_gather_into_tensor(full, xyz)
        s1.record()
        torch.cuda.synchronize()
        ms_ag = dist.max(s0.elapsed_time(s1) / reps)
        nbytes = full.numel() * 4
        allgather = {
            "ms": round(ms_ag, 4),
            "bytes": nbytes,
            "bus_gbs": round(nbytes * (dist.world - 1) / dist.world / (ms_ag * 1e-3) / 1e9, 1),
        }

    # the reference's own kernels on the same box (single-GPU runs only)
    ref_kernels = None
    if dist.world == 1 and not args.no_ref_kernels:
        ref_kernels = time_reference_kernels(cufk, sg, n, stream, args)

    # end to end through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(cufk, host, dev, args, dist, global_batch)

    workload = {
        "strong": "config 1: block reconstruct forward+backward, B=4096 chains split over the GPUs, N=768 atoms, fp32",
        "weak": "config 1: block reconstruct forward+backward, B=4096 chains per GPU, N=768 atoms, fp32",
    }[args.scaling if dist.world > 1 else "strong"]
    result = {
        "metric": METRIC,
        "value": value,
        "unit": "atoms/s",
        "n_gpus": dist.world,
        "steps": (args.steps // per_graph) * per_graph,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": args.scaling if dist.world > 1 else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded backbone internal coordinates, oracle/nerf64.make_inputs)",
        "config": {
            "workload": workload,
            "global_batch": global_batch,
            "points": n,
            "per_gpu_batch": b_local,
            "parallelism": f"chains independent, {'each rank its own B' if args.scaling == 'weak' and dist.world > 1 else 'one B split'} x{dist.world}; no collective on the hot path",
            "l2": f"{sg.n_sets} rotating input/output sets, {sg.n_sets * sg.set_bytes / 2**20:.0f} MiB > L2 (126 MB); unflushed: every step on one set",
            "timing": f"CUDA graphs of {per_graph} steps each (fwd+bwd launches per step, consecutive input sets), CUDA events, max over ranks, median of {args.repeats} repeats of {(args.steps // per_graph) * per_graph} steps",
        },
        "spread": spread(step_ms),
        "unflushed": {"ms_per_step": statistics.median(unflushed_ms), "value": atoms_total / (statistics.median(unflushed_ms) * 1e-3), "spread": spread(unflushed_ms)},
        "roofline": roofline,
        "e2e": e2e,
        "gpu_launches": 2 * (args.steps // per_graph) * per_graph,
        "kernels": "block_forward_vec_kernel + block_backward_xyz_vec_kernel per step",
        "clocks": sampler.summary(),
    }
    if other is not None:
        result[other["scaling"]] = other
    if allgather is not None:
        result["allgather"] = allgather
    if ref_kernels is not None:
        result["ref_kernels"] = ref_kernels
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(n)
    return result


def time_reference_kernels(cufk, sg: "StepGraphs", n: int, stream, args) -> dict:
    """The reference's own block kernels (its block.cu compiled from source into oracle/_ref by
    oracle/build_ref.py) against cufk_b200 on the same rotating input sets, both through their
    autograd path, eagerly (a forward, then backward of the step's grad): a measurement leg, like
    cpu_baseline; the timed step above never touches oracle/."""
    try:
        from oracle import ref_kernels
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"oracle.ref_kernels: {exc}"}
    if not ref_kernels.available("block"):
        return {"unavailable": "oracle/_ref/block/cufk_ref_block.so not built"}
    dev = sg.sets[0]["lengths"].device
    anchors = {
        "p0": torch.zeros(3, device=dev),
        "first_direction": torch.tensor([1.0, 0.0, 0.0], device=dev),
        "initial_normal": torch.tensor([0.0, 0.0, 1.0], device=dev),
    }

    def step(fn, d):
        L, A, D = (d[k].detach().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
        xyz = fn(L, A, D, **anchors)
        xyz.backward(d["grad"])

    out = {}
    reps = min(args.steps, 200)
    with torch.cuda.stream(stream):
        for name, fn in (("reference", ref_kernels.ref_reconstruct), ("cufk_b200", cufk.reconstruct)):
            for k in range(5):
                step(fn, sg.sets[k % len(sg.sets)])
            times = []
            for _ in range(max(1, args.repeats)):
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for k in range(reps):
                    step(fn, sg.sets[k % len(sg.sets)])
                e1.record(stream)
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) / reps)
            out[name] = {"ms_per_step": statistics.median(times), "spread": spread(times)}
    ref_ms, our_ms = out["reference"]["ms_per_step"], out["cufk_b200"]["ms_per_step"]
    return {
        "reference_ms_per_step": ref_ms,
        "cufk_b200_ms_per_step": our_ms,
        "speedup": ref_ms / our_ms,
        "reference_value": sg.b_local * n / (ref_ms * 1e-3),
        "mode": "both through autograd, eager (forward + backward of a fixed grad per step), explicit default anchors, the same rotating input sets",
        "detail": out,
        "kernels": "reference: block_forward_kernel / block_backward_kernel of its block.cu built for sm_100a (oracle/_ref)",
    }


def gpu_local_cpus(device_index: int) -> set[int]:
    """The host CPUs NVML reports as local to the GPU (its NUMA node), within this process's allowed
    set; empty when NVML cannot say.  A read-only query."""
    try:
        import pynvml

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, max(1, (os.cpu_count() or 64) // 64 + 1))
    except Exception:  # noqa: BLE001 - no affinity information: leave the process as it is
        return set()
    cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1}
    return cpus & os.sched_getaffinity(0)


def numa_node_of(cpus: set[int]) -> int:
    """NUMA node of the first of `cpus` (from sysfs), -1 when unknown."""
    for cpu in sorted(cpus)[:1]:
        for entry in Path(f"/sys/devices/system/cpu/cpu{cpu}").glob("node*"):
            try:
                return int(entry.name[4:])
            except ValueError:
                pass
    return -1


def run_e2e(cufk, host, dev, args, dist: Dist, global_batch: int) -> dict:
    """Runs `_run_e2e` with the calling thread on the GPU's own NUMA node: the pinned host buffers
    are allocated (first touched) there, so the copies do not cross the socket interconnect.  The
    thread's CPU set is restored afterwards."""
    before = os.sched_getaffinity(0)
    local = gpu_local_cpus(dev.index)
    if local:
        os.sched_setaffinity(0, local)
    try:
        out = _run_e2e(cufk, host, dev, args, dist, global_batch)
    finally:
        os.sched_setaffinity(0, before)
    out["host_cpus"] = f"{len(local)} GPU-local cores (NVML affinity)" if local else "unchanged (no NVML affinity)"
    node = numa_node_of(local if local else before)
    ranks = dist.gather([node, out.pop("_h2d_gbs"), out.pop("_d2h_gbs"), out.pop("_duplex_ms")])
    out.update(e2e_rank_summary(ranks, out["ms_per_step"]))
    out["ceiling_note"] = (
        "each step moves h2d_bytes_per_step + d2h_bytes_per_step per rank over its PCIe link; h2d_gbs / d2h_gbs "
        "are each direction alone, copy_floor_ms one step's copy-in and copy-out issued together on two streams "
        "(both directions at once, as the e2e loop overlaps them), the slowest rank's; of_copy_floor = "
        "copy_floor_ms / ms_per_step"
    )
    return out


def e2e_rank_summary(ranks: list[list[float]], ms_per_step: float) -> dict:
    """The e2e record's per-rank part from every rank's gathered [NUMA node, H2D GB/s, D2H GB/s,
    copy floor ms]: `per_rank`, the slowest rank's `copy_floor_ms`, and `of_copy_floor` (that floor
    over the e2e step time, the max over ranks)."""
    floor = max(v[3] for v in ranks)
    return {
        "per_rank": [
            {"rank": r, "numa_node": int(v[0]), "h2d_gbs": round(v[1], 1), "d2h_gbs": round(v[2], 1), "copy_floor_ms": round(v[3], 4)}
            for r, v in enumerate(ranks)
        ],
        "copy_floor_ms": round(floor, 4),
        "of_copy_floor": round(floor / ms_per_step, 3),
    }


def _run_e2e(cufk, host, dev, args, dist: Dist, global_batch: int) -> dict:
    """The metric through the public API with host buffers: every step copies the inputs and the
    grad host->device from pinned memory, runs ``cufk_b200.reconstruct`` + ``backward`` and copies
    xyz and the three gradients device->host.  Copy-in, compute and copy-out are on three streams,
    and alternate steps use two device input sets, so that one step's results travel back while
    the next step's inputs arrive (both PCIe directions at once), as a caller streaming batches
    would run it."""
    b = host["lengths"].shape[0]
    pinned = {k: v.pin_memory() for k, v in host.items()}
    outs = {
        "xyz": torch.empty(b, args.points, 3).pin_memory(),
        "gl": torch.empty_like(host["lengths"]).pin_memory(),
        "ga": torch.empty_like(host["angles"]).pin_memory(),
        "gd": torch.empty_like(host["dihedrals"]).pin_memory(),
    }
    h2d = sum(v.numel() * v.element_size() for v in pinned.values())
    d2h = sum(v.numel() * v.element_size() for v in outs.values())
    # two device input sets, used by alternate steps: a step's copy-in waits only for the compute two
    # steps back, so it runs while the previous step computes and copies out
    bufs = [{k: torch.empty_like(v, device=dev) for k, v in host.items()} for _ in range(2)]
    buf = bufs[0]
    s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    free = [None, None]
    turn = [0]

    def step():
        slot = turn[0]
        turn[0] ^= 1
        b = bufs[slot]
        with torch.cuda.stream(s_in):
            if free[slot] is not None:
                s_in.wait_event(free[slot])  # the compute that last read this input set is done
            for k in ("lengths", "angles", "dihedrals", "grad"):
                b[k].copy_(pinned[k], non_blocking=True)
            copied = torch.cuda.Event()
            copied.record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(copied)
            L, A, D = (b[k].detach().requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
            xyz = cufk.reconstruct(L, A, D)
            xyz.backward(b["grad"])
            done = torch.cuda.Event()
            done.record(s_run)
            free[slot] = done
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for src, key in ((xyz.detach(), "xyz"), (L.grad, "gl"), (A.grad, "ga"), (D.grad, "gd")):
                src.record_stream(s_out)
                outs[key].copy_(src, non_blocking=True)

    steps = min(args.steps, 100)
    for _ in range(max(3, min(args.warmup, 10))):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(cur)
    for st in (s_in, s_run, s_out):
        st.wait_stream(cur)
    for _ in range(steps):
        step()
    for st in (s_in, s_run, s_out):
        cur.wait_stream(st)
    s1.record(cur)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(s0.elapsed_time(s1)) / steps
    # the results arrived: check them against a direct call
    ref = cufk.reconstruct(pinned["lengths"].to(dev), pinned["angles"].to(dev), pinned["dihedrals"].to(dev))
    assert torch.equal(outs["xyz"], ref.cpu()), "e2e output mismatch"
    # copy-only rates of this rank's link, each direction alone (all ranks at once)
    def copy_rate(direction):
        reps = 10
        with torch.cuda.stream(s_in):
            for _ in range(2):
                copy_once(direction)
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s_in)
            for _ in range(reps):
                copy_once(direction)
            e1.record(s_in)
            torch.cuda.synchronize()
        nbytes = h2d if direction == "h2d" else d2h
        return nbytes * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9

    dev_out = {k: torch.empty_like(v, device=dev) for k, v in outs.items()}

    def copy_once(direction):
        if direction == "h2d":
            for k in ("lengths", "angles", "dihedrals", "grad"):
                buf[k].copy_(pinned[k], non_blocking=True)
        else:
            for k, v in outs.items():
                v.copy_(dev_out[k], non_blocking=True)

    def duplex_ms():
        # one step's copy-in and copy-out issued together on two streams (both PCIe directions at
        # once, as the e2e loop overlaps them): the copy floor of an e2e step
        reps = 10
        for _ in range(2):
            copy_once("h2d")
            copy_once("d2h")
        torch.cuda.synchronize()
        dist.barrier()
        cur = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        for _ in range(reps):
            with torch.cuda.stream(s_in):
                copy_once("h2d")
            with torch.cuda.stream(s_out):
                copy_once("d2h")
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)
        e1.record(cur)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    h2d_gbs, d2h_gbs = copy_rate("h2d"), copy_rate("d2h")
    both_ms = duplex_ms()
    return {
        "value": global_batch * args.points / (ms * 1e-3),
        "unit": "atoms/s",
        "h2d_bytes_per_step": h2d,
        "d2h_bytes_per_step": d2h,
        "ms_per_step": ms,
        "steps": steps,
        "path": "cufk_b200.reconstruct + autograd backward; pinned host buffers, copies inside the timed region; copy-in / compute / copy-out on three streams, two device input sets alternating",
        "_h2d_gbs": h2d_gbs,
        "_d2h_gbs": d2h_gbs,
        "_duplex_ms": both_ms,
    }


# ------------------------------------------------------------------------------------------------
# CPU baseline and the reference arm: the float64 restatement on the host cores
# ------------------------------------------------------------------------------------------------
def _cpu_sample(points: int, chains: int):
    from oracle import nerf64

    inp = make_inputs(chains, points, seed=1)

    def once():
        nerf64.reconstruct64_with_grads(inp["lengths"], inp["angles"], inp["dihedrals"], inp["grad"])

    return once


def cpu_baseline(points: int, budget_s: float = 12.0, chains: int = 256) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    once = _cpu_sample(points, chains)
    once()  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        once()
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return {
        "value": chains * points / dt,
        "unit": "atoms/s",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{chains} chains x N={points} fwd+bwd (float64 torch, autograd backward), {reps} reps in {budget_s:.0f}s",
    }


def workload_inputs(kind: str, batch: int, points: int, dtype, anchors: bool, seed: int) -> dict:
    """Seeded synthetic inputs of one configuration, generated in float64 on the CPU then cast:
    block rows as in ``make_inputs`` (anchors: p0 ~ N(0,1)^3, first_direction / initial_normal a
    random orthonormal pair); torsion raw pairs (B, 2(N-3)) ~ N(0,1); grad_out ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    f64 = torch.float64
    out = {}
    if kind in ("block", "mse"):
        base = make_inputs(batch, points, seed=seed)
        out = {k: base[k].to(f64).to(dtype) for k in ("lengths", "angles", "dihedrals", "grad")}
        if kind == "mse":
            # a target: the grad tensor's shape, values of the coordinate scale
            out["target"] = (3.0 * out.pop("grad").to(f64)).to(dtype)
        if anchors:
            q, _ = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=f64))
            out["p0"] = torch.randn(3, generator=g, dtype=f64).to(dtype)
            out["first_direction"] = q[:, 0].contiguous().to(dtype)
            out["initial_normal"] = q[:, 1].contiguous().to(dtype)
    else:
        out["raw"] = torch.randn(batch, 2 * (points - 3), generator=g, dtype=f64).to(dtype)
        out["grad"] = torch.randn(batch, points, 3, generator=g, dtype=f64).to(dtype)
    return out


def run_workload(args, dist: Dist) -> dict:
    """One configuration other than the headline: forward + backward (the kernels autograd runs)
    on this rank's shard, CUDA graphs over rotating input sets, per-kernel launch times and
    algorithmic-byte rooflines."""
    sys.path.insert(0, str(ROOT))
    import cufk_b200  # noqa: F401
    from cufk_b200 import _native
    from cufk_b200.torsion import torsion_constants

    C = _native._C
    kind, batch, points, dtype, anchors = WORKLOADS[args.workload]
    dev = torch.device("cuda", torch.cuda.current_device())
    host, global_batch = rank_inputs(
        lambda b, seed: workload_inputs(kind, b, points, dtype, anchors, seed=seed), batch, args.scaling, dist.world, dist.rank
    )
    elem = torch.empty(0, dtype=dtype).element_size()
    b_local = host["grad" if "grad" in host else "target"].shape[0]
    steps_s = points - 3
    if kind == "block":
        fwd_b, bwd_b = (6 * points - 6) * elem, (9 * points - 12) * elem
        if elem == 2:
            # the 16-bit forward also writes float32 positions, which its backward reads
            names = ("block_forward_kernel", "block_backward_xyz32_kernel")
        else:
            vec = elem == 4 or points <= VEC_MAX_POINTS_LONG
            names = (
                "block_forward_vec_kernel" if vec else "block_forward_kernel",
                "block_backward_xyz_vec_kernel" if points <= VEC_MAX_POINTS_LONG else "block_backward_xyz_kernel",
            )
    elif kind == "mse":
        # one kernel: read lengths/angles/dihedrals and the target, write the three gradient rows
        fwd_b, bwd_b = (9 * points - 12) * elem, 0
        names = ("block_mse_kernel", None)
    else:
        fwd_b, bwd_b = (2 * steps_s + 3 * points) * elem, (4 * steps_s + 3 * points) * elem
        # the 16-bit forward also writes float32 positions, which its backward reads
        names = ("torsion_forward_kernel", "torsion_backward_xyz_vec_kernel" if elem >= 4 else "torsion_backward_xyz32_kernel")
    set_bytes = b_local * (fwd_b + bwd_b)
    n_sets = max(2, min(16, math.ceil(3 * L2_BYTES / max(set_bytes, 1))))
    consts = torsion_constants(BACKBONE_LENGTHS, BACKBONE_ANGLES)
    sets = []
    for i in range(n_sets):
        d = {k: v.to(dev) for k, v in host.items()}
        if kind in ("block", "mse"):
            d["dihedrals"] = d["dihedrals"] + 1e-3 * i
        else:
            d["raw"] = d["raw"] + 1e-3 * i
        sets.append(d)
    anchor_args = lambda d: (d.get("p0"), d.get("first_direction"), d.get("initial_normal"))  # noqa: E731

    def unfused(d):
        # the sequence the fused kernel replaces: forward, the loss and dL/dxyz in torch, backward
        xyz = C.block_forward(d["lengths"], d["angles"], d["dihedrals"], None, None, None)
        diff = xyz - d["target"]
        d["loss_unfused"] = (diff * diff).sum(-1).mean(-1)
        return C.block_backward_from_xyz(d["lengths"], d["angles"], d["dihedrals"], None, None, None, xyz, diff * (2.0 / points))

    def fwd(d):
        if kind == "mse":
            return C.block_mse(d["lengths"], d["angles"], d["dihedrals"], None, None, None, d["target"], True)
        if kind == "block" and elem == 2:
            return C.block_forward_xyz32(d["lengths"], d["angles"], d["dihedrals"], *anchor_args(d))
        if kind == "block":
            return C.block_forward(d["lengths"], d["angles"], d["dihedrals"], *anchor_args(d))
        if elem == 2:
            return C.torsion_forward_xyz32(d["raw"], consts)
        return C.torsion_forward(d["raw"], consts)

    def bwd(d, xyz):
        if kind == "block" and elem == 2:
            return C.block_backward_from_xyz32(d["lengths"], d["angles"], d["dihedrals"], *anchor_args(d), xyz[1], d["grad"])
        if kind == "block":
            return C.block_backward_from_xyz(d["lengths"], d["angles"], d["dihedrals"], *anchor_args(d), xyz, d["grad"])
        if elem == 2:
            return C.torsion_backward_from_xyz32(d["raw"], consts, xyz[1], d["grad"])
        return C.torsion_backward_from_xyz(d["raw"], consts, xyz, d["grad"])

    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    g_step, g_fwd, g_bwd, g_unfused = [], [], [], []
    with torch.cuda.stream(stream):
        for d in sets:
            d["xyz"] = fwd(d)
            if kind == "mse":
                unfused(d)
            else:
                bwd(d, d["xyz"])
        stream.synchronize()
        # `per` consecutive sets per graph, as for the headline: the device's per-replay launch gap
        # stays out of the per-step time
        per = max(1, min(args.per_graph, args.steps))
        for i in range(n_sets):
            group = [sets[(i + r) % n_sets] for r in range(per)]
            if kind == "mse":
                bodies = ((g_step, lambda g=group: [fwd(d) for d in g]), (g_unfused, lambda g=group: [unfused(d) for d in g]))
            else:
                bodies = (
                    (g_step, lambda g=group: [bwd(d, fwd(d)) for d in g]),
                    (g_fwd, lambda g=group: [fwd(d) for d in g]),
                    (g_bwd, lambda g=group: [bwd(d, d["xyz"]) for d in g]),
                )
            for lst, body in bodies:
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    body()
                lst.append(gr)
    torch.cuda.synchronize()
    replays = max(1, args.steps // per)

    def ms_per_step(graphs):
        return statistics.median(time_graphs(graphs, replays, max(1, args.warmup // per), dist, stream, args.repeats)) / (replays * per)

    sampler = ClockSampler(dev.index)
    extra = {}
    with torch.cuda.stream(stream):
        with sampler:
            ms_step = ms_per_step(g_step)
        if kind == "mse":
            ms_fwd, ms_bwd = ms_step, 0.0
            ms_unfused = ms_per_step(g_unfused)
            extra["unfused"] = {
                "ms_per_step": ms_unfused,
                "value": batch * points / (ms_unfused * 1e-3),
                "sequence": "block_forward_kernel, torch loss and dL/dxyz (3 elementwise/reduction kernels), block_backward_xyz_kernel",
            }
        else:
            ms_fwd = ms_per_step(g_fwd)
            ms_bwd = ms_per_step(g_bwd)
    peak, peak_kind = measured_peak()
    per_kernel = {}
    for name, ms, nbytes in ((names[0], ms_fwd, fwd_b), (names[1], ms_bwd, bwd_b)):
        if name is None:
            continue
        gbs = nbytes * b_local / (ms * 1e-3) / 1e9
        per_kernel[name] = {"launch_ms": round(ms, 5), "bytes_per_atom": round(nbytes / points, 3), "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
    dom = max(per_kernel, key=lambda k: per_kernel[k]["launch_ms"])
    return {
        "metric": f"fwd+bwd atoms/s ({args.workload}: {kind}, B={batch}, N={points}, {str(dtype).replace('torch.', '')})",
        "value": global_batch * points / (ms_step * 1e-3),
        "unit": "atoms/s",
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": {torch.float32: "f32", torch.float64: "f64", torch.float16: "f16", torch.bfloat16: "bf16"}[dtype],
        "data": "synthetic (seeded, the distributions of the configuration)",
        "config": {
            "workload": args.workload,
            "kind": kind,
            "global_batch": global_batch,
            "points": points,
            "anchors": anchors,
            "per_gpu_batch": b_local,
            "l2": f"{n_sets} rotating input/output sets, {n_sets * set_bytes / 2**20:.0f} MiB",
            "timing": f"CUDA graphs of {per} steps each over rotating input sets, CUDA events, max over ranks, median of {args.repeats} repeats",
        },
        "roofline": {
            "kernel": dom,
            "bound": "hbm",
            "achieved": per_kernel[dom]["achieved_gbs"],
            "peak": peak,
            "unit": "GB/s",
            "frac": per_kernel[dom]["frac"],
            "peak_source": peak_kind,
            "traffic": None,
            "per_kernel": per_kernel,
            "step_frac": round((fwd_b + bwd_b) * b_local / (ms_step * 1e-3) / 1e9 / peak, 4),
        },
        "gpu_launches": (1 if names[1] is None else 2) * args.steps,
        "kernels": names[0] if names[1] is None else f"{names[0]} + {names[1]} per step",
        "clocks": sampler.summary(),
        **extra,
    }


def run_reference(args) -> dict | None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sys.path.insert(0, str(ROOT))
    torch.set_num_threads(os.cpu_count() or 1)
    chains = 64
    once = _cpu_sample(args.points, chains)
    for _ in range(max(1, args.warmup)):
        once()
    steps = args.steps
    t0 = time.perf_counter()
    for _ in range(steps):
        once()
    dt = (time.perf_counter() - t0) / steps
    value = chains * args.points / dt
    cores = torch.get_num_threads()
    sample = f"each step: {chains} of the {args.batch} chains x N={args.points} fwd+bwd in float64 torch (autograd backward)"
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "atoms/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic (seeded backbone internal coordinates)",
        "config": {
            "workload": "config 1: block reconstruct forward+backward, B=4096 chains, N=768 atoms",
            "global_batch": args.batch * (world if args.scaling == "weak" else 1),
            "points": args.points,
            "implementation": "the reference path has no CPU code; its algorithm restated in float64 torch (oracle/nerf64.py)",
        },
        "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        out = run_reference(args)
        if out is not None:
            print(json.dumps(out), flush=True)
        return 0
    # The JSON line is the only thing this process writes to its stdout: libraries that print there
    # from native code (NCCL's version line under NCCL_DEBUG=VERSION, for one) write to stderr while
    # the step runs, through a file descriptor 1 pointed at stderr.
    sys.stdout.flush()
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    dist = Dist(args.gpus)
    try:
        out = run_ours(args, dist) if args.workload == "cfg1" else run_workload(args, dist)
    finally:
        torch.cuda.synchronize()
        dist.close()
    if dist.rank == 0 and out is not None:
        print(json.dumps(out), file=json_out, flush=True)
    json_out.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
