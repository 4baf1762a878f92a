"""Times the reference's own CUDA kernels (built from its sources into oracle/_ref by
oracle/build_ref.py) against cufk_b200 on the same inputs, for every benchmark configuration.

MEASUREMENT OF THE REFERENCE, not part of the product.  Both sides run through their public
autograd path (reference: the restated Python layer of src/cufk/reconstruct.py:29-81 and the
torsion extension's ``apply``; cufk_b200: ``reconstruct`` / ``compile_torsion``): a step is the
forward plus ``backward`` of a fixed grad.  Inputs are device-resident; several input sets rotate
so that each step reads from HBM; CUDA events around ``--reps`` steps after warm-up.

    python oracle/compare_gpu.py [--reps 50] > compare.json
    python oracle/compare_gpu.py --accuracy > accuracy.json   # errors against float64
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import cufk_b200 as cufk  # noqa: E402
from oracle import nerf64, ref_kernels  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
ANCHOR_KEYS = ("p0", "first_direction", "initial_normal")


def _sets(make, nbytes):
    n = max(2, min(8, -(-3 * L2_BYTES // max(nbytes, 1))))
    return [make(i) for i in range(n)]


def _time(fn, sets, reps, warmup=5):
    for k in range(warmup):
        fn(sets[k % len(sets)])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for k in range(reps):
        fn(sets[k % len(sets)])
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3  # us


def block_case(batch, points, dtype, anchors, reps):
    host = nerf64.make_inputs(batch, points, seed=0, anchors=anchors)
    elem = torch.empty((), dtype=dtype).element_size()
    nbytes = batch * points * 9 * elem

    def make(i):
        d = {k: v.to("cuda", dtype) for k, v in host.items()}
        d["dihedrals"] = d["dihedrals"] + 1e-3 * i
        return d

    sets = _sets(make, nbytes)

    def step(fn, backward):
        def run(d):
            L, A, D = (d[k].requires_grad_(backward) for k in ("lengths", "angles", "dihedrals"))
            kw = {k: d[k] for k in ANCHOR_KEYS} if anchors else {}
            xyz = fn(L, A, D, **kw)
            if backward:
                xyz.backward(d["grad"])
                for t in (L, A, D):
                    t.grad = None

        return run

    out = {}
    for name, fn in (("reference", ref_kernels.ref_reconstruct), ("cufk_b200", cufk.reconstruct)):
        try:
            out[name] = {"fwd_us": round(_time(step(fn, False), sets, reps), 2), "fwd_bwd_us": round(_time(step(fn, True), sets, reps), 2)}
        except RuntimeError as exc:  # the reference refuses float64 backward above 1024 steps
            out[name] = {"error": str(exc).splitlines()[0]}
    return out


def torsion_case(batch, points, dtype, reps):
    host = nerf64.make_torsion_inputs(batch, points, seed=0)
    elem = torch.empty((), dtype=dtype).element_size()
    nbytes = batch * points * 7 * elem
    f = cufk.compile_torsion(nerf64.BACKBONE_LENGTHS, nerf64.BACKBONE_ANGLES)

    def make(i):
        return {"raw": host["raw"].to("cuda", dtype) + 1e-3 * i, "grad": host["grad"].to("cuda", dtype)}

    sets = _sets(make, nbytes)

    def step(fn, backward):
        def run(d):
            raw = d["raw"].requires_grad_(backward)
            xyz = fn(raw)
            if backward:
                xyz.backward(d["grad"])
                raw.grad = None

        return run

    out = {}
    for name, fn in (("reference", ref_kernels.ref_torsion), ("cufk_b200", f)):
        out[name] = {"fwd_us": round(_time(step(fn, False), sets, reps), 2), "fwd_bwd_us": round(_time(step(fn, True), sets, reps), 2)}
    return out


def _errors(fn, inp, dtype, anchors):
    """max-abs xyz error and worst gradient relative-L2 error against the float64 oracle, for inputs
    cast to `dtype` (the oracle sees the same rounded inputs)."""
    L, A, D = (inp[k].to("cuda", dtype).requires_grad_(True) for k in ("lengths", "angles", "dihedrals"))
    kw = {k: inp[k].to("cuda", dtype) for k in ANCHOR_KEYS} if anchors else {}
    xyz = fn(L, A, D, **kw)
    xyz.backward(inp["grad"].to("cuda", dtype))
    c = {k: v.to(dtype).double() for k, v in inp.items()}
    ref = nerf64.reconstruct64_with_grads(c["lengths"], c["angles"], c["dihedrals"], c["grad"], **({k: c[k] for k in ANCHOR_KEYS} if anchors else {}))
    xerr = float((xyz.detach().double().cpu() - ref[0]).abs().max())
    gerr = max(float((g.double().cpu() - r).norm() / r.norm()) for g, r in zip((L.grad, A.grad, D.grad), ref[1:]))
    return {"xyz_max_abs": xerr, "grad_rel_l2": gerr}


def accuracy() -> dict:
    out = {}
    for name, batch, points, dtype, anchors in (
        ("config2 fp32 B=16 N=2051 anchors", 16, 2051, torch.float32, True),
        ("config4 fp16 B=64 N=1026", 64, 1026, torch.float16, False),
        ("config4 bf16 B=64 N=1026", 64, 1026, torch.bfloat16, False),
    ):
        inp = nerf64.make_inputs(batch, points, seed=points, anchors=anchors)
        out[name] = {"reference": _errors(ref_kernels.ref_reconstruct, inp, dtype, anchors), "cufk_b200": _errors(cufk.reconstruct, inp, dtype, anchors)}
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--accuracy", action="store_true", help="errors against float64 instead of timings")
    args = ap.parse_args()
    if not (ref_kernels.available("block") and ref_kernels.available("torsion")):
        raise SystemExit("reference kernels not built (python oracle/build_ref.py)")
    if args.accuracy:
        print(json.dumps(accuracy(), indent=1))
        return
    r = args.reps
    res = {
        "config0 block B=64 N=384 fp32": block_case(64, 384, torch.float32, False, r),
        "config1 block B=4096 N=768 fp32": block_case(4096, 768, torch.float32, False, r),
        "config2 block B=2048 N=2051 fp32 anchors": block_case(2048, 2051, torch.float32, True, r),
        "config2 block B=2048 N=2051 fp64 anchors": block_case(2048, 2051, torch.float64, True, r),
        "config3 torsion B=16384 N=768 fp32": torsion_case(16384, 768, torch.float32, r),
        "config3 torsion B=16384 N=768 bf16": torsion_case(16384, 768, torch.bfloat16, r),
        "config4 block B=8192 N=1026 fp16": block_case(8192, 1026, torch.float16, False, r),
        "config4 block B=8192 N=1026 bf16": block_case(8192, 1026, torch.bfloat16, False, r),
        "config4 single chain N=2051 fp32": block_case(1, 2051, torch.float32, False, r),
    }
    for v in res.values():
        a, b = v.get("reference", {}), v.get("cufk_b200", {})
        for key in ("fwd_us", "fwd_bwd_us"):
            if key in a and key in b:
                v[f"speedup_{key[:-3]}"] = round(a[key] / b[key], 2)
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
