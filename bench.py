"""Benchmark of the B200 BiGEMM hot path (one JSON line on rank 0).

Workload (the operator sweep the metric is quoted on):
B=128 per GPU, bf16 compute with fp32 accumulation, forward + backward
(dX and all weight gradients) of every stage shape {56x56x128 d64,
28x28x256 d64, 14x14x512 d128, 7x7x1024 d128} under each of the local,
shifted and radix routes, radix at levels 0, 1 and 2 (levels 1 and 2 gather
channel groups with stride Q_c).  One step = those 20 fwd+bwd calls.  Inputs
are seeded synthetic tensors in config 2's order: ``torch.manual_seed(1)``,
an fp32 ``OmniWeaveBlock`` with default init, then x and dY ~ N(0,1) (drawn
on the device), all cast to bf16.  The per-step working set (~2 GB) is far
larger than the 126 MB L2, so every step streams from HBM.

``value`` = algorithmic FLOPs of all ranks / max-over-ranks device time
(CUDA events, inputs resident in HBM).  FLOPs per tile follow the operator
definition: fwd = 4g^2 d + 2g^2 rd + 6 g d rd over padded tiles, bwd = 2x fwd.
``e2e`` = the same FLOPs timed through the public ``bigemm`` API with inputs
copied from pinned host memory and outputs and gradients copied back inside
the timed region.

``--impl reference`` times the reference's own implementation of the path,
``bigemm_delta_reference`` plus torch autograd (omniweave/ops/reference.py,
from the unmodified install under baseline/_ref), on the host cores with
every thread, in bf16 on a B=8 sample of each of the 20 cases per step.
Under torchrun only rank 0 runs it.  ``cpu_baseline`` in the main line is
the same measurement, bounded to ~10 s.

Multi-GPU: one process per GPU; the batch is sharded (each rank runs its own
B=128 sweep, no data-path collective), so scaling is weak.

The same line carries ``omniweave_t``: the reference's own OmniWeave-T
(``omniweave.models.registry.create_model``) with ``backend="cuda"``
installed by ``omniwave_b200.integration`` (random init broadcast from rank
0, synthetic N(0,1) images, per-rank seeds) measured as BASELINE configs
3-5 -- bf16 inference at 256 images per GPU, batch-sharded with no
communication, and the training step at 128 images per GPU (bf16 autocast,
cross-entropy on uniform labels, AdamW lr 1e-3 wd 0.05; one CUDA graph per
step on one GPU, DDP with NCCL gradient all-reduce on several).  Images/s
are whole-job totals over max-over-ranks time.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SHAPES = [(56, 56, 128, 64), (28, 28, 256, 64), (14, 14, 512, 128), (7, 7, 1024, 128)]
ROUTES = [("local", 0), ("shifted", 0), ("radix", 0), ("radix", 1), ("radix", 2)]
BATCH = 128
G = 16
METRIC = "BiGEMM TFLOP/s (fwd+bwd, bf16, operator sweep B=128)"
_COMPUTE = {"bf16": torch.bfloat16, "fp32": torch.float32}
REF_SITE = os.path.join(ROOT, "baseline", "_ref")


def fwd_flops(b: int, h: int, w: int, c: int, d: int) -> float:
    qs = math.ceil(h * w / G)
    qc = math.ceil(c / d)
    rd = 2 * d
    return float(b * qs * qc * (4 * G * G * d + 2 * G * G * rd + 6 * G * d * rd))


def _kernel_flops(name: str, b: int, h: int, w: int, c: int, d: int) -> float:
    """Algorithmic FLOPs one launch of ``name`` accounts for.  The forward is
    split between its pack kernel (the input token mixes P_u = A_u T,
    P_v = A_v T) and the forward kernel (everything else); the backward's
    (2x forward) between the backward pack kernel, which does the three 16x16
    token mixes of the operands (P_u, P_v, dY'), and the role kernel."""
    tiles = b * math.ceil(h * w / G) * math.ceil(c / d)
    mixes = tiles * 3 * 2 * G * G * d
    if name == "tc_pack_fwd_kernel":
        return float(tiles * 4 * G * G * d)
    if name == "tc_fwd_kernel":  # its pre-pass did the input token mixes (strided channel groups)
        return fwd_flops(b, h, w, c, d) - tiles * 4 * G * G * d
    if name == "tc_fwd_gather_kernel":  # the TMA-gather forward does the whole forward
        return fwd_flops(b, h, w, c, d)
    if name == "tc_pack_kernel":
        return float(mixes)
    return 2.0 * fwd_flops(b, h, w, c, d) - mixes


# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum), keyed by (kernel,
# case, batch), with the sha256 of the kernel's source file and the shared
# headers at capture time: a line whose sources differ reports traffic null
# instead of a stale figure.  The B=128 figure is the B=64 capture scaled by
# the items processed (the role kernel's traffic is per item: operand images
# in, dX out).
_KERNEL_SRC = {"tc_bwd_kernel": "ow_tc_bwd.cu", "tc_pack_kernel": "ow_tc_bwd.cu", "tcf_kernel": "ow_tcf.cu",
               "tc_fwd_kernel": "ow_tc.cu", "tc_fwd_gather_kernel": "ow_tcf.cu"}
_TRAFFIC = {
    ("tc_bwd_kernel", "56x56x128/radix1", 128): (2 * (541.915392e6 + 93.980928e6), "cb20fe4683d3ebcb08543c290d60815c09ec506ae55ba551c49fc0a086f1ec1e"),
    ("tc_bwd_kernel", "56x56x128/radix2", 128): (2 * (541.527552e6 + 94.035712e6), "cb20fe4683d3ebcb08543c290d60815c09ec506ae55ba551c49fc0a086f1ec1e"),
}


def _src_digest(kernel: str) -> str:
    import hashlib

    csrc = os.path.join(ROOT, "omniwave_b200", "csrc")
    files = [os.path.join(csrc, _KERNEL_SRC.get(kernel, "ow_api.cu"))]
    files += sorted(os.path.join(csrc, f) for f in os.listdir(csrc) if f.endswith((".cuh", ".h")))
    files.append(os.path.join(ROOT, "include", "omniwave_b200.h"))
    h = hashlib.sha256()
    for f in files:
        with open(f, "rb") as fh:
            h.update(os.path.basename(f).encode() + b"\0" + fh.read())
    return h.hexdigest()


def _traffic(kernel: str, case: str, batch: int):
    t = _TRAFFIC.get((kernel, case, batch))
    return t[0] if t is not None and t[1] == _src_digest(kernel) else None


def fwd_bytes(b, h, w, c, elem=2) -> float:
    return 2.0 * b * h * w * c * elem


def step_flops(batch: int) -> float:
    return sum(3.0 * fwd_flops(batch, h, w, c, d) for (h, w, c, d) in SHAPES for _ in ROUTES)


# ---------------------------------------------------------------------------
def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _make_case(h, w, c, d, route, level, batch, dev, seed, dtype=torch.bfloat16):
    """Operator tensors in BASELINE config 2's order: seed, an fp32
    ``OmniWeaveBlock`` with default init (orthogonal A_u/A_v, identity A_o,
    xavier B, gamma 1e-5), then x and dY ~ N(0,1), all cast to ``dtype``
    (bf16 as config 2; scripts/benchmark.py:56-110)."""
    from omniwave_b200 import OmniWeaveBlock

    torch.manual_seed(seed)
    blk = OmniWeaveBlock(h, w, c, d, route, level)
    tensors = {k: getattr(blk, k).detach().to(dev, dtype)
               for k in ("a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")}
    tensors["x"] = torch.randn(batch, h, w, c, device=dev).to(dtype)
    dout = torch.randn(batch, h, w, c, device=dev).to(dtype)
    return blk.plan, tensors, dout


class _Clocks:
    """nvidia-smi sampler running during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    from omniwave_b200 import _lib, bigemm

    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", device_id=dev,
                                             timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()
    if args.model_only:
        # Profiling aid: only the OmniWeave-T legs (no operator sweep).
        m = _model_bench(args, dev, world, rank, lib)
        if rank == 0:
            print(json.dumps({"impl": "ours", "model_only": True, "omniweave_t": m}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    names = ("x", "a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")

    batch = args.batch
    only = set(args.cases.split(",")) if args.cases else None
    cases = []
    for si, (h, w, c, d) in enumerate(SHAPES):
        for ri, (route, lvl) in enumerate(ROUTES):
            if only is not None and f"{h}x{w}x{c}/{route}{lvl}" not in only:
                continue
            plan, tensors, dout = _make_case(h, w, c, d, route, lvl, batch, dev, seed=1 + 1000 * rank,
                                             dtype=_COMPUTE[args.compute])
            leaves = {k: v.detach().requires_grad_(True) for k, v in tensors.items()}
            cases.append(dict(shape=(h, w, c, d), route=f"{route}{lvl}", plan=plan,
                              leaves=leaves, dout=dout))
    if not cases:
        raise SystemExit(f"--cases {args.cases!r} selects nothing")
    sweep_flops = sum(3.0 * fwd_flops(batch, *cs["shape"]) for cs in cases)
    case_names = sorted(f"{cs['shape'][0]}x{cs['shape'][1]}x{cs['shape'][2]}/{cs['route']}" for cs in cases)

    def one_case(cs, ev=None):
        # ev: call boundaries [0..2] and, through ow_profile_events, the
        # forward kernel [3, 4], the backward pack kernel [5, 6], the backward
        # role kernel [7, 8] and the forward pack kernel [9, 10] on the same
        # stream.
        if ev is not None:
            for k, i in ((0, 3), (1, 5), (2, 7), (3, 9)):
                lib.ow_profile_events(k, ctypes.c_void_p(ev[i].cuda_event), ctypes.c_void_p(ev[i + 1].cuda_event))
            ev[0].record()
        out = bigemm(plan=cs["plan"], backend="cuda", **cs["leaves"])
        if ev is not None:
            ev[1].record()
        grads = torch.autograd.grad(out, [cs["leaves"][k] for k in names], cs["dout"])
        if ev is not None:
            ev[2].record()
            for k in range(4):
                lib.ow_profile_events(k, None, None)
        return out, grads

    def step(evs=None):
        for i, cs in enumerate(cases):
            one_case(cs, None if evs is None else evs[i])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # --- device-timed region -------------------------------------------------
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(11)] for _ in cases]
           for _ in range(args.steps)]
    for e in (e for st in evs for ce in st for e in ce):
        e.record()  # torch creates the CUDA event on first record; the library needs the handle
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    launches0 = lib.ow_launch_count()
    clk = _Clocks(dev.index).__enter__()  # sampled over every timed region below
    t0.record()
    for s in range(args.steps):
        step(evs[s])
    t1.record()
    torch.cuda.synchronize()
    launches = lib.ow_launch_count() - launches0
    # Every wait in the kernels is bounded; a run in which one gave up is void.
    _lib.check_device_fault(dev.index, reset=False)
    if world > 1:
        torch.distributed.barrier()
    ms = t0.elapsed_time(t1)
    ms_t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    flops = sweep_flops * args.steps * world
    value = flops / (ms_max * 1e-3) / 1e12

    # Per-call breakdown (fwd / bwd of each case) and per-kernel launch times
    # from the in-region events.
    def mean_ms(i, a, b):
        return statistics.mean(evs[s][i][a].elapsed_time(evs[s][i][b]) for s in range(args.steps))

    per, kern = {}, {}
    for i, cs in enumerate(cases):
        per[(cs["shape"], cs["route"])] = (mean_ms(i, 0, 1), mean_ms(i, 1, 2))
        pre = mean_ms(i, 9, 10)
        fwd_name = "tc_fwd_kernel" if pre > 1e-3 else "tc_fwd_gather_kernel"
        kern[(cs["shape"], cs["route"])] = {"tc_pack_fwd_kernel": pre,
                                            fwd_name: mean_ms(i, 3, 4), "tc_pack_kernel": mean_ms(i, 5, 6),
                                            "tc_bwd_kernel": mean_ms(i, 7, 8)}
    # Dominant kernel: the single launch with the largest device time.
    dom_key, dom_name, dom_ms = max(((k, n, t) for k, v in kern.items() for n, t in v.items()),
                                    key=lambda x: x[2])
    (h, w, c, d), route = dom_key
    dom_flops = _kernel_flops(dom_name, batch, h, w, c, d)
    peaks = _peaks()
    # (The fp32 profiling mode runs no tensor-core kernel: no launch is timed.)
    achieved = dom_flops / (dom_ms * 1e-3) / 1e12 if dom_ms > 1e-4 else 0.0
    traffic = _traffic(dom_name, f"{h}x{w}x{c}/{route}", batch)

    # --- end-to-end through the public API with host buffers -----------------
    e2e = None if args.no_e2e else _e2e(args, cases, names, dev, world, sweep_flops)
    ref_gpu = None if args.no_ref_gpu else _ref_gpu_bench(args, cases, names, dev, batch)
    del cases
    torch.cuda.empty_cache()

    model_line = None
    if not args.no_model:
        model_line = _model_bench(args, dev, world, rank, lib)
    clk.__exit__(None, None, None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": args.compute,
            "data": "synthetic (seeded N(0,1) inputs and upstream grads, default-init weights)",
            "config": {
                "workload": "bigemm_sweep_fwd_bwd",
                "batch_per_gpu": batch,
                "global_batch": batch * world,
                "shapes": [f"{h}x{w}x{c}/d{d}" for (h, w, c, d) in SHAPES],
                "routes": [f"{r}{l}" for r, l in ROUTES],
                "cases": case_names if only is not None else "all",
                "parallelism": f"batch-shard x{world}",
                "l2": "per-step working set ~1 GB > 126 MB L2 (inputs larger than L2)",
                "flops_per_step_per_gpu": sweep_flops,
            },
            "roofline": {
                "bound": "tensor",
                "kernel": f"{dom_name} {h}x{w}x{c}/d{d} {route} B={batch}",
                "achieved": round(achieved, 3),
                "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_source": peaks["source"],
                "launch_ms": round(dom_ms, 4),
                "algorithmic_flops_per_launch": dom_flops,
                "traffic": traffic,
                "traffic_source": None if traffic is None else
                "ncu capture of this kernel and case at B=64 (dram__bytes_read.sum + dram__bytes_write.sum), "
                "scaled by the items to B=128; same kernel sources",
            },
            "per_call_ms": {f"{k[0][0]}x{k[0][1]}x{k[0][2]}/{k[1]}": [round(v[0], 4), round(v[1], 4)]
                            for k, v in per.items()},
            "per_call_ms_note": "[forward call, backward call] per case; radix1/radix2 gather "
                                "channel groups with stride Q_c",
            "route_totals_ms": {r: round(sum(v[0] + v[1] for k, v in per.items() if k[1] == r), 4)
                                for r in sorted({k[1] for k in per})},
            "per_kernel_ms": {f"{k[0][0]}x{k[0][1]}x{k[0][2]}/{k[1]}": {n: round(t, 4) for n, t in v.items()}
                              for k, v in kern.items()},
            "e2e": e2e,
            "gpu_launches": int(launches),
            "device_fault": _lib.device_fault(dev.index),
            "clocks": clk.summary(),
        }
        if model_line is not None:
            line["omniweave_t"] = model_line
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def _e2e(args, cases, names, dev, world, sweep_flops):
    """Same metric through ``bigemm`` with pinned host inputs and outputs.

    Every step copies each case's inputs and upstream gradient from pinned
    host memory and its output and all gradients back.  The copies are
    pipelined as a user of the API would schedule them: case i+1's inputs
    upload on one copy stream while case i computes, and case i's results
    download on a second copy stream."""
    from omniwave_b200 import bigemm

    host = []
    for cs in cases:
        hx = {k: v.detach().cpu().pin_memory() for k, v in cs["leaves"].items()}
        hd = cs["dout"].cpu().pin_memory()
        outs = {k: torch.empty(v.shape, dtype=v.dtype).pin_memory() for k, v in cs["leaves"].items()}
        hout = torch.empty(cs["leaves"]["x"].shape, dtype=torch.bfloat16).pin_memory()
        host.append((hx, hd, outs, hout))
    main = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    h2d = d2h = 0

    def upload(i):
        hx, hd, _, _ = host[i]
        with torch.cuda.stream(up):
            lv = {k: v.to(dev, non_blocking=True) for k, v in hx.items()}
            go = hd.to(dev, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(up)
        return lv, go, ev

    def run_step(count):
        nonlocal h2d, d2h
        up.wait_stream(main)
        nxt = upload(0)
        for i, cs in enumerate(cases):
            lv, go, ev = nxt
            if i + 1 < len(cases):
                nxt = upload(i + 1)
            main.wait_event(ev)
            for t in list(lv.values()) + [go]:
                t.record_stream(main)
            lv = {k: v.requires_grad_(True) for k, v in lv.items()}
            out = bigemm(plan=cs["plan"], backend="cuda", **lv)
            grads = torch.autograd.grad(out, [lv[k] for k in names], go)
            _, _, outs, hout = host[i]
            down.wait_stream(main)
            with torch.cuda.stream(down):
                out.record_stream(down)
                hout.copy_(out, non_blocking=True)
                for k, g in zip(names, grads):
                    g.record_stream(down)
                    outs[k].copy_(g, non_blocking=True)
            if count:
                h2d += sum(v.numel() * v.element_size() for v in host[i][0].values()) + go.numel() * go.element_size()
                d2h += out.numel() * out.element_size() + sum(g.numel() * g.element_size() for g in grads)
        main.wait_stream(down)

    steps = max(1, min(args.steps, 3))
    run_step(False)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        run_step(True)
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    val = sweep_flops * steps * world / (float(ms.item()) * 1e-3) / 1e12
    return {"value": round(val, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d // steps,
            "d2h_bytes_per_step": d2h // steps, "copies": "pinned host, pipelined on two copy streams"}


def _ref_gpu_bench(args, cases, names, dev, batch):
    """The reference's own GPU paths on this B200, same cases and inputs:
    its Triton forward (``_TritonBiGEMM``, ops/triton.py:90-292, with the
    fp32 reference backward it ships) and its ``reference`` backend
    (einsums, bf16) forward + backward.  A secondary point of comparison."""
    try:
        _reference_package()
        from omniweave.ops.reference import bigemm_delta_reference
        from omniweave.ops.triton import _TRITON_AVAILABLE, bigemm_delta_triton
    except ImportError as exc:
        return {"unavailable": f"reference package not installed ({exc})"}
    if not _TRITON_AVAILABLE:
        return {"unavailable": "triton is not importable"}
    reps = 2

    def timed(fn):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    out = {"batch": batch, "dtype": "bf16", "per_case_ms": {}}
    tot = {"triton_fwd": 0.0, "triton_fwd_bwd": 0.0, "reference_fwd_bwd": 0.0}
    fw = fb = 0.0
    try:
        for cs in cases:
            t = {k: v.detach() for k, v in cs["leaves"].items()}
            plan, dy = cs["plan"], cs["dout"]
            h, w, c, d = cs["shape"]
            f1 = fwd_flops(batch, h, w, c, d)

            def tri_fwd():
                with torch.no_grad():
                    bigemm_delta_triton(plan=plan, **t)

            def fwd_bwd(fn):
                lv = {k: v.requires_grad_(True) for k, v in ((k, t[k].clone()) for k in names)}
                o = fn(plan=plan, **lv)
                torch.autograd.grad(o, [lv[k] for k in names], dy.to(o.dtype))

            ms = (timed(tri_fwd), timed(lambda: fwd_bwd(bigemm_delta_triton)),
                  timed(lambda: fwd_bwd(bigemm_delta_reference)))
            key = f"{h}x{w}x{c}/{cs['route']}"
            out["per_case_ms"][key] = [round(m, 3) for m in ms]
            for k, m in zip(tot, ms):
                tot[k] += m
            fw += f1
            fb += 3.0 * f1
            torch.cuda.empty_cache()
    except Exception as exc:  # the reference's GPU code, not ours: record and go on
        out["error"] = f"{type(exc).__name__}: {exc}"[:300]
        return out
    out["per_case_ms_note"] = "[triton fwd, triton fwd + its fp32 reference bwd, reference backend fwd+bwd]"
    out["triton_fwd_tflops"] = round(fw / (tot["triton_fwd"] * 1e-3) / 1e12, 3)
    out["triton_fwd_bwd_tflops"] = round(fb / (tot["triton_fwd_bwd"] * 1e-3) / 1e12, 3)
    out["reference_fwd_bwd_tflops"] = round(fb / (tot["reference_fwd_bwd"] * 1e-3) / 1e12, 3)
    return out


MODEL_FWD_GFLOP_PER_IMG = 3.757  # OmniWeave-T at 224x224: 2.895 BiGEMM + 0.863 Linear


def _timed(fn, steps, warmup, dev, world):
    """Max-over-ranks device time (ms) of ``steps`` calls after ``warmup``."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    return float(ms.item())


def _reference_package():
    """Import the unmodified reference package from baseline/_ref (or the
    environment); raises ImportError when it is not installed."""
    if os.path.isdir(os.path.join(REF_SITE, "omniweave")) and REF_SITE not in sys.path:
        sys.path.append(REF_SITE)
    import omniweave  # noqa: F401

    return omniweave


def _model_bench(args, dev, world, rank, lib):
    """BASELINE configs 3-5 on the reference's own OmniWeave-T with the cuda backend."""
    from omniwave_b200 import _lib
    from omniwave_b200.train import TrainStep, broadcast_parameters

    try:
        _reference_package()
    except ImportError as exc:
        return {"model": "omniweave_t", "unavailable": f"reference package not installed ({exc})"}
    from omniwave_b200 import integration

    integration.install()
    from omniweave.models.registry import create_model

    out = {"model": "omniweave_t (reference modules, backend='cuda' via omniwave_b200.integration)",
           "input": "224x224", "data": "synthetic N(0,1), per-rank seeds"}
    # ---- inference (configs 3/4): bf16 weights, 256 images per GPU
    torch.manual_seed(0)
    model = create_model("omniweave_t", backend="cuda").to(dev)
    broadcast_parameters(model)
    model = model.to(torch.bfloat16).eval()
    bi = args.model_batch or 256
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    imgs = torch.randn(bi, 3, 224, 224, device=dev, generator=g, dtype=torch.bfloat16)

    @torch.no_grad()
    def infer():
        model(imgs)

    ms = _timed(infer, args.model_steps, args.warmup, dev, world)
    out["infer_batch_per_gpu"] = bi
    out["infer_img_per_s"] = round(bi * world * args.model_steps / (ms * 1e-3), 1)
    out["infer_ms_per_step"] = round(ms / args.model_steps, 3)
    out["infer_tflops"] = round(bi * world * args.model_steps / (ms * 1e-3) * MODEL_FWD_GFLOP_PER_IMG / 1e3, 2)
    del model, imgs
    torch.cuda.empty_cache()
    # ---- training step (config 5): AdamW, bf16 autocast, 128 per GPU; one
    # CUDA graph per step on one GPU, DDP (NCCL all-reduce) on several
    torch.manual_seed(0)
    model = create_model("omniweave_t", backend="cuda").to(dev)
    graph = world == 1 and not args.no_graph
    ts = TrainStep(model, lr=1e-3, weight_decay=0.05, amp_dtype=torch.bfloat16, cuda_graph=graph,
                   graph_warmup=2)
    bt = args.model_batch or 128
    x = torch.randn(bt, 3, 224, 224, device=dev, generator=g)
    y = torch.randint(0, 1000, (bt,), device=dev, generator=g)
    launches0 = lib.ow_launch_count()
    ms = _timed(lambda: ts.step(x, y), args.model_steps, max(args.warmup, 3), dev, world)
    ts.check_finite()
    _lib.check_device_fault(dev.index, reset=False)
    img_s = bt * world * args.model_steps / (ms * 1e-3)
    out["train_batch_per_gpu"] = bt
    out["train_img_per_s"] = round(img_s, 1)
    out["train_ms_per_step"] = round(ms / args.model_steps, 3)
    out["train_tflops"] = round(img_s * 3 * MODEL_FWD_GFLOP_PER_IMG * 1e9 / 1e12, 2)
    out["train_parallelism"] = f"DDP x{world} (NCCL bucketed all-reduce)" if world > 1 else "single GPU"
    out["train_cuda_graph"] = graph
    out["bigemm_launches_in_train_region"] = (
        int(lib.ow_launch_count() - launches0) if not graph else
        "inside one CUDA graph per step (launch counter counts host-side launches only)")
    del ts, model, x, y
    torch.cuda.empty_cache()
    if world == 1:
        out["pool_head"] = _head_bench(dev)
    return out


def _head_bench(dev):
    """The model's tail, ``head(stage4.mean(dim=(1, 2)))``, at the two model
    workloads: the fused pool + head kernel (``omniwave_b200.head``) against
    PyTorch's mean + ``nn.Linear`` (cuBLAS).  Device time per call from a
    CUDA graph of eight calls on eight different inputs (205 MB > L2)."""
    from omniwave_b200 import head

    def graph_us(fns, reps=20):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for f in fns:
                f()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for f in fns:
                f()
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps / len(fns)
        del g
        return round(us, 2)

    res = {"timing": "device time per call, CUDA graph of 8 calls on 8 inputs (> L2)"}
    gen = torch.Generator(device=dev).manual_seed(7)
    for name, b, xdt, amp in (("infer_b256_bf16", 256, torch.bfloat16, False),
                              ("train_b128_f32_autocast", 128, torch.float32, True)):
        xs = [torch.randn(b, 7, 7, 1024, device=dev, generator=gen).to(xdt) for _ in range(8)]
        lin = torch.nn.Linear(1024, 1000).to(dev)
        if not amp:
            lin = lin.to(xdt)
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=amp):
            fused = graph_us([lambda x=x: head.pool_head(x, lin.weight, lin.bias) for x in xs])
            ref = graph_us([lambda x=x: lin(x.mean(dim=(1, 2))) for x in xs])
        res[name] = {"fused_us": fused, "torch_mean_linear_us": ref,
                     "fused_gbs": round(xs[0].numel() * xs[0].element_size() / (fused * 1e-6) / 1e9, 1)}
        del xs, lin
    torch.cuda.empty_cache()
    return res


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return {"bf16_tflops": float(j["bf16_tflops"]), "hbm_gbs": float(j["hbm_gbs"]),
                "source": "measured (MEASURED_PEAKS.json, burst)"}
    except (OSError, KeyError, ValueError):
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# CPU legs: the reference's own implementation on the host cores
# ---------------------------------------------------------------------------
CPU_SAMPLE_BATCH = 8
_WNAMES = ("a_u", "a_v", "a_o", "b_u", "b_v", "b_o", "gamma")


def _cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _cpu_model_name():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_ref_cases(batch, dtype):
    """The 20 sweep cases at ``batch``, in config 2's seed order, for the
    reference's ``bigemm_delta_reference``."""
    from omniweave.models.block import OmniWeaveBlock

    cases = []
    for (h, w, c, d) in SHAPES:
        for route, lvl in ROUTES:
            torch.manual_seed(1)
            blk = OmniWeaveBlock(h, w, c, d, route, lvl)
            x = torch.randn(batch, h, w, c).to(dtype).requires_grad_(True)
            dy = torch.randn(batch, h, w, c).to(dtype)
            ws = {k: getattr(blk, k).detach().to(dtype).requires_grad_(True) for k in _WNAMES}
            cases.append((blk.plan, x, ws, dy, 3.0 * fwd_flops(batch, h, w, c, d)))
    return cases


def _cpu_ref_sweep(cases):
    """One step: forward + autograd backward of every case (returns FLOPs)."""
    from omniweave.ops.reference import bigemm_delta_reference

    flops = 0.0
    for plan, x, ws, dy, f in cases:
        out = bigemm_delta_reference(x=x, plan=plan, **ws)
        torch.autograd.grad(out, [x] + list(ws.values()), dy.to(out.dtype))
        flops += f
    return flops


def _cpu_info(threads):
    return {"cores": threads, "nproc": os.cpu_count(), "cpu_model": _cpu_model_name(),
            "torch_threads": torch.get_num_threads()}


def _cpu_baseline(seconds):
    """Bounded CPU baseline for the main line: the reference implementation
    (bf16, every host thread) on a B=8 sample of the 20-case sweep."""
    threads = _cpu_threads()
    torch.set_num_threads(threads)
    try:
        _reference_package()
    except ImportError as exc:
        return {"value": None, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                "sample": f"unavailable: reference package not installed ({exc})"}
    cases = _cpu_ref_cases(CPU_SAMPLE_BATCH, torch.bfloat16)
    _cpu_ref_sweep(cases[:1])
    flops, reps = 0.0, 0
    t0 = time.perf_counter()
    while True:
        flops += _cpu_ref_sweep(cases)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    out = {"value": round(flops / el / 1e12, 5), "unit": "TFLOP/s", "kind": "reference",
           "sample": f"reference bigemm_delta_reference + autograd (torch CPU, bf16) fwd+bwd of the "
                     f"20-case sweep at B={CPU_SAMPLE_BATCH} (x{reps} repetitions, {el:.1f} s)"}
    out.update(_cpu_info(threads))
    return out


def _cpu_model_bench():
    """BASELINE's CPU model plan: the reference OmniWeave-T (reference backend)
    at B=8 -- inference fp32 and bf16 autocast, and an AdamW train step under
    bf16 autocast; min of 3 after 1 warm-up."""
    from omniweave.models.registry import create_model

    b = 8
    torch.manual_seed(0)
    model = create_model("omniweave_t")
    x = torch.randn(b, 3, 224, 224)
    y = torch.randint(0, 1000, (b,))
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3, weight_decay=0.05)

    def best(fn):
        fn()
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    def infer(amp):
        model.eval()
        with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16, enabled=amp):
            model(x)

    def train():
        model.train()
        with torch.autocast("cpu", dtype=torch.bfloat16):
            loss = torch.nn.functional.cross_entropy(model(x), y)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()

    return {"batch": b, "infer_fp32_img_per_s": round(b / best(lambda: infer(False)), 2),
            "infer_bf16_img_per_s": round(b / best(lambda: infer(True)), 2),
            "train_bf16_img_per_s": round(b / best(train), 2)}


def run_reference(args) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    threads = _cpu_threads()
    torch.set_num_threads(threads)
    try:
        _reference_package()
    except ImportError as exc:
        print(json.dumps({"impl": "reference", "unavailable": f"reference package not installed: {exc}"}),
              flush=True)
        return
    cases = _cpu_ref_cases(CPU_SAMPLE_BATCH, torch.bfloat16)
    for _ in range(args.warmup):
        _cpu_ref_sweep(cases)
    t0 = time.perf_counter()
    flops = 0.0
    for _ in range(args.steps):
        flops += _cpu_ref_sweep(cases)
    el = time.perf_counter() - t0
    val = flops / el / 1e12
    # fp32 once (the reference's default dtype), for the record.
    c32 = _cpu_ref_cases(CPU_SAMPLE_BATCH, torch.float32)
    t1 = time.perf_counter()
    f32 = _cpu_ref_sweep(c32)
    f32_val = f32 / (time.perf_counter() - t1) / 1e12
    del c32
    model = None if args.no_model else _cpu_model_bench()
    info = _cpu_info(threads)
    sample = (f"reference bigemm_delta_reference + autograd (torch CPU, bf16, {threads} threads) fwd+bwd "
              f"of the 20-case sweep at B={CPU_SAMPLE_BATCH} per step")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(val, 5),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (config 2 seed order: seed 1, default-init block, x and dY ~ N(0,1))",
        "config": {"workload": "bigemm_sweep_fwd_bwd", "batch_per_case_per_step": CPU_SAMPLE_BATCH,
                   "batch_note": "B=8 sample of the B=128 sweep (TFLOP/s is per-FLOP normalised)",
                   "shapes": [f"{h}x{w}x{c}/d{d}" for (h, w, c, d) in SHAPES],
                   "routes": [f"{r}{l}" for r, l in ROUTES]},
        "cpu_baseline": dict({"value": round(val, 5), "unit": "TFLOP/s", "kind": "reference",
                              "sample": sample}, **info),
        "fp32_value": round(f32_val, 5),
        "e2e": {"value": round(val, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if model is not None:
        line["omniweave_t_cpu"] = model
    print(json.dumps(line), flush=True)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model", action="store_true", help="skip the OmniWeave-T measurements")
    ap.add_argument("--model-steps", type=int, default=5)
    ap.add_argument("--batch", type=int, default=BATCH, help="operator-sweep batch per GPU")
    ap.add_argument("--cases", default="",
                    help="comma-separated subset of the sweep, e.g. 56x56x128/local0 (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-graph", action="store_true", help="train step without CUDA-graph capture")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip timing the reference's own GPU paths")
    ap.add_argument("--model-only", action="store_true", help="profiling aid: only the OmniWeave-T legs")
    ap.add_argument("--model-batch", type=int, default=0,
                    help="profiling aid: images per GPU for both OmniWeave-T legs (default 256 / 128)")
    ap.add_argument("--compute", choices=sorted(_COMPUTE), default="bf16",
                    help="profiling aid: operator-sweep dtype (fp32 runs the CUDA-core kernels)")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
