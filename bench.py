"""Headline benchmark: scanND (Scan-A) forward, 2D 64x64 grid, D=512, M=64,
batch 32 per GPU, reported as state-updates/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

* value  : device-resident inputs, CUDA-event time of K steps (max over
           ranks); one step = one scannd_forward_async() over the whole batch.
           Inputs (52.6 GB) are far larger than L2 (126 MB), so no flush.
* e2e    : the same metric through the public C ABI with HOST (pinned)
           buffers: scannd_batched() copies the inputs in, runs, copies h and y
           out and synchronises, every step.
* roofline: algorithmic bytes per launch (12 B per state update + 16 B per
           (point, channel)) / mean kernel time, against MEASURED_PEAKS.json.
* cpu_baseline: the reference's own scannd_ref (oracle/_ref, compiled from the
           reference sources) on a bounded sample of the same workload, all
           host threads, rank 0, N=1.
* other_configs (N=1): every other BASELINE config (--workload all: configs
           0-4 forward / backward / block / model), run in a child process
           after the headline and summarised in the same line (value, ms per
           step, roofline fraction, e2e, CPU-baseline rate).
Multi-GPU: one process per GPU (torchrun), every rank scans its own batch of
32 items (weak scaling); the scan has no cross-rank exchange in forward.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DIMS = (64, 64)
D, M, BATCH = 512, 64, 32
WORKLOAD = "scannd_fwd_2d64x64_D512_M64_b32"


def set_workload(dims, d, m, batch):
    """Headline by default; --batch/--dims/--D/--M shrink it for profiling runs."""
    global DIMS, D, M, BATCH, ND, P, UPDATES, ALG_BYTES, WORKLOAD
    DIMS, D, M, BATCH = tuple(dims), d, m, batch
    ND = len(DIMS)
    P = 1
    for v in DIMS:
        P *= v
    UPDATES = BATCH * P * D * M                                   # per GPU per step
    ALG_BYTES = UPDATES * 12 + BATCH * P * D * (4 + 4 * ND + 4)   # B,C read + h write; x, delta, y
    if (DIMS, D, M, BATCH) != ((64, 64), 512, 64, 32):
        WORKLOAD = "scannd_fwd_" + "x".join(map(str, DIMS)) + f"_D{D}_M{M}_b{BATCH} (non-headline)"


set_workload(DIMS, D, M, BATCH)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=BATCH, help="profiling override (default: headline 32)")
    ap.add_argument("--dims", type=int, nargs="+", default=list(DIMS))
    ap.add_argument("--D", type=int, default=D)
    ap.add_argument("--M", type=int, default=M)
    ap.add_argument("--workload", default="scan_fwd",
                    choices=["scan_fwd", "scan_fwd_c0", "scan_fwd_c1", "scan_fwd_3d", "scan_bwd", "scan_bwd_c1", "scan_bwd_3d", "convnd2d",
                             "convnd3d", "block", "block_bf16", "model", "all"],
                    help="scan_fwd = the headline line; the others measure the other BASELINE configs "
                         "(all = every other one, one line each)")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="N=1 headline run: skip the summary of the other BASELINE configs (one child process, ~35 s)")
    ap.add_argument("--chunks", type=int, default=4, help="N > 1: item chunks of the scan / gather overlap")
    ap.add_argument("--gather-mode", default="overlap", choices=["overlap", "after"],
                    help="N > 1: gather each chunk's y while the next is scanned, or all of y after the scan")
    ap.add_argument("--sm-reserve", type=int, default=0,
                    help="N > 1: SMs the scan leaves to the NCCL kernels (measured at N=2: 0 best, 9.9 vs 10.6 ms at 8)")
    ap.add_argument("--exp2", type=int, default=0,
                    help="exponential of the 2D forward: 0 default, 1 opt-in fast ex2.approx")
    a = ap.parse_args()
    set_workload(a.dims, a.D, a.M, a.batch)
    return a


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_uuid):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", dev_uuid, f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def make_inputs(dev, seed):
    import torch
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    f32 = torch.float32
    x = torch.randn((BATCH, P, D), generator=g, device=dev, dtype=f32)
    delta = torch.nn.functional.softplus(torch.randn((BATCH, ND, P, D), generator=g, device=dev) * 0.5 - 4.0)
    A = -torch.exp(torch.rand((ND, D, M), generator=g, device=dev) * torch.log(torch.tensor(16.0)))
    Bpm = torch.randn((BATCH, P, 1, M), generator=g, device=dev) * 0.25
    Cpm = torch.randn((BATCH, P, 1, M), generator=g, device=dev) * 0.25
    B = Bpm.expand(BATCH, P, D, M).contiguous()
    Cm = Cpm.expand(BATCH, P, D, M).contiguous()
    del Bpm, Cpm
    h = torch.empty((BATCH, P, D, M), device=dev)
    y = torch.empty((BATCH, P, D), device=dev)
    return dict(x=x, delta=delta, A=A, B=B, C=Cm, h=h, y=y)


def cpu_reference_rate(target_s=3.0, max_total_s=25.0):
    """scannd_ref (the reference's own code) on a bounded sample: one item,
    full 64x64 grid and M, a channel slice sized to ~target_s per call."""
    import numpy as np
    from oracle import pyoracle as po
    threads = po.set_threads(len(os.sched_getaffinity(0)) or os.cpu_count() or 1)
    d_s = 16
    t = None
    while True:
        inp = po.gen_scan(list(DIMS), d_s, M, batch=1, seed=3)
        t0 = time.perf_counter()
        po.ref_scannd(inp)
        t = time.perf_counter() - t0
        if t > target_s / 4 or d_s >= D:
            break
        d_s = min(D, d_s * 4)
    reps = max(1, min(5, int(max_total_s / max(t, 1e-3))))
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        po.ref_scannd(inp)
        times.append(time.perf_counter() - t0)
    upd = P * d_s * M
    return {"value": upd / statistics.median(times), "unit": "state-updates/s", "cores": threads,
            "kind": "reference",
            "sample": f"scannd_ref (oracle/_ref) on 1 item, 64x64 grid, D={d_s} of 512 channels, M=64; "
                      f"median of {reps} calls"}, times


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    import numpy as np
    from oracle import pyoracle as po
    threads = po.set_threads(len(os.sched_getaffinity(0)) or os.cpu_count() or 1)
    d_s = 64
    inp = po.gen_scan(list(DIMS), d_s, M, batch=1, seed=3)
    t0 = time.perf_counter()
    po.ref_scannd(inp)
    t = time.perf_counter() - t0
    # size each step to ~3 s of CPU work
    d_s = int(min(D, max(8, d_s * 3.0 / max(t, 1e-3)))) // 8 * 8 or 8
    inp = po.gen_scan(list(DIMS), d_s, M, batch=1, seed=3)
    for _ in range(args.warmup):
        po.ref_scannd(inp)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        po.ref_scannd(inp)
        times.append(time.perf_counter() - t0)
    upd = P * d_s * M
    value = upd * len(times) / sum(times)
    line = {"impl": "reference", "metric": "scanND state-updates/sec", "value": value,
            "unit": "state-updates/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE config-0 distributions)",
            "config": {"workload": WORKLOAD, "dims": list(DIMS), "D": D, "M": M, "batch": BATCH,
                       "sample_per_step": f"1 item, D={d_s} channels"},
            "cpu_baseline": {"value": value, "unit": "state-updates/s", "cores": threads, "kind": "reference",
                             "sample": f"scannd_ref (oracle/_ref, reference sources) 1 item x {d_s} channels "
                                       f"of the 64x64/M=64 workload per step"},
            "e2e": {"value": value, "unit": "state-updates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.workload != "scan_fwd":
        run_other_workload(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    import bissimamba_b200 as kmb

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    lib = kmb.lib()
    lib.kmb_set_scan_exp2(args.exp2)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    t = make_inputs(dev, seed=1234 + rank)
    p = kmb.scan_params(list(DIMS), D, M, t["x"], t["A"], t["B"], t["C"], t["delta"], t["h"], t["y"])
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    gather = None
    if world > 1:
        # The final output gather of the north star: every rank receives every rank's y over NCCL
        # (the library's own communicator, include/kmamba_distributed.h).  The batch is scanned in
        # item chunks and each chunk's y is gathered on a second stream while the next chunk is
        # scanned; the scan's persistent grid leaves a few SMs free for the NCCL kernels.
        from bissimamba_b200.distributed import Context
        if args.sm_reserve > 0:
            os.environ.setdefault("KMB_NCCL_MAX_CTAS", str(args.sm_reserve))   # NCCL fits in the SMs left free
        ctx = Context(world, rank)
        lib.kmb_set_sm_reserve(args.sm_reserve if args.gather_mode == "overlap" else 0)
        nch = max(1, min(args.chunks, BATCH))
        ipc = (BATCH + nch - 1) // nch
        chunks = []
        for c0 in range(0, BATCH, ipc):
            c1 = min(BATCH, c0 + ipc)
            sl = lambda k: t[k][c0:c1]
            chunks.append((c1 - c0, kmb.scan_params(list(DIMS), D, M, sl("x"), t["A"], sl("B"), sl("C"), sl("delta"),
                                                    sl("h"), sl("y"))))
        yall = torch.empty((world,) + tuple(t["y"].shape), device=dev)   # [chunk-major per rank] gathered y
        comm = torch.cuda.Stream(dev)
        cp = C.c_void_p(comm.cuda_stream)
        evs = [torch.cuda.Event() for _ in chunks]
        gather = dict(ctx=ctx, chunks=len(chunks), bytes_per_rank=t["y"].numel() * 4)

    def step():
        if world == 1:
            rc = lib.scannd_forward_async(C.byref(p), BATCH, sp)
            if rc != 0:
                raise RuntimeError(kmb.last_error())
            return
        if args.gather_mode == "after":
            kmb.check(lib.scannd_forward_async(C.byref(p), BATCH, sp))
            ctx.allgather(t["y"].data_ptr(), yall.data_ptr(), BATCH * P * D, sp)
            return
        off = 0
        for i, (nb, pc) in enumerate(chunks):
            kmb.check(lib.scannd_forward_async(C.byref(pc), nb, sp))
            evs[i].record(stream)
            comm.wait_event(evs[i])
            cnt = nb * P * D
            ctx.allgather(t["y"].data_ptr() + off * 4, yall.data_ptr() + off * world * 4, cnt, cp)
            off += cnt
        stream.wait_stream(comm)

    for _ in range(max(args.warmup, 3) if args.warmup >= 3 else 3):
        step()
    torch.cuda.synchronize()
    path = lib.kmb_last_forward_path()

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = str(local)
    clocks = ClockSampler(uuid)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    total_ms = max_over_ranks(t_start.elapsed_time(t_end))
    kern_ms = [a.elapsed_time(b) for a, b in ev]
    mean_kern_s = statistics.mean(kern_ms) / 1e3
    ms_per_step = total_ms / args.steps
    value = UPDATES * world * args.steps / (total_ms / 1e3)

    peak, peak_src = peaks()
    achieved = ALG_BYTES / mean_kern_s / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_src,
                # measured DRAM bytes of a launch come from ncu (profiles/scan_fwd_strips_headline.md),
                # not from this run
                "traffic": None,
                "alg_bytes_per_launch": ALG_BYTES, "kernel": ("scan_fwd_strips" if len(DIMS) == 2 else "scan_fwd_tma") if path == 1 else "scan_fwd_generic"}

    gather_info = None
    if gather is not None:
        # the gathers alone (no scan running), for the collective's share of the step
        def gathers():
            off = 0
            for nb, _ in chunks:
                cnt = nb * P * D
                gather["ctx"].allgather(t["y"].data_ptr() + off * 4, yall.data_ptr() + off * world * 4, cnt, cp)
                off += cnt
        gathers()
        torch.cuda.synchronize()
        g_ms = max_over_ranks(_events(comm, gathers, 5) / 5)
        gather_info = {"op": "ncclAllGather of y (every rank's outputs to every rank)", "chunks": gather["chunks"],
                       "bytes_received_per_rank_per_step": (world - 1) * gather["bytes_per_rank"],
                       "alone_ms": g_ms, "share_of_step_if_serial": round(g_ms / ms_per_step, 4),
                       "sm_reserve": args.sm_reserve, "mode": args.gather_mode,
                       "nccl_max_ctas": os.environ.get("KMB_NCCL_MAX_CTAS")}

    # the opt-in ex2.approx exponential on the same inputs (reported beside the default path)
    variants = {}
    if path == 1 and len(DIMS) == 2:
        lib.kmb_set_scan_exp2(0 if args.exp2 else 1)
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        vms = _events(stream, step, max(args.steps // 3, 5)) / max(args.steps // 3, 5)
        lib.kmb_set_scan_exp2(args.exp2)
        variants["exp2" if not args.exp2 else "expf"] = {
            "value": UPDATES * world / (vms / 1e3), "ms_per_step": vms,
            "hbm_frac": round(ALG_BYTES / (vms / 1e3) / 1e9 / peak, 4)}

    # ------------------------------------------------------------- e2e
    e2e = None
    if not args.no_e2e:
        # host RAM bound: the whole job pins at most one headline batch (52.6 GB)
        # of inputs + outputs, split over the ranks (the metric is a rate, so a
        # smaller per-rank batch measures the same quantity)
        eb = BATCH if world == 1 else max(1, BATCH // world)
        shapes = {k: ((eb,) + tuple(v.shape[1:]) if k != "A" else tuple(v.shape)) for k, v in t.items()}
        host = {}
        for k, v in t.items():
            hb = torch.empty(shapes[k], dtype=torch.float32, pin_memory=True)
            if k not in ("h", "y"):
                hb.copy_(v if k == "A" else v[:eb])
            host[k] = hb
        del t, p
        torch.cuda.empty_cache()
        ph = kmb.scan_params(list(DIMS), D, M, host["x"], host["A"], host["B"], host["C"], host["delta"],
                             host["h"], host["y"])
        rc = lib.scannd_batched(C.byref(ph), eb)   # warm-up: grows the staging workspace once
        if rc != 0:
            raise RuntimeError(kmb.last_error())
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            rc = lib.scannd_batched(C.byref(ph), eb)
            if rc != 0:
                raise RuntimeError(kmb.last_error())
        dt = max_over_ranks(time.perf_counter() - t0)
        h2d = sum(host[k].numel() * 4 for k in ("x", "A", "B", "C", "delta"))
        d2h = sum(host[k].numel() * 4 for k in ("h", "y"))
        e2e = {"value": (UPDATES // BATCH) * eb * world * args.e2e_steps / dt, "unit": "state-updates/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
               "ms_per_step": 1e3 * dt / args.e2e_steps, "batch_per_gpu": eb,
               "path": "scannd_batched() with pinned host buffers: H2D inputs, kernel, D2H h and y, pipelined by item chunks over three streams (PCIe-bound)"}
        del hb, ph

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu, _ = cpu_reference_rate()
        except Exception as exc:  # the reference build is test infrastructure: report, do not fail
            cpu = {"value": None, "error": str(exc)[:200]}

    others = None
    if rank == 0 and world == 1 and not args.no_other_configs:
        host = None   # the child pins its own host buffers: release the headline's first  # noqa: F841
        torch.cuda.empty_cache()
        if hasattr(torch._C, "_host_emptyCache"):
            torch._C._host_emptyCache()
        others = other_configs(args)

    if rank == 0:
        line = {"metric": "scanND state-updates/sec", "value": value, "unit": "state-updates/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, BASELINE config-0 distributions), generated on device",
                "config": {"workload": WORKLOAD, "dims": list(DIMS), "D": D, "M": M, "batch_per_gpu": BATCH,
                           "global_batch": BATCH * world, "rope": False, "lambda": "default 0.5",
                           "parallelism": (f"dp{world}: batch shards; every rank's y all-gathered to every rank "
                                           f"over NCCL inside the step, overlapped by item chunks")
                           if world > 1 else "dp1",
                           "l2": f"inputs {ALG_BYTES / 1e9:.1f} GB/GPU >> 126 MB L2, no flush"},
                "hbm_gbs": round(achieved, 1),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "exp": "expf, reference operation order" if not args.exp2 else "ex2.approx (opt-in)",
                "variants": variants,
                "gpu_launches": args.steps * (1 if world == 1 else gather["chunks"]), "clocks": clk,
                "collective": gather_info,
                "kernel_ms": {"mean": statistics.mean(kern_ms), "min": min(kern_ms), "max": max(kern_ms)},
                "other_configs": others}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------- other configs
# Every BASELINE config gets a full line: metric / value (device-resident
# inputs, CUDA-event time), roofline of the step, cpu_baseline (the reference's
# own CPU code on a bounded sample, rank 0 at N=1) and e2e (host buffers, the
# H2D copies of the step's inputs and the D2H copies of its results inside the
# timed region).  `--workload all` prints every line.
OTHER = ("scan_fwd_c0", "scan_fwd_c1", "scan_fwd_3d", "scan_bwd", "scan_bwd_c1", "scan_bwd_3d", "convnd2d", "convnd3d", "block", "block_bf16",
         "model")


def _events(stream, step, steps):
    """CUDA-event time (ms) of `steps` calls of step() on `stream`."""
    import torch
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def _timed(step, steps, warmup, stream):
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    return _events(stream, step, steps)


def _e2e(stream, host_in, dev_in, dev_out, host_out, call, steps, unit_count, unit):
    """Same metric through the C ABI with host buffers: every step copies the
    inputs in from pinned host memory, calls, and copies the results out."""
    import torch

    def step():
        for k in host_in:
            dev_in[k].copy_(host_in[k], non_blocking=True)
        call()
        for k in dev_out:
            host_out[k].copy_(dev_out[k], non_blocking=True)
    step()
    torch.cuda.synchronize()
    ms = _events(stream, step, steps)
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    d2h = sum(v.numel() * v.element_size() for v in host_out.values())
    return {"value": unit_count * steps / (ms / 1e3), "unit": unit, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms / steps, "steps": steps,
            "path": "pinned host inputs -> device (cudaMemcpyAsync), C-ABI call, results -> pinned host, same stream"}


def _pinned(t):
    import torch
    h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    h.copy_(t)
    return h


def _cpu_rate(fn, units, target_s=10.0, max_reps=5):
    """Median seconds of fn() (after one warm-up) -> units/s."""
    fn()
    times = []
    t_all = time.perf_counter()
    for _ in range(max_reps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > target_s:
            break
    return units / statistics.median(times), len(times)


def _scan_inputs(g, dev, dims, D_, M_, B_, rope):
    import torch
    P_ = int(np.prod(dims))
    nd = len(dims)
    rn = lambda *s: torch.randn(s, generator=g, device=dev)
    t = dict(x=rn(B_, P_, D_), delta=torch.nn.functional.softplus(rn(B_, nd, P_, D_) * 0.5 - 4.0),
             A=-torch.exp(torch.rand((nd, D_, M_), generator=g, device=dev) * float(np.log(16.0))),
             B=(rn(B_, P_, 1, M_) * 0.25).expand(B_, P_, D_, M_).contiguous(),
             C=(rn(B_, P_, 1, M_) * 0.25).expand(B_, P_, D_, M_).contiguous())
    t["theta"] = (torch.rand(D_ // 2, generator=g, device=dev) * 2 - 1) * float(np.pi) if rope else None
    return t


def wl_scan_fwd_small(args, dev, stream, lib, kmb, g, which, peak, peak_src, rank, world):
    """BASELINE config 0 (1D {1024}, D 64, M 16, batch 1) or config 1 forward
    (2D 32x32, D 64, M 16, batch 8, RoPE)."""
    import torch
    if which == "scan_fwd_c0":
        dims, D_, M_, B_, rope, name = (1024,), 64, 16, 1, False, "scannd_fwd_1d1024_D64_M16_b1 (config 0)"
    else:
        dims, D_, M_, B_, rope, name = (32, 32), 64, 16, 8, True, "scannd_fwd_2d32x32_D64_M16_b8_rope (config 1)"
    P_, nd = int(np.prod(dims)), len(dims)
    t = _scan_inputs(g, dev, dims, D_, M_, B_, rope)
    h, y = torch.empty(B_, P_, D_, M_, device=dev), torch.empty(B_, P_, D_, device=dev)
    p = kmb.scan_params(list(dims), D_, M_, t["x"], t["A"], t["B"], t["C"], t["delta"], h, y, theta=t["theta"])
    sp = C.c_void_p(stream.cuda_stream)
    steps = max(args.steps, 20)
    ms = _timed(lambda: kmb.check(lib.scannd_forward_async(C.byref(p), B_, sp)), steps, max(args.warmup, 3), stream)
    upd = B_ * P_ * D_ * M_
    alg = upd * 12 + B_ * P_ * D_ * (4 + 4 * nd + 4)
    tt = ms / steps / 1e3
    line = {"metric": "scanND state-updates/sec", "value": upd * world / tt, "unit": "state-updates/s",
            "ms_per_step": ms / steps, "steps": steps, "config": {"workload": name, "l2": "inputs < L2: L2-resident"},
            "roofline": {"bound": "hbm", "achieved": round(alg / tt / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / tt / 1e9 / peak, 4), "peak_source": peak_src, "traffic": None,
                         "alg_bytes_per_launch": alg,
                         "kernel": "scan_fwd_tma" if nd == 1 else "scan_fwd_strips",
                         "note": "inputs fit in L2 and one launch is a few microseconds: launch-latency bound"},
            "gpu_launches": steps}
    hin = {k: _pinned(v) for k, v in t.items() if v is not None and k != "A" and k != "theta"}
    line["e2e"] = _e2e(stream, hin, {k: t[k] for k in hin}, {"h": h, "y": y},
                       {"h": torch.empty(h.shape, pin_memory=True), "y": torch.empty(y.shape, pin_memory=True)},
                       lambda: kmb.check(lib.scannd_forward_async(C.byref(p), B_, sp)), 20, upd * world,
                       "state-updates/s")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import pyoracle as po
        threads = po.set_threads(len(os.sched_getaffinity(0)) or 1)
        inp = po.gen_scan(list(dims), D_, M_, batch=B_, seed=3, rope=rope)
        rate, n = _cpu_rate(lambda: po.ref_scannd(inp), upd)
        line["cpu_baseline"] = {"value": rate, "unit": "state-updates/s", "cores": threads, "kind": "reference",
                                "sample": f"scannd_ref (oracle/_ref) on the whole workload ({B_} items), median of {n}"}
    return line


def wl_scan_fwd_3d(args, dev, stream, lib, kmb, g, which, peak, peak_src, rank, world):
    """Scan-A forward on the 3D grid {16,32,32} (the model config's spatial
    grid) at the headline's channel and state counts: D 512, M 64, RoPE,
    batch 2 (13 GB of B, C and h: inputs > L2)."""
    import torch
    dims, D_, M_, B_ = (16, 32, 32), 512, 64, 2
    P_, nd = int(np.prod(dims)), len(dims)
    t = _scan_inputs(g, dev, dims, D_, M_, B_, True)
    h, y = torch.empty(B_, P_, D_, M_, device=dev), torch.empty(B_, P_, D_, device=dev)
    p = kmb.scan_params(list(dims), D_, M_, t["x"], t["A"], t["B"], t["C"], t["delta"], h, y, theta=t["theta"])
    sp = C.c_void_p(stream.cuda_stream)
    call = lambda: kmb.check(lib.scannd_forward_async(C.byref(p), B_, sp))
    steps = max(args.steps, 5)
    ms = _timed(call, steps, max(args.warmup, 3), stream)
    path = lib.kmb_last_forward_path()
    upd = B_ * P_ * D_ * M_
    # B, C read + h written per update, plus the plane predecessor's h and B read back (L2 or HBM)
    alg = upd * 12 + B_ * P_ * D_ * (4 + 4 * nd + 4)
    tt = ms / steps / 1e3
    line = {"metric": "scanND state-updates/sec", "value": upd * world / tt, "unit": "state-updates/s",
            "ms_per_step": ms / steps, "steps": steps,
            "config": {"workload": "scannd_fwd_3d16x32x32_D512_M64_b2_rope", "l2": "inputs > L2 (13 GB)"},
            "roofline": {"bound": "hbm", "achieved": round(alg / tt / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / tt / 1e9 / peak, 4), "peak_source": peak_src, "traffic": None,
                         "alg_bytes_per_launch": alg, "kernel": "scan_fwd_strips (3D: plane predecessor by TMA)",
                         "note": "algorithmic bytes count B, C, h once; the plane predecessor's h and B are "
                                 "re-read (8 B per update more when they miss L2)"},
            "fast_path": path, "gpu_launches": steps}
    hin = {k: _pinned(v) for k, v in t.items() if v is not None and k != "A" and k != "theta"}
    line["e2e"] = _e2e(stream, hin, {k: t[k] for k in hin}, {"h": h, "y": y},
                       {"h": torch.empty(h.shape, pin_memory=True), "y": torch.empty(y.shape, pin_memory=True)},
                       call, 3, upd * world, "state-updates/s")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import pyoracle as po
        threads = po.set_threads(len(os.sched_getaffinity(0)) or 1)
        inp = po.gen_scan(list(dims), 16, M_, batch=1, seed=3, rope=True)
        units = P_ * 16 * M_
        rate, n = _cpu_rate(lambda: po.ref_scannd(inp), units)
        line["cpu_baseline"] = {"value": rate, "unit": "state-updates/s", "cores": threads, "kind": "reference",
                                "sample": f"scannd_ref (oracle/_ref): one item, 16 of the 512 channels, median of {n}"}
    return line


def wl_scan_bwd(args, dev, stream, lib, kmb, g, which, peak, peak_src, rank, world):
    """Scan-A backward: the headline geometry (2D 64x64, D 512, M 64, batch 32)
    or BASELINE config 1 (2D 32x32, D 64, M 16, batch 8, RoPE)."""
    import torch
    if which == "scan_bwd":
        B_ = args.batch   # 32 unless --batch overrides it (profiling)
        dims, D_, M_, rope = (64, 64), 512, 64, False
        name = f"scannd_bwd_2d64x64_D512_M64_b{B_} (headline geometry)"
    elif which == "scan_bwd_3d":
        dims, D_, M_, B_, rope, name = (16, 32, 32), 512, 64, 2, True, "scannd_bwd_3d16x32x32_D512_M64_b2_rope"
    else:
        dims, D_, M_, B_, rope, name = (32, 32), 64, 16, 8, True, "scannd_bwd_2d32x32_D64_M16_b8_rope (config 1)"
    P_, nd = int(np.prod(dims)), len(dims)
    t = _scan_inputs(g, dev, dims, D_, M_, B_, rope)
    h, y = torch.empty(B_, P_, D_, M_, device=dev), torch.empty(B_, P_, D_, device=dev)
    p = kmb.scan_params(list(dims), D_, M_, t["x"], t["A"], t["B"], t["C"], t["delta"], h, y, theta=t["theta"])
    sp = C.c_void_p(stream.cuda_stream)
    kmb.check(lib.scannd_forward_async(C.byref(p), B_, sp))
    torch.cuda.synchronize()
    del y
    dy = torch.randn((B_, P_, D_), generator=g, device=dev)
    gr = {"dA": torch.zeros(nd, D_, M_, device=dev), "dB": torch.zeros(B_, P_, D_, M_, device=dev),
          "dC": torch.zeros(B_, P_, D_, M_, device=dev), "ddelta": torch.zeros(B_, nd, P_, D_, device=dev),
          "dlambda": torch.zeros(B_, P_, device=dev), "dtheta": torch.zeros(max(D_ // 2, 1), device=dev)}
    dx = torch.zeros(B_, P_, D_, device=dev)
    pb = kmb.scan_params(list(dims), D_, M_, t["x"], t["A"], t["B"], t["C"], t["delta"], h, dy, theta=t["theta"],
                         grads=gr)
    steps = max(args.steps // 6, 5) if which != "scan_bwd_c1" else max(args.steps, 20)
    call = lambda: kmb.check(lib.scannd_backward_async(C.byref(pb), B_, dx.data_ptr(), sp))
    ms = _timed(call, steps, max(args.warmup, 3), stream)
    path = lib.kmb_last_backward_path()
    upd = B_ * P_ * D_ * M_
    # accumulate (+=) semantics: read h, B, C, dB, dC; write dB, dC = 28 B per update; per (point, channel):
    # read x, dy, delta[nd]; read + write ddelta[nd] and dx
    alg = upd * 28 + B_ * P_ * D_ * (4 * (2 + nd) + 8 * (nd + 1)) + B_ * P_ * 8
    tt = ms / steps / 1e3
    line = {"metric": "scanND backward state-updates/sec", "value": upd * world / tt, "unit": "state-updates/s",
            "ms_per_step": ms / steps, "steps": steps,
            "config": {"workload": name, "semantics": "accumulate (+=) into every gradient, as the reference",
                       "l2": "inputs ~ L2 size" if which == "scan_bwd_c1" else "inputs >> L2"},
            "roofline": {"bound": "hbm", "achieved": round(alg / tt / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / tt / 1e9 / peak, 4), "peak_source": peak_src, "traffic": None,
                         "alg_bytes_per_launch": alg,
                         "kernel": {2: "scan_bwd_strips", 1: "scan_bwd_wave", 0: "scan_bwd_generic"}.get(path)},
            "gpu_launches": steps * {2: 5 if M_ == 64 else 4, 1: 2 + 3 * max(M_ // 32, 1)}.get(path, 4)}
    # the same step with overwrite semantics (scannd_backward_ex): no read-back of the gradients
    ovw = lambda: kmb.check(lib.scannd_backward_ex(C.byref(pb), B_, dx.data_ptr(), 1, sp))
    ms_o = _timed(ovw, steps, 2, stream)
    alg_o = upd * 20 + B_ * P_ * D_ * (4 * (2 + nd) + 4 * (nd + 1)) + B_ * P_ * 4
    line["overwrite_variant"] = {"value": upd * world / (ms_o / steps / 1e3), "ms_per_step": ms_o / steps,
                                 "hbm_frac": round(alg_o / (ms_o / steps / 1e3) / 1e9 / peak, 4)}
    eb = B_ if which != "scan_bwd" else min(4, B_)   # host RAM: 4 headline items (5.5 GB in, 4.4 GB out) per e2e step
    hin = {"x": _pinned(t["x"][:eb]), "delta": _pinned(t["delta"][:eb]), "B": _pinned(t["B"][:eb]),
           "C": _pinned(t["C"][:eb]), "h": _pinned(h[:eb]), "dy": _pinned(dy[:eb])}
    din = {k: torch.empty_like(v, device=dev) for k, v in hin.items()}
    gre = {k: (torch.zeros_like(v[:eb]) if v.dim() > 1 and k not in ("dA",) else torch.zeros_like(v)) for k, v in gr.items()}
    dxe = torch.zeros((eb, P_, D_), device=dev)
    pe = kmb.scan_params(list(dims), D_, M_, din["x"], t["A"], din["B"], din["C"], din["delta"], din["h"], din["dy"],
                         theta=t["theta"], grads=gre)
    outs = {"dB": gre["dB"], "dC": gre["dC"], "ddelta": gre["ddelta"], "dx": dxe, "dA": gre["dA"]}
    line["e2e"] = _e2e(stream, hin, din, outs, {k: torch.empty(v.shape, pin_memory=True) for k, v in outs.items()},
                       lambda: kmb.check(lib.scannd_backward_ex(C.byref(pe), eb, dxe.data_ptr(), 1, sp)), 3,
                       eb * P_ * D_ * M_ * world, "state-updates/s")
    line["e2e"]["batch_per_gpu"] = eb
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import pyoracle as po
        d_s = D_ if which == "scan_bwd_c1" else 4
        inp = po.gen_scan(list(dims), d_s, M_, batch=1, seed=3, rope=rope)
        hs, _ = po.oracle_scannd(inp)
        dys = np.random.default_rng(1).standard_normal((1, P_, d_s)).astype(np.float32)
        rate, n = _cpu_rate(lambda: po.oracle_scannd_bwd(inp, hs, dys), P_ * d_s * M_)
        line["cpu_baseline"] = {"value": rate, "unit": "state-updates/s", "cores": 1, "kind": "port",
                                "sample": f"the exact adjoint restated in C (oracle/scannd_oracle.c, double, one "
                                          f"thread) on 1 item x {d_s} channels: the reference has no correct CPU "
                                          f"Scan-A backward; median of {n}"}
    return line


def wl_convnd(args, dev, stream, lib, kmb, g, which, peak, peak_src, rank, world):
    """depthwise convND forward + backward, D 256, K 3, batch 16,
    2D {32,32} or 3D {16,16,16}."""
    import torch
    dims = (32, 32) if which == "convnd2d" else (16, 16, 16)
    D_, K_, B_ = 256, 3, 16
    P_, V_ = int(np.prod(dims)), K_ ** len(dims)
    rn = lambda *s: torch.randn(s, generator=g, device=dev)
    xi, dy = rn(B_, P_, D_), rn(B_, P_, D_)
    ker, bias = rn(V_, D_) / V_ ** 0.5, rn(D_) * 0.02 ** 0.5
    out, din = torch.empty(B_, P_, D_, device=dev), torch.empty(B_, P_, D_, device=dev)
    dk, db = torch.empty(V_, D_, device=dev), torch.empty(D_, device=dev)
    p = kmb.conv_params(list(dims), D_, K_, xi, ker, bias, out, dy, din, dk, db)
    sp = C.c_void_p(stream.cuda_stream)
    steps = max(args.steps, 20)
    call = lambda: kmb.check(lib.convnd_batched_async(C.byref(p), B_, 3, sp))
    ms = _timed(call, steps, max(args.warmup, 3), stream)
    tt = ms / steps / 1e3
    units = B_ * P_ * D_
    alg = units * 20    # forward: read input, write output; backward: read dy, input, write dinput
    line = {"metric": "convND fwd+bwd outputs/sec", "value": units * world / tt, "unit": "outputs/s",
            "ms_per_step": ms / steps, "steps": steps,
            "config": {"workload": f"convnd_{'x'.join(map(str, dims))}_D256_K3_b16 (config 2)",
                       "l2": "16 MB of inputs: L2-resident between steps"},
            "roofline": {"bound": "hbm", "achieved": round(alg / tt / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / tt / 1e9 / peak, 4), "peak_source": peak_src, "traffic": None,
                         "alg_bytes_per_launch": alg},
            "gpu_launches": steps * 3}
    hin = {"input": _pinned(xi), "dy": _pinned(dy)}
    dinp = {"input": xi, "dy": dy}
    outs = {"output": out, "dinput": din, "dkernel": dk, "dbias": db}
    line["e2e"] = _e2e(stream, hin, dinp, outs, {k: torch.empty(v.shape, pin_memory=True) for k, v in outs.items()},
                       call, 20, units * world, "outputs/s")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import pyoracle as po
        threads = po.set_threads(len(os.sched_getaffinity(0)) or 1)
        nb = 16 if len(dims) == 2 else 1
        inp = po.gen_conv(list(dims), D_, K_, batch=nb, seed=3)
        rate, n = _cpu_rate(lambda: po.conv_run(inp, "ref", 3), nb * P_ * D_)
        line["cpu_baseline"] = {"value": rate, "unit": "outputs/s", "cores": threads, "kind": "reference",
                                "sample": f"convnd_forward_wavefront + convnd_backward_wavefront (oracle/_ref) on "
                                          f"{nb} item(s); the reference backward is serial; median of {n}"}
    return line


def _block_weights(lib, kmb, dims, dim, N, R, dev, g):
    """Block parameters from kmamba_init(seed=42)'s stream (bit-identical to the
    reference's), lambda_proj ~ N(0, 0.02) as BASELINE config 3 asks."""
    import torch
    cfg = kmb.model_config(list(dims), 256, dim, N, R, 1)
    W = {}
    for k in kmb.BLOCK_FIELDS:
        n = {"W_in": R * dim, "W_out": dim * R, "A_log": N, "W_B": N * R * dim, "W_C": N * R * dim,
             "delta_proj": dim, "lambda_proj": dim, "b_B": N * R, "b_C": N * R, "theta": max(N // 2, 1)}[k]
        a = np.zeros(n, np.float32)
        kmb.check(0 if lib.kmb_init_tensor(C.byref(cfg), 42, f"layers.0.{k}".encode(), a.ctypes.data, n) == n else -1)
        W[k] = torch.from_numpy(a).to(dev)
    W["lambda_proj"] = torch.randn(dim, generator=g, device=dev) * 0.02
    return W


def wl_block(args, dev, stream, lib, kmb, g, which, peak, peak_src, rank, world):
    """Mamba-3 block forward + backward, dim 512, N 64, R 2,
    2D 64x64, batch 32 (fp32 storage, or bf16 storage with fp32 state)."""
    import torch
    bf16 = which == "block_bf16"
    dims, dim, N_, R_, B_ = (64, 64), 512, 64, 2, 32
    L_ = 4096
    W = _block_weights(lib, kmb, dims, dim, N_, R_, dev, g)
    cfg = kmb.block_config(list(dims), dim, N_, R_, bf16=bf16)
    w = kmb.KMBlockWeights(**{k: W[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    G = {k: torch.zeros_like(v) for k, v in W.items()}
    gw = kmb.KMBlockGrads(**{k: G[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    act_f = lib.kmb_block_activation_floats(C.byref(cfg), B_)
    act = torch.empty(act_f, device=dev)
    rn = lambda *s: torch.randn(s, generator=g, device=dev)
    x, dout = rn(B_, L_, dim), rn(B_, L_, dim)
    if bf16:
        x, dout = x.to(torch.bfloat16), dout.to(torch.bfloat16)
    out, dx = torch.empty_like(x), torch.empty_like(x)
    sp = C.c_void_p(stream.cuda_stream)

    def step():
        kmb.check(lib.kmb_block_forward(C.byref(cfg), C.byref(w), x.data_ptr(), out.data_ptr(), B_, act.data_ptr(), sp))
        kmb.check(lib.kmb_block_backward(C.byref(cfg), C.byref(w), x.data_ptr(), dout.data_ptr(), dx.data_ptr(),
                                         C.byref(gw), B_, act.data_ptr(), sp))
    steps = max(args.steps // 6, 10)
    ms = _timed(step, steps, max(args.warmup, 3), stream)
    tt = ms / steps / 1e3
    esz = 2 if bf16 else 4
    # compulsory traffic of the step: the saved activations written by the forward and read by the backward,
    # x read twice, out, dout, dx once (weights and their gradients are < 1 MB)
    alg = act_f * 4 * 2 + B_ * L_ * dim * esz * 5
    line = {"metric": "Mamba-3 block fwd+bwd tokens/sec", "value": B_ * L_ * world / tt, "unit": "tokens/s",
            "ms_per_step": ms / steps, "steps": steps,
            "dtype": "bf16 storage / f32 state" if bf16 else "f32",
            "config": {"workload": "block_dim512_N64_R2_2d64x64_b32 (config 3, "
                                   + ("bf16 storage, fp32 state)" if bf16 else "fp32 storage)"),
                       "init": "kmamba_init(seed=42) stream (reference-identical), lambda_proj ~ N(0, 0.02)"},
            "scan_updates_per_s": B_ * L_ * N_ * R_ * world / tt,
            "roofline": {"bound": "hbm", "achieved": round(alg / tt / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / tt / 1e9 / peak, 4), "peak_source": peak_src, "traffic": None,
                         "alg_bytes_per_launch": alg,
                         "note": "whole-step compulsory bytes over the step time; per-kernel shares in profiles/"}}
    hin = {"x": _pinned(x), "dout": _pinned(dout)}
    outs = {"out": out, "dx": dx}
    line["e2e"] = _e2e(stream, hin, {"x": x, "dout": dout}, outs,
                       {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in outs.items()}, step, 5,
                       B_ * L_ * world, "tokens/s")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import pyoracle as po
        threads = po.set_threads(len(os.sched_getaffinity(0)) or 1)
        params = {k: v.cpu().numpy() for k, v in W.items()}
        xs = np.random.default_rng(1).standard_normal((L_, dim)).astype(np.float32)
        dys = np.random.default_rng(2).standard_normal((L_, dim)).astype(np.float32)
        rate, n = _cpu_rate(lambda: po.ref_block_run(list(dims), dim, N_, R_, params, xs, dy=dys), L_, max_reps=3)
        line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "reference",
                                "sample": f"mamba_block_forward_ws + mamba_backward_ws (oracle/_ref, fp32) on 1 item "
                                          f"of the 32; median of {n}"}
    return line


def wl_model(args, dev, stream, lib, kmb, g, which, peak, peak_src, rank, world):
    """12-layer k-mamba train step (forward, backward, AdamW),
    dim 512, N 64, R 4, 3D {16,32,32}, batch 64, vocab 256."""
    import torch
    dims, V_, dim, N_, R_, nl, B_ = (16, 32, 32), 256, 512, 64, 4, 12, 64
    B_ = int(os.environ.get("KMB_BENCH_MODEL_BATCH", B_))
    cfgm = kmb.model_config(list(dims), V_, dim, N_, R_, nl)
    m = lib.kmamba_create(C.byref(cfgm))
    if not m:
        raise RuntimeError(kmb.last_error())
    kmb.check(lib.kmamba_init(m, 42))
    opt = kmb.MBOptimConfig()
    lib.kmamba_optim_config_set_defaults(C.byref(opt))
    lib.kmamba_enable_training(m, C.byref(opt), 1e-3, 0.01)
    L_ = 16384
    tok = torch.randint(0, V_, (B_, L_ + 1), generator=g, device=dev, dtype=torch.int32)
    sp = C.c_void_p(stream.cuda_stream)
    losses = []

    def step():
        # NaN is a legitimate value at this scale (the 3D recurrence overflows fp32, as the reference's does)
        loss = lib.kmb_model_forward_backward(m, tok.data_ptr(), B_, sp)
        if loss != loss and kmb.last_error():
            raise RuntimeError(kmb.last_error())
        kmb.check(lib.kmb_model_optimizer_step(m, sp))
        losses.append(loss if loss == loss else None)
    steps = 3
    ms = _timed(step, steps, 2, stream)
    tt = ms / steps / 1e3
    line = {"metric": "k-mamba train step tokens/sec", "value": B_ * L_ * world / tt, "unit": "tokens/s",
            "ms_per_step": ms / steps, "steps": steps, "warmup": 2,
            "config": {"workload": f"model_12x512_N64_R4_3d16x32x32_b{B_}_vocab256 (config 4)",
                       "init": "kmamba_init(seed=42), reference-identical"},
            "loss_first_last": [losses[0], losses[-1]],
            "roofline": None}
    # e2e: kmamba_train_batch with host tokens (copy in, forward, backward, AdamW, loss out)
    htok = tok.cpu().numpy().astype(np.uint32)
    eb = B_
    lib.kmamba_train_batch(m, htok.ctypes.data, eb)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(2):
        lib.kmamba_train_batch(m, htok.ctypes.data, eb)
    dt = time.perf_counter() - t0
    line["e2e"] = {"value": eb * L_ * world * 2 / dt, "unit": "tokens/s", "h2d_bytes_per_step": htok.nbytes,
                   "d2h_bytes_per_step": 4, "steps": 2, "path": "kmamba_train_batch() with host tokens"}
    lib.kmamba_free(m)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import pyoracle as po
        threads = po.set_threads(len(os.sched_getaffinity(0)) or 1)
        W = _block_weights(lib, kmb, dims, dim, N_, R_, dev, g)
        params = {k: v.cpu().numpy() for k, v in W.items()}
        xs = np.random.default_rng(1).standard_normal((L_, dim)).astype(np.float32) * 0.1
        dys = np.random.default_rng(2).standard_normal((L_, dim)).astype(np.float32)
        rate, n = _cpu_rate(lambda: po.ref_block_run(list(dims), dim, N_, R_, params, xs, dy=dys), L_, max_reps=2)
        # one block of the 12, one sequence: tokens/s of the whole model is the block rate / 12 (the head,
        # embedding and AdamW are a few percent of a layer and are not counted: an upper bound)
        line["cpu_baseline"] = {"value": rate / nl, "unit": "tokens/s", "cores": threads, "kind": "reference",
                                "sample": f"one reference block (mamba_block_forward_ws + mamba_backward_ws, "
                                          f"oracle/_ref) on 1 sequence of 16384 tokens, rate / 12 layers; "
                                          f"median of {n}"}
    return line


def other_configs(args):
    """The other BASELINE configs (every workload of --workload all), measured in
    a child process after the headline and summarised into the headline line:
    value, ms per step, roofline fraction, e2e and CPU-baseline rates."""
    cmd = [sys.executable, os.path.abspath(__file__), "--workload", "all", "--steps", "10", "--warmup", "3"]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    except Exception as exc:
        return {"error": str(exc)[:200]}
    out = {}
    for ln in r.stdout.splitlines():
        if not ln.startswith("{"):
            continue
        try:
            d = json.loads(ln)
        except ValueError:
            continue
        rf, e2, cb = d.get("roofline") or {}, d.get("e2e") or {}, d.get("cpu_baseline") or {}
        out[d["config"]["workload"]] = {
            "metric": d.get("metric"), "value": d.get("value"), "unit": d.get("unit"),
            "ms_per_step": d.get("ms_per_step"), "dtype": d.get("dtype"), "steps": d.get("steps"),
            "roofline_frac": rf.get("frac"), "roofline_bound": rf.get("bound"), "e2e": e2.get("value"),
            "cpu_baseline": cb.get("value"), "cpu_baseline_kind": cb.get("kind"), "cpu_cores": cb.get("cores")}
    if r.returncode != 0:
        out["error"] = (r.stderr or "")[-300:]
    return out


def run_other_workload(args, rank, world):
    import torch
    import torch.distributed as dist
    import bissimamba_b200 as kmb

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    lib = kmb.lib()
    stream = torch.cuda.current_stream(dev)
    peak, peak_src = peaks()
    names = OTHER if args.workload == "all" else (args.workload,)
    fns = {"scan_fwd_c0": wl_scan_fwd_small, "scan_fwd_c1": wl_scan_fwd_small, "scan_fwd_3d": wl_scan_fwd_3d,
           "scan_bwd": wl_scan_bwd,
           "scan_bwd_c1": wl_scan_bwd, "scan_bwd_3d": wl_scan_bwd, "convnd2d": wl_convnd, "convnd3d": wl_convnd, "block": wl_block,
           "block_bf16": wl_block, "model": wl_model}
    for name in names:
        g = torch.Generator(device=dev)
        g.manual_seed(7 + rank)
        line = {"n_gpus": world, "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE distributions), on device"}
        line.update(fns[name](args, dev, stream, lib, kmb, g, name, peak, peak_src, rank, world))
        if world > 1:
            t = torch.tensor([line["ms_per_step"]], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            line["ms_per_step"] = float(t.item())
        if rank == 0:
            print(json.dumps(line), flush=True)
        torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
