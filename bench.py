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
PROFILE_MD = os.path.join(ROOT, "profiles", "scan_fwd_strips_headline.md")


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
                    choices=["scan_fwd", "scan_bwd", "convnd", "block", "model"],
                    help="scan_fwd = the headline line; the others measure the other BASELINE configs")
    ap.add_argument("--bf16", action="store_true", help="block workload: bf16 storage, fp32 state (config 3)")
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


def profiled_traffic_per_update():
    """dram bytes per state update of the top kernel from the committed ncu summary."""
    try:
        for line in open(PROFILE_MD):
            if line.strip().startswith("dram_bytes_per_update:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


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

    def step():
        rc = lib.scannd_forward_async(C.byref(p), BATCH, sp)
        if rc != 0:
            raise RuntimeError(kmb.last_error())

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
    tpu = profiled_traffic_per_update()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_src,
                "traffic": (tpu * UPDATES if tpu else None),
                "alg_bytes_per_launch": ALG_BYTES, "kernel": ("scan_fwd_strips" if len(DIMS) == 2 else "scan_fwd_tma") if path == 1 else "scan_fwd_generic"}

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

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu, _ = cpu_reference_rate()
        except Exception as exc:  # the reference build is test infrastructure: report, do not fail
            cpu = {"value": None, "error": str(exc)[:200]}

    if rank == 0:
        line = {"metric": "scanND state-updates/sec", "value": value, "unit": "state-updates/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, BASELINE config-0 distributions), generated on device",
                "config": {"workload": WORKLOAD, "dims": list(DIMS), "D": D, "M": M, "batch_per_gpu": BATCH,
                           "global_batch": BATCH * world, "rope": False, "lambda": "default 0.5",
                           "parallelism": f"dp{world} (batch shards, no collective)",
                           "l2": f"inputs {ALG_BYTES / 1e9:.1f} GB/GPU >> 126 MB L2, no flush"},
                "hbm_gbs": round(achieved, 1),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": args.steps, "clocks": clk,
                "kernel_ms": {"mean": statistics.mean(kern_ms), "min": min(kern_ms), "max": max(kern_ms)}}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------- other configs
def _timed(step, steps, warmup, stream):
    """CUDA-event time (ms) of `steps` calls after `warmup` calls."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def run_other_workload(args, rank, world):
    """BASELINE configs 1-4 on one GPU (per rank; weak scaling like the headline)."""
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
    sp = C.c_void_p(stream.cuda_stream)
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    rn = lambda *s: torch.randn(s, generator=g, device=dev)
    steps, warm = max(args.steps // 6, 5), max(args.warmup, 3)
    peak, peak_src = peaks()
    line = {"n_gpus": world, "steps": steps, "warmup": warm, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE distributions), on device"}

    if args.workload == "scan_bwd":
        # BASELINE config 1 backward: 2D 32x32, D 64, M 16, batch 8, RoPE, dy ~ N(0,1)
        dims, D_, M_, B_ = (32, 32), 64, 16, 8
        P_ = 1024
        x, dl = rn(B_, P_, D_), torch.nn.functional.softplus(rn(B_, 2, P_, D_) * 0.5 - 4.0)
        A = -torch.exp(torch.rand((2, D_, M_), generator=g, device=dev) * torch.log(torch.tensor(16.0)))
        Bm = (rn(B_, P_, 1, M_) * 0.25).expand(B_, P_, D_, M_).contiguous()
        Cm = (rn(B_, P_, 1, M_) * 0.25).expand(B_, P_, D_, M_).contiguous()
        th = torch.rand(D_ // 2, generator=g, device=dev) * 6.283 - 3.1416
        h, y = torch.empty(B_, P_, D_, M_, device=dev), torch.empty(B_, P_, D_, device=dev)
        p = kmb.scan_params(list(dims), D_, M_, x, A, Bm, Cm, dl, h, y, theta=th)
        kmb.check(lib.scannd_forward_async(C.byref(p), B_, sp))
        dy = rn(B_, P_, D_)
        gr = {k: torch.zeros(s, device=dev) for k, s in (("dA", (2, D_, M_)), ("dB", (B_, P_, D_, M_)),
                                                           ("dC", (B_, P_, D_, M_)), ("ddelta", (B_, 2, P_, D_)),
                                                           ("dlambda", (B_, P_)), ("dtheta", (D_ // 2,)))}
        dx = torch.zeros(B_, P_, D_, device=dev)
        pb = kmb.scan_params(list(dims), D_, M_, x, A, Bm, Cm, dl, h, dy, theta=th, grads=gr)
        ms = _timed(lambda: kmb.check(lib.scannd_backward_async(C.byref(pb), B_, dx.data_ptr(), sp)), steps, warm,
                    stream)
        upd = B_ * P_ * D_ * M_
        alg = upd * 20 + B_ * P_ * D_ * 4 * 7
        t = ms / steps / 1e3
        line.update(metric="scanND backward state-updates/sec", value=upd * world / t, unit="state-updates/s",
                    ms_per_step=ms / steps, config={"workload": "scannd_bwd_2d32x32_D64_M16_b8_rope (config 1)"},
                    roofline={"bound": "hbm", "achieved": round(alg / t / 1e9, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(alg / t / 1e9 / peak, 4), "peak_source": peak_src},
                    gpu_launches=steps * 4)
    elif args.workload == "convnd":
        # dims {32,32} and {16,16,16}, D 256, K 3, batch 16, forward + backward
        res = {}
        for dims in ((32, 32), (16, 16, 16)):
            D_, K_, B_ = 256, 3, 16
            P_ = int(np.prod(dims)) if False else (dims[0] * dims[1] * (dims[2] if len(dims) > 2 else 1))
            V_ = K_ ** len(dims)
            xi, dy = rn(B_, P_, D_), rn(B_, P_, D_)
            ker, bias = rn(V_, D_) / V_ ** 0.5, rn(D_) * 0.14
            out, din = torch.empty(B_, P_, D_, device=dev), torch.empty(B_, P_, D_, device=dev)
            dk, db = torch.empty(V_, D_, device=dev), torch.empty(D_, device=dev)
            p = kmb.conv_params(list(dims), D_, K_, xi, ker, bias, out, dy, din, dk, db)
            ms = _timed(lambda: kmb.check(lib.convnd_batched_async(C.byref(p), B_, 3, sp)), steps, warm, stream)
            t = ms / steps / 1e3
            alg = B_ * P_ * D_ * 20
            res["x".join(map(str, dims))] = {"outputs_per_s": B_ * P_ * D_ * world / t, "ms_per_step": ms / steps,
                                             "hbm_gbs": round(alg / t / 1e9, 1),
                                             "frac": round(alg / t / 1e9 / peak, 4)}
        line.update(metric="convND fwd+bwd outputs/sec (config 2, 2D and 3D)",
                    value=res["32x32"]["outputs_per_s"], unit="outputs/s", ms_per_step=res["32x32"]["ms_per_step"],
                    config={"workload": "convnd_D256_K3_b16 (config 2)", "per_shape": res}, gpu_launches=None)
    elif args.workload == "block":
        # Mamba-3 block, dim 512, N 64, R 2, 2D 64x64, batch 32, forward + backward (fp32)
        dims, dim, N_, R_, B_ = (64, 64), 512, 64, 2, 32
        L_ = 4096
        from oracle import pyoracle as po  # parameter init only (seeded numpy), not a compute path
        params = po.gen_block_params(dim, N_, R_, seed=42)
        W = {k: torch.from_numpy(v).to(dev) for k, v in params.items()}
        cfg = kmb.block_config(list(dims), dim, N_, R_, bf16=args.bf16)
        w = kmb.KMBlockWeights(**{k: W[k].data_ptr() for k in kmb.BLOCK_FIELDS})
        G = {k: torch.zeros_like(v) for k, v in W.items()}
        gw = kmb.KMBlockGrads(**{k: G[k].data_ptr() for k in kmb.BLOCK_FIELDS})
        act = torch.empty(lib.kmb_block_activation_floats(C.byref(cfg), B_), device=dev)
        x, dout = rn(B_, L_, dim), rn(B_, L_, dim)
        if args.bf16:
            x, dout = x.to(torch.bfloat16), dout.to(torch.bfloat16)
        out, dx = torch.empty_like(x), torch.empty_like(x)

        def step():
            kmb.check(lib.kmb_block_forward(C.byref(cfg), C.byref(w), x.data_ptr(), out.data_ptr(), B_,
                                            act.data_ptr(), sp))
            kmb.check(lib.kmb_block_backward(C.byref(cfg), C.byref(w), x.data_ptr(), dout.data_ptr(), dx.data_ptr(),
                                             C.byref(gw), B_, act.data_ptr(), sp))
        ms = _timed(step, steps, warm, stream)
        t = ms / steps / 1e3
        line.update(metric="Mamba-3 block fwd+bwd tokens/sec (config 3)", value=B_ * L_ * world / t,
                    unit="tokens/s", ms_per_step=ms / steps,
                    config={"workload": "block_dim512_N64_R2_2d64x64_b32 (config 3, "
                                        + ("bf16 storage, fp32 state)" if args.bf16 else "fp32 storage)")},
                    dtype="bf16 storage / f32 state" if args.bf16 else "f32",
                    scan_updates_per_s=B_ * L_ * N_ * R_ * world / t)
    else:
        # 12-layer model, dim 512, N 64, R 4, 3D {16,32,32}, batch 64, vocab 256, AdamW
        dims, V_, dim, N_, R_, nl, B_ = (16, 32, 32), 256, 512, 64, 4, 12, 64
        B_ = int(os.environ.get("KMB_BENCH_MODEL_BATCH", B_))
        cfgm = kmb.model_config(list(dims), V_, dim, N_, R_, nl)
        m = lib.kmamba_create(C.byref(cfgm))
        if not m:
            raise RuntimeError(kmb.last_error())
        lib.kmamba_init(m, 42)
        opt = kmb.MBOptimConfig()
        lib.kmamba_optim_config_set_defaults(C.byref(opt))
        lib.kmamba_enable_training(m, C.byref(opt), 1e-3, 0.01)
        L_ = 16384
        tok = torch.randint(0, V_, (B_, L_ + 1), generator=g, device=dev, dtype=torch.int32)
        losses = []

        def step():
            # NaN is a legitimate value here (the recurrence overflows fp32 at this scale, as the
            # reference's does); an error leaves a message in kmb_last_error()
            loss = lib.kmb_model_forward_backward(m, tok.data_ptr(), B_, sp)
            if loss != loss and kmb.last_error():
                raise RuntimeError(kmb.last_error())
            kmb.check(lib.kmb_model_optimizer_step(m, sp))
            losses.append(loss if loss == loss else None)
        steps = max(2, min(steps, 3))
        ms = _timed(step, steps, 2, stream)
        t = ms / steps / 1e3
        line.update(metric="k-mamba train step tokens/sec (config 4)", value=B_ * L_ * world / t, unit="tokens/s",
                    ms_per_step=ms / steps, steps=steps, warmup=2,
                    config={"workload": f"model_12x512_N64_R4_3d16x32x32_b{B_}_vocab256 (config 4)"},
                    loss_first_last=[losses[0], losses[-1]])
        lib.kmamba_free(m)
    if world > 1:
        t = torch.tensor([line["ms_per_step"]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        line["ms_per_step"] = float(t.item())
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
