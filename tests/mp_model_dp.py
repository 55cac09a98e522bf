"""Multi-rank driver for tests/test_gpu_multi.py (one process per GPU, NCCL
through the library's own communicator, include/kmamba_distributed.h):

* the data-parallel k-mamba step (kmb_dist_model_train_step) on an uneven
  global batch equals the single-GPU full-batch step;
* the batch-sharded Scan-A backward (kmb_dist_scannd_backward) gives every
  rank the full-batch dA / dtheta, and the convnd backward the full-batch
  dkernel / dbias;
* the output gather (kmb_dist_allgather_async) assembles every rank's y."""
import ctypes as C
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bissimamba_b200 as kmb  # noqa: E402
from bissimamba_b200.distributed import Context, split_batch  # noqa: E402


def make(dims, V, dim, N, R, nl, seed):
    cfg = kmb.model_config(dims, V, dim, N, R, nl)
    m = kmb.lib().kmamba_create(C.byref(cfg))
    kmb.lib().kmamba_init(m, seed)
    opt = kmb.MBOptimConfig()
    kmb.lib().kmamba_optim_config_set_defaults(C.byref(opt))
    kmb.lib().kmamba_enable_training(m, C.byref(opt), 1e-3, 0.01)
    return m


def arena(m, which, dev):
    n = C.c_size_t()
    fn = kmb.lib().kmb_model_param_arena if which == "p" else kmb.lib().kmb_model_grad_arena
    return torch.as_tensor(kmb.DeviceArray(fn(m, C.byref(n)), n.value), device=dev)


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = Context(world, rank)            # kmamba_distributed_init_nccl: TCP id exchange + ncclCommInitRank
    ok = True
    # ---- model data parallel
    dims, V, dim, N, R, nl = [4, 8], 16, 32, 16, 2, 2
    m = make(dims, V, dim, N, R, nl, seed=42 if rank == 0 else 7)   # other ranks start wrong
    pa = arena(m, "p", dev)
    ctx.broadcast(pa.data_ptr(), pa.numel(), 0)
    torch.cuda.synchronize()
    gb = 5  # does not divide evenly over 2 ranks
    tok = np.random.default_rng(0).integers(0, V, (gb, 33)).astype(np.int32)
    a, b = split_batch(gb, world, rank)
    dtok = torch.from_numpy(np.ascontiguousarray(tok[a:b])).to(dev)
    torch.cuda.synchronize()
    losses = [ctx.model_train_step(m, dtok.data_ptr(), b - a, gb) for _ in range(2)]
    params = arena(m, "p", dev).clone()
    ref = make(dims, V, dim, N, R, nl, seed=42)
    ref_losses = [kmb.lib().kmamba_train_batch(ref, np.ascontiguousarray(tok.astype(np.uint32)).ctypes.data, gb)
                  for _ in range(2)]
    err = (arena(ref, "p", dev) - params).abs().max().item()
    ok &= err < 2e-5 and all(abs(x - y) < 1e-5 * abs(y) + 1e-6 for x, y in zip(losses, ref_losses))
    print(f"[{rank}] dp losses {losses} single {ref_losses} max param diff {err:.3g}", flush=True)
    # ---- Scan-A backward, batch-sharded (2D, RoPE, 5 items over the ranks)
    g = torch.Generator(device=dev).manual_seed(3)
    B_, H, W, D, M = 5, 8, 12, 8, 16
    P = H * W
    full = dict(x=torch.randn(B_, P, D, generator=g, device=dev),
                delta=torch.nn.functional.softplus(torch.randn(B_, 2, P, D, generator=g, device=dev) * 0.5 - 4),
                A=-torch.exp(torch.rand(2, D, M, generator=g, device=dev) * 2.7),
                B=torch.randn(B_, P, D, M, generator=g, device=dev) * 0.25,
                C=torch.randn(B_, P, D, M, generator=g, device=dev) * 0.25,
                theta=torch.rand(D // 2, generator=g, device=dev) * 6.28 - 3.14,
                dy=torch.randn(B_, P, D, generator=g, device=dev))
    h = torch.empty(B_, P, D, M, device=dev)
    y = torch.empty(B_, P, D, device=dev)
    pf = kmb.scan_params([H, W], D, M, full["x"], full["A"], full["B"], full["C"], full["delta"], h, y,
                         theta=full["theta"])
    kmb.check(kmb.lib().scannd_forward_async(C.byref(pf), B_, None))
    torch.cuda.synchronize()

    def grads(nb):
        return {"dA": torch.zeros(2, D, M, device=dev), "dB": torch.zeros(nb, P, D, M, device=dev),
                "dC": torch.zeros(nb, P, D, M, device=dev), "ddelta": torch.zeros(nb, 2, P, D, device=dev),
                "dlambda": torch.zeros(nb, P, device=dev), "dtheta": torch.zeros(D // 2, device=dev)}
    gref = grads(B_)
    pr = kmb.scan_params([H, W], D, M, full["x"], full["A"], full["B"], full["C"], full["delta"], h, full["dy"],
                         theta=full["theta"], grads=gref)
    kmb.check(kmb.lib().scannd_backward_batched(C.byref(pr), B_, None))
    a, b = split_batch(B_, world, rank)
    gl = grads(b - a)
    sl = lambda t: t[a:b].contiguous()
    pl = kmb.scan_params([H, W], D, M, sl(full["x"]), full["A"], sl(full["B"]), sl(full["C"]), sl(full["delta"]),
                         sl(h), sl(full["dy"]), theta=full["theta"], grads=gl)
    torch.cuda.synchronize()   # the context's stream does not order after torch's
    ctx.scannd_backward(pl, b - a, None, 0)
    torch.cuda.synchronize()
    for k in ("dA", "dtheta"):
        e = ((gl[k] - gref[k]).abs().max() / gref[k].abs().max()).item()
        ok &= e < 1e-5
        print(f"[{rank}] scan {k} rel diff {e:.3g}", flush=True)
    ok &= torch.equal(gl["dB"], gref["dB"][a:b])
    # ---- output gather: every rank's y, in rank order (shards padded to the largest, as NCCL needs
    # one count on every rank)
    per = (B_ + world - 1) // world
    cnt = per * P * D
    ysend = torch.zeros(per, P, D, device=dev)
    ysend[:b - a] = y[a:b]
    yall = torch.empty(world, per, P, D, device=dev)
    torch.cuda.synchronize()
    ctx.allgather(ysend.data_ptr(), yall.data_ptr(), cnt)
    torch.cuda.synchronize()
    for r in range(world):
        ra, rb = split_batch(B_, world, r)
        ok &= torch.equal(yall[r, :rb - ra], y[ra:rb])
    # ---- convnd backward, batch-sharded
    cdims, CD, K = [6, 7], 16, 3
    xi = torch.randn(B_, 42, CD, generator=g, device=dev)
    cdy = torch.randn(B_, 42, CD, generator=g, device=dev)
    ker = torch.randn(9, CD, generator=g, device=dev)
    dk_ref, db_ref = torch.empty(9, CD, device=dev), torch.empty(CD, device=dev)
    din_ref = torch.empty(B_, 42, CD, device=dev)
    cp = kmb.conv_params(cdims, CD, K, xi, ker, None, None, cdy, din_ref, dk_ref, db_ref)
    kmb.check(kmb.lib().convnd_batched_async(C.byref(cp), B_, 2, None))
    dk, db, din = torch.empty(9, CD, device=dev), torch.empty(CD, device=dev), torch.empty(b - a, 42, CD, device=dev)
    cl = kmb.conv_params(cdims, CD, K, sl(xi), ker, None, None, sl(cdy), din, dk, db)
    torch.cuda.synchronize()
    ctx.convnd_backward(cl, b - a)
    torch.cuda.synchronize()
    e = ((dk - dk_ref).abs().max() / dk_ref.abs().max()).item()
    ok &= e < 1e-5 and torch.equal(din, din_ref[a:b])
    print(f"[{rank}] convnd dkernel rel diff {e:.3g}", flush=True)
    # all ranks agree
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    ctx.allreduce(flag.data_ptr(), 1)
    torch.cuda.synchronize()
    ctx.close()
    sys.exit(0 if flag.item() == world else 1)


if __name__ == "__main__":
    main()
