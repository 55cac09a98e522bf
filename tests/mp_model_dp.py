"""Multi-rank driver for tests/test_gpu_multi.py (run under torchrun, one
process per GPU, NCCL): the data-parallel k-mamba step on a global batch must
equal the single-GPU full-batch step computed on rank 0."""
import ctypes as C
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bissimamba_b200 as kmb  # noqa: E402
from bissimamba_b200.distributed import model_data_parallel  # noqa: E402


def make(dims, V, dim, N, R, nl, seed):
    cfg = kmb.model_config(dims, V, dim, N, R, nl)
    m = kmb.lib().kmamba_create(C.byref(cfg))
    kmb.lib().kmamba_init(m, seed)
    opt = kmb.MBOptimConfig()
    kmb.lib().kmamba_optim_config_set_defaults(C.byref(opt))
    kmb.lib().kmamba_enable_training(m, C.byref(opt), 1e-3, 0.01)
    return m


def main():
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    dims, V, dim, N, R, nl = [4, 8], 16, 32, 16, 2, 2
    m = make(dims, V, dim, N, R, nl, seed=42 if rank == 0 else 7)   # other ranks start wrong
    dp = model_data_parallel(kmb, m, dev)
    dp.broadcast_params(0)
    gb = 5  # does not divide evenly over 2 ranks
    tok = torch.from_numpy(np.random.default_rng(0).integers(0, V, (gb, 33)).astype(np.int32))
    losses = [dp.train_step(tok, gb) for _ in range(2)]
    torch.cuda.synchronize()
    params = dp.params.clone()
    ok = True
    if rank == 0:
        ref = make(dims, V, dim, N, R, nl, seed=42)
        ref_losses = [kmb.lib().kmamba_train_batch(ref, np.ascontiguousarray(tok.numpy().astype(np.uint32)).ctypes.data,
                                                   gb) for _ in range(2)]
        n = C.c_size_t()
        rp = torch.as_tensor(kmb.DeviceArray(kmb.lib().kmb_model_param_arena(ref, C.byref(n)), n.value), device=dev)
        err = (rp - params).abs().max().item()
        ok = err < 2e-5 and all(abs(a - b) < 1e-5 * abs(b) + 1e-6 for a, b in zip(losses, ref_losses))
        print(f"dp losses {losses} single {ref_losses} max param diff {err:.3g}", flush=True)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
