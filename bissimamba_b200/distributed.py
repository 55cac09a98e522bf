"""Batch / channel sharding across the GPUs of one node (rebuild of the
reference's kmamba_distributed, src/kmamba_distributed.c and
cuda/kmamba_distributed.cu, which were never called and broadcast no NCCL id).

One process per GPU over ``torch.distributed`` (NCCL on GPUs, gloo on CPU for
tests).  The scans and convnd have no cross-rank exchange in the forward: each
rank owns whole batch items (or whole RoPE channel pairs).  The only
collectives are the parameter broadcast at start-up and the all-reduce of the
gradient arena after the backward.  Each rank scales its gradients by its share
of the batch before the sum, so the update equals the full-batch update even
when the batch does not divide evenly.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist


def split_batch(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of this rank's batch items; earlier ranks take the extra
    items (reference src/kmamba_distributed.c:120-139)."""
    if world <= 0:
        raise ValueError("world must be > 0")
    per, rem = divmod(batch, world)
    if rank < rem:
        start = rank * (per + 1)
        return start, start + per + 1
    start = rank * per + rem
    return start, start + per


def split_layers(n_layers: int, world: int, rank: int) -> tuple[int, int]:
    """Same rule over layers (reference src/kmamba_distributed.c:141-160)."""
    return split_batch(n_layers, world, rank)


def split_channel_pairs(D: int, world: int, rank: int) -> tuple[int, int]:
    """Channel range for channel sharding: whole RoPE pairs (2i, 2i+1) stay on
    one rank, so ranges start on even channels."""
    pairs = (D + 1) // 2
    a, b = split_batch(pairs, world, rank)
    return min(D, 2 * a), min(D, 2 * b)


def scale_and_allreduce_(t: torch.Tensor, weight: float, group=None) -> torch.Tensor:
    """t <- sum over ranks of weight_r * t_r (in place)."""
    t.mul_(weight)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class DataParallel:
    """Data-parallel driver for anything that exposes a parameter buffer, a
    gradient buffer and a local forward+backward:

    * ``params`` / ``grads``: 1-D float32 tensors (views of the model arenas);
    * ``forward_backward(local_batch) -> local mean loss``;
    * ``step()``: the optimizer update on the reduced gradients.
    """

    def __init__(self, params: torch.Tensor, grads: torch.Tensor, forward_backward, step, group=None):
        self.params, self.grads = params, grads
        self.forward_backward, self.step = forward_backward, step
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def broadcast_params(self, src: int = 0):
        if self.world > 1:
            dist.broadcast(self.params, src=src, group=self.group)

    def train_step(self, global_batch, global_size: int) -> float:
        """global_batch: indexable by item; every rank passes the same global
        batch and processes its own slice.  Returns the global mean loss."""
        a, b = split_batch(global_size, self.world, self.rank)
        share = (b - a) / global_size
        loss = self.forward_backward(global_batch[a:b]) if b > a else 0.0
        scale_and_allreduce_(self.grads, share, self.group)
        lt = torch.tensor([loss * share], dtype=torch.float64, device=self.grads.device)
        if self.world > 1:
            dist.all_reduce(lt, op=dist.ReduceOp.SUM, group=self.group)
        self.step()
        return float(lt.item())


def model_data_parallel(kmb, model, device, group=None) -> DataParallel:
    """DataParallel over a library KMamba handle (GPU)."""
    n = C.c_size_t()
    gptr = kmb.lib().kmb_model_grad_arena(model, C.byref(n))
    pptr = kmb.lib().kmb_model_param_arena(model, C.byref(n))
    grads = torch.as_tensor(kmb.DeviceArray(gptr, n.value), device=device)
    params = torch.as_tensor(kmb.DeviceArray(pptr, n.value), device=device)
    stream = torch.cuda.current_stream(device)

    def fb(tokens):
        t = tokens.to(device=device, dtype=torch.int32).contiguous()
        loss = kmb.lib().kmb_model_forward_backward(model, t.data_ptr(), t.shape[0], C.c_void_p(stream.cuda_stream))
        if loss != loss:
            raise RuntimeError(kmb.last_error())
        return loss

    def step():
        kmb.check(kmb.lib().kmb_model_optimizer_step(model, C.c_void_p(stream.cuda_stream)), "optimizer step")

    return DataParallel(params, grads, fb, step, group)
