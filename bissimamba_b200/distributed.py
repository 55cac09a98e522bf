"""Python view of the library's multi-GPU layer (include/kmamba_distributed.h,
csrc/distributed.cu): one process per GPU over NCCL, rebuilt from the
reference's src/kmamba_distributed.c and cuda/kmamba_distributed.cu.

Everything here calls the C ABI; the collectives, the id exchange and the
batch-split rule are native code.  Batch items are independent through the
scans and convnd, so the forward has no exchange but the optional final output
gather; the backward sums the weight gradients (Scan-A dA / dtheta, convnd
dkernel / dbias, the model's gradient arena) over the ranks."""
from __future__ import annotations

import ctypes as C

from . import lib as _lib


class DistConfig(C.Structure):
    """reference include/kmamba_distributed.h:17-33"""
    _fields_ = [("world_size", C.c_int), ("rank", C.c_int), ("local_rank", C.c_int),
                ("layer_start", C.c_size_t), ("layer_end", C.c_size_t),
                ("batch_start", C.c_size_t), ("batch_end", C.c_size_t),
                ("use_nccl", C.c_int), ("use_p2p", C.c_int)]


def split_batch(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of this rank's items (reference src/kmamba_distributed.c:120-139,
    kmamba_distributed_split_batch): earlier ranks take the extra items."""
    if world <= 0:
        raise ValueError("world must be > 0")
    c = DistConfig(rank=rank)
    _lib().kmamba_distributed_split_batch(C.byref(c), batch, world)
    return c.batch_start, c.batch_end


def split_layers(n_layers: int, world: int, rank: int) -> tuple[int, int]:
    """The same rule over layers (reference src/kmamba_distributed.c:141-160)."""
    if world <= 0:
        raise ValueError("world must be > 0")
    c = DistConfig(rank=rank)
    _lib().kmamba_distributed_split_layers(C.byref(c), n_layers, world)
    return c.layer_start, c.layer_end


def split_channel_pairs(D: int, world: int, rank: int) -> tuple[int, int]:
    """Channel range for channel sharding: whole RoPE pairs (2i, 2i+1) stay on
    one rank, so ranges start on even channels."""
    pairs = (D + 1) // 2
    a, b = split_batch(pairs, world, rank)
    return min(D, 2 * a), min(D, 2 * b)


def exchange_id(id128: bytes | None, world: int, rank: int, addr: str = "127.0.0.1", port: int = 0) -> bytes:
    """kmb_dist_exchange_id: rank 0 sends its 128-byte id to the other ranks over TCP."""
    buf = C.create_string_buffer(id128 if id128 is not None else b"", 128)
    if _lib().kmb_dist_exchange_id(buf, world, rank, addr.encode(), port) != 0:
        raise RuntimeError(_lib().kmb_last_error().decode())
    return buf.raw


class Context:
    """A KMambaDistributedContext: NCCL communicator + stream of this rank."""

    def __init__(self, world: int, rank: int, device: int = -1, id128: bytes | None = None):
        L = _lib()
        if id128 is None:
            # the reference's entry: rank 0 makes the id and sends it over TCP (MASTER_ADDR / MASTER_PORT + 1)
            self.h = L.kmamba_distributed_init_nccl(world, rank)
        else:
            self.h = L.kmb_dist_init(C.create_string_buffer(id128, 128), world, rank, device)
        if not self.h:
            raise RuntimeError("distributed init failed: " + L.kmb_last_error().decode())
        self.world, self.rank = world, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        if _lib().kmb_dist_unique_id(buf) != 0:
            raise RuntimeError(_lib().kmb_last_error().decode())
        return buf.raw

    def _chk(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: {_lib().kmb_last_error().decode()}")

    def allreduce(self, ptr: int, count: int, scale: float = 1.0, stream=None):
        self._chk(_lib().kmb_dist_allreduce_async(self.h, ptr, count, scale, stream), "allreduce")

    def allgather(self, send: int, recv: int, count: int, stream=None):
        self._chk(_lib().kmb_dist_allgather_async(self.h, send, recv, count, stream), "allgather")

    def broadcast(self, ptr: int, count: int, root: int = 0, stream=None):
        self._chk(_lib().kmb_dist_broadcast_async(self.h, ptr, count, root, stream), "broadcast")

    def scannd_backward(self, params, local_batch: int, dx: int | None, overwrite: int = 0, stream=None):
        self._chk(_lib().kmb_dist_scannd_backward(self.h, C.byref(params), local_batch, dx, overwrite, stream),
                  "scannd backward")

    def convnd_backward(self, params, local_batch: int, stream=None):
        self._chk(_lib().kmb_dist_convnd_backward(self.h, C.byref(params), local_batch, stream), "convnd backward")

    def model_train_step(self, model, d_tokens: int, local_batch: int, global_batch: int, stream=None) -> float:
        return _lib().kmb_dist_model_train_step(self.h, model, d_tokens, local_batch, global_batch, stream)

    def close(self):
        if self.h:
            _lib().kmamba_distributed_fini_nccl(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
