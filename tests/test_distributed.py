"""Host-side logic of the multi-GPU path, on CPU with the gloo backend
(world size 2): batch / layer / channel splits (reference
src/kmamba_distributed.c:120-160) and the data-parallel step (broadcast,
share-weighted gradient all-reduce, global loss) against a single-process
full-batch step on a toy model."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bissimamba_b200.distributed import DataParallel, split_batch, split_channel_pairs, split_layers


def test_split_batch_matches_reference_rule():
    # 10 items over 4 ranks: 3, 3, 2, 2 (earlier ranks take the remainder)
    assert [split_batch(10, 4, r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert [split_batch(8, 8, r) for r in range(8)] == [(r, r + 1) for r in range(8)]
    assert split_batch(1, 2, 1) == (1, 1)
    assert [split_layers(12, 5, r) for r in range(5)] == [(0, 3), (3, 6), (6, 8), (8, 10), (10, 12)]


def test_split_channel_pairs_keeps_rope_pairs():
    for D in (8, 9, 64, 512):
        for world in (1, 2, 3, 8):
            ranges = [split_channel_pairs(D, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == D
            for (a, b), (c, _) in zip(ranges, ranges[1:]):
                assert b == c and (a % 2 == 0 or a == D)


class Toy:
    """loss = mean over items of 0.5 * ||W x - y||^2, plain SGD."""

    def __init__(self, W):
        self.params = W.reshape(-1).clone()
        self.grads = torch.zeros_like(self.params)

    def fb(self, batch):
        W = self.params.view(3, 4)
        X, Y = batch[:, :4], batch[:, 4:]
        R = X @ W.T - Y
        self.grads.copy_((R.T @ X / len(batch)).reshape(-1))
        return float(0.5 * (R * R).sum(1).mean())

    def step(self):
        self.params.sub_(0.1 * self.grads)


def _worker(rank, world, port, batch, W0, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    toy = Toy(torch.randn(3, 4) if rank else W0)  # rank 1 starts wrong: broadcast must fix it
    dp = DataParallel(toy.params, toy.grads, toy.fb, toy.step)
    dp.broadcast_params(0)
    losses = [dp.train_step(batch, len(batch)) for _ in range(3)]
    out[rank] = (losses, toy.params.clone())
    dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("n_items", [8, 7])
def test_data_parallel_step_equals_full_batch(n_items):
    torch.manual_seed(0)
    W0 = torch.randn(3, 4)
    batch = torch.randn(n_items, 7)
    ref = Toy(W0)
    ref_losses = []
    for _ in range(3):
        ref_losses.append(ref.fb(batch))
        ref.step()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _free_port(), batch, W0, out), nprocs=2, join=True)
    for r in range(2):
        losses, params = out[r]
        assert torch.allclose(params, ref.params, atol=1e-6)
        assert all(abs(a - b) < 1e-6 for a, b in zip(losses, ref_losses))
