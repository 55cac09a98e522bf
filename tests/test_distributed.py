"""Host-side logic of the multi-GPU layer on CPU (no GPU, world size 2 as
processes): the reference's batch / layer split rule
(src/kmamba_distributed.c:120-160, here kmamba_distributed_split_*) and the
TCP exchange of the NCCL unique id that kmamba_distributed_init_nccl performs
(the reference's own init never distributed it)."""
import multiprocessing as mp
import os
import socket

import pytest

from bissimamba_b200.distributed import exchange_id, split_batch, split_channel_pairs, split_layers


def test_split_batch_matches_reference_rule():
    # 10 items over 4 ranks: 3, 3, 2, 2 (earlier ranks take the remainder)
    assert [split_batch(10, 4, r) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert [split_batch(8, 8, r) for r in range(8)] == [(r, r + 1) for r in range(8)]
    assert split_batch(1, 2, 1) == (1, 1)
    assert [split_layers(12, 5, r) for r in range(5)] == [(0, 3), (3, 6), (6, 8), (8, 10), (10, 12)]
    with pytest.raises(ValueError):
        split_batch(4, 0, 0)


def test_split_channel_pairs_keeps_rope_pairs():
    for D in (8, 9, 64, 512):
        for world in (1, 2, 3, 8):
            ranges = [split_channel_pairs(D, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == D
            for (a, b), (c, _) in zip(ranges, ranges[1:]):
                assert b == c and (a % 2 == 0 or a == D)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    idb = bytes(range(128)) if rank == 0 else None
    q.put((rank, exchange_id(idb, world, rank, "127.0.0.1", port)))


@pytest.mark.parametrize("world", [2, 3])
def test_id_exchange_reaches_every_rank(world):
    """Rank 0's 128-byte id arrives intact at every other rank; ranks that
    start before rank 0 listens keep retrying."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in reversed(range(world))]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(got[r] == bytes(range(128)) for r in range(world))
