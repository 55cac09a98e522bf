"""GPU test of convnd_backward_noalloc, the convnd backward for callers that
must not allocate device memory (fixed pools / arenas, allocator hooks,
lock-free paths).  It keeps its partial sums in a fixed device array inside
the library instead of a workspace.  Its results are checked against the
regular backward (convnd_batched_async) on two calls in a row, since the
array keeps the previous call's contents.  This file is named so that pytest
collects it last."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po

pytestmark = pytest.mark.gpu


def _run(kmb, dev, inp, noalloc):
    import torch
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    batch = inp["input"].shape[0]
    P = int(np.prod(inp["dims"]))
    D, K = inp["D"], inp["K"]
    V = K ** len(inp["dims"])
    din = torch.full((batch, P, D), float("nan"), device=dev)
    dk = torch.full((V, D), float("nan"), device=dev)
    db = torch.full((D,), float("nan"), device=dev)
    p = kmb.conv_params(inp["dims"], D, K, t(inp["input"]), t(inp["kernel"]), t(inp["bias"]), None,
                        t(inp["dy"]), din, dk, db)
    if noalloc:
        rc = kmb.lib().convnd_backward_noalloc(C.byref(p), batch, None)
        assert rc == 0, kmb.lib().convnd_backward_noalloc_error().decode()
    else:
        kmb.check(kmb.lib().convnd_batched_async(C.byref(p), batch, 2, None), "convnd backward")
    torch.cuda.synchronize()
    return din.cpu().numpy(), dk.cpu().numpy(), db.cpu().numpy()


def test_noalloc_backward_matches_regular_twice(kmb, cuda):
    cases = [po.gen_conv([16, 16, 16], 256, 3, batch=4, seed=31),   # BASELINE config-2 shape
             po.gen_conv([32, 32], 64, 3, batch=3, seed=32),
             # (K^3 + 1) * D = 126 * 2048 floats per partial-sum chunk: the array holds 4 chunks,
             # fewer than the regular path uses, so the rows are regrouped into 4 chunks
             po.gen_conv([16, 16, 16], 2048, 5, batch=1, seed=33)]
    for inp in cases:  # two calls in a row, different shapes: the shared array is reused
        got = _run(kmb, cuda, inp, noalloc=True)
        ref = _run(kmb, cuda, inp, noalloc=False)
        for g, r in zip(got, ref):
            np.testing.assert_allclose(g, r, rtol=1e-4, atol=1e-5 * max(1.0, np.abs(r).max()))


def test_noalloc_rejects_oversize(kmb, cuda):
    import torch
    buf = torch.zeros(16, device=cuda)
    # (K^nd + 1) * D = (5^4 + 1) * 2048 floats > the 1 Mi-float limit
    p = kmb.conv_params([5, 5, 5, 5], 2048, 5, buf, buf, None, None, buf, buf, buf, None)
    assert kmb.lib().convnd_backward_noalloc(C.byref(p), 1, None) == -1
    assert b"limit" in kmb.lib().convnd_backward_noalloc_error()
    # K^ndims far beyond any integer width is rejected the same way, not wrapped
    p = kmb.conv_params([2] * 16, 4, 1000, buf, buf, None, None, buf, buf, buf, None)
    assert kmb.lib().convnd_backward_noalloc(C.byref(p), 1, None) == -1
    assert b"limit" in kmb.lib().convnd_backward_noalloc_error()
