"""GPU parity of convnd forward/backward through the C ABI against the
reference's outputs (golden fixtures) and the restatement (BASELINE config 2
shapes)."""
import ctypes as C

import numpy as np
import pytest

import make_golden as mg
from oracle import pyoracle as po

pytestmark = pytest.mark.gpu


def _gpu_conv(kmb, dev, inp, b=None):
    import torch
    sl = slice(None) if b is None else slice(b, b + 1)
    batch = inp["input"][sl].shape[0]
    P = int(np.prod(inp["dims"]))
    D, K = inp["D"], inp["K"]
    V = K ** len(inp["dims"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    x, ker, dy = t(inp["input"][sl]), t(inp["kernel"]), t(inp["dy"][sl])
    bias = t(inp["bias"]) if inp.get("bias") is not None else None
    out = torch.full((batch, P, D), float("nan"), device=dev)
    din = torch.full((batch, P, D), float("nan"), device=dev)
    dk = torch.full((V, D), float("nan"), device=dev)
    db = torch.full((D,), float("nan"), device=dev) if bias is not None else None
    p = kmb.conv_params(inp["dims"], D, K, x, ker, bias, out, dy, din, dk, db)
    kmb.check(kmb.lib().convnd_batched_async(C.byref(p), batch, 3, None), "convnd_batched_async")
    torch.cuda.synchronize()
    return (out.cpu().numpy(), din.cpu().numpy(), dk.cpu().numpy(),
            db.cpu().numpy() if db is not None else None)


@pytest.mark.parametrize("name", list(mg.CONV_CASES))
def test_conv_matches_reference_fixture(kmb, cuda, name):
    inp, ref = mg.load_conv(name)
    for b in range(inp["batch"]):
        o, di, dk, db = _gpu_conv(kmb, cuda, inp, b)
        np.testing.assert_allclose(o[0], ref["output"][b], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(di[0], ref["dinput"][b], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(dk, ref["dkernel"][b], rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(db, ref["dbias"][b], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dims", [[32, 32], [16, 16, 16]])
def test_config2_shapes(kmb, cuda, dims):
    # D 256, K 3 (batch reduced to 2 for the CPU oracle)
    inp = po.gen_conv(dims, 256, 3, batch=2, seed=5)
    o, di, dk, db = _gpu_conv(kmb, cuda, inp)
    ro, rdi, rdk, rdb = po.conv_run(inp, "oracle")
    np.testing.assert_allclose(o, ro, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(di, rdi, rtol=1e-4, atol=1e-4)
    # dkernel / dbias: sums over batch*P products; relative to the sum magnitude
    scale = np.abs(rdk).max()
    np.testing.assert_allclose(dk, rdk, rtol=1e-4, atol=1e-5 * scale)
    np.testing.assert_allclose(db, rdb, rtol=1e-4, atol=1e-5 * np.abs(rdb).max())


def test_convnd_host_entry(kmb, cuda):
    """convnd() with host buffers (the reference's CPU calling convention)."""
    inp, ref = mg.load_conv("conv_2d_k2")
    P = 16
    out = np.zeros((P, 3), np.float32)
    din = np.zeros((P, 3), np.float32)
    dk = np.zeros((4, 3), np.float32)
    db = np.zeros((3,), np.float32)
    x = np.ascontiguousarray(inp["input"][0])
    dy = np.ascontiguousarray(inp["dy"][0])
    p = kmb.conv_params(inp["dims"], 3, 2, x, inp["kernel"], inp["bias"], out, dy, din, dk, db)
    kmb.lib().convnd(C.byref(p), 3)
    assert kmb.lib().convnd_status() == 0, kmb.last_error()
    np.testing.assert_allclose(out, ref["output"][0], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(din, ref["dinput"][0], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(dk, ref["dkernel"][0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dims,D,K,bias", [([1, 8], 8, 3, True), ([8, 1], 4, 3, False), ([1], 4, 3, True),
                                           ([2, 3], 8, 4, True), ([2, 2, 2, 2], 4, 2, True), ([5, 6], 7, 3, True),
                                           ([3, 3, 3], 4, 5, False), ([33], 12, 4, True)])
def test_conv_degenerate_shapes(kmb, cuda, dims, D, K, bias):
    """Size-1 axes, kernels wider than the grid (every tap out of range somewhere),
    four dimensions, odd channel counts (generic kernels) and missing bias,
    forward and backward against the restatement."""
    inp = po.gen_conv(dims, D, K, batch=2, seed=len(dims) + K + D, bias=bias)
    o, di, dk, db = _gpu_conv(kmb, cuda, inp)
    ro, rdi, rdk, rdb = po.conv_run(inp, "oracle")
    np.testing.assert_allclose(o, ro, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(di, rdi, rtol=1e-4, atol=1e-5)
    scale = max(np.abs(rdk).max(), 1e-30)
    np.testing.assert_allclose(dk, rdk, rtol=1e-4, atol=1e-5 * scale)
    if bias:
        np.testing.assert_allclose(db, rdb, rtol=1e-4, atol=1e-5 * max(np.abs(rdb).max(), 1e-30))


def test_conv_rejects_invalid(kmb, cuda):
    """Zero-sized axes, K = 0 and an empty batch are invalid arguments."""
    import torch
    z = torch.zeros(16, device=cuda)
    for dims, K, batch in (([4, 0], 3, 1), ([4, 4], 0, 1), ([4, 4], 3, 0)):
        p = kmb.conv_params(dims, 1, K, z, z, None, z, z, z, z, None)
        assert kmb.lib().convnd_batched_async(C.byref(p), batch, 3, None) == -1


@pytest.mark.parametrize("dims,D,K", [([1024], 8, 4), ([36], 16, 3), ([37], 8, 2), ([32, 32], 64, 3),
                                      ([13, 30], 8, 2), ([6, 10], 16, 4), ([48, 64], 8, 3), ([16, 16, 16], 16, 3),
                                      ([20, 16, 16], 8, 3), ([5, 7, 6], 8, 2), ([16, 16, 16], 4, 2),
                                      ([7, 9, 13], 12, 3), ([33, 5, 20], 4, 3), ([3, 11, 8], 20, 2)])
def test_fused_kernel_shapes(kmb, cuda, dims, D, K):
    """The fused forward + backward kernels (D a multiple of 8 for ndims <= 2,
    of 4 for the 3D variant):
    slabs with their causal halos, runs of 4 and of 1 along the innermost
    axis.  The forward is bit-identical to the reference's tap order; mode 1
    and mode 2 alone give the same bits as mode 3."""
    import torch
    inp = po.gen_conv(dims, D, K, batch=3, seed=sum(dims) + K, bias=True)
    o, di, dk, db = _gpu_conv(kmb, cuda, inp)
    ro, rdi, rdk, rdb = po.conv_run(inp, "oracle")
    assert np.array_equal(o, ro)
    np.testing.assert_allclose(di, rdi, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dk, rdk, rtol=1e-4, atol=1e-5 * max(np.abs(rdk).max(), 1e-30))
    np.testing.assert_allclose(db, rdb, rtol=1e-4, atol=1e-5 * max(np.abs(rdb).max(), 1e-30))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    P, V = int(np.prod(dims)), K ** len(dims)
    out = torch.zeros((3, P, D), device=cuda)
    din = torch.zeros((3, P, D), device=cuda)
    dk2, db2 = torch.zeros((V, D), device=cuda), torch.zeros((D,), device=cuda)
    p = kmb.conv_params(dims, D, K, t(inp["input"]), t(inp["kernel"]), t(inp["bias"]), out, t(inp["dy"]), din, dk2, db2)
    kmb.check(kmb.lib().convnd_batched_async(C.byref(p), 3, 1, None))
    kmb.check(kmb.lib().convnd_batched_async(C.byref(p), 3, 2, None))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), o)
    assert np.array_equal(din.cpu().numpy(), di)
    assert np.array_equal(dk2.cpu().numpy(), dk)
    assert np.array_equal(db2.cpu().numpy(), db)
