"""GPU parity of the Mamba-3 block scan (Scan-B) through the C ABI.

Forward: against the fp32 restatement, which is bit-equal to the reference
MambaBlock's scan (tests/test_oracle_blockscan.py), elementwise relative to the
largest state of the point, and normwise against the exact double-precision
forward (as accurate as the reference, or within 1e-5).  Backward: against the
double-precision exact adjoint (finite-difference pinned)."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po

pytestmark = pytest.mark.gpu


def _dev(inp, dev):
    import torch
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return {k: t(inp.get(k)) for k in ("u", "dt", "lam", "B", "C", "A", "theta")}


def _fwd(kmb, dev, inp):
    import torch
    d = _dev(inp, dev)
    b, L, N, R = inp["batch"], int(np.prod(inp["dims"])), inp["N"], inp["R"]
    h = torch.full((b, L, N), float("nan"), device=dev)
    Bu = torch.full((b, L, N), float("nan"), device=dev)
    y = torch.full((b, L, R), float("nan"), device=dev)
    p = kmb.blockscan_params(inp["dims"], N, R, d["u"], d["dt"], d["lam"], d["B"], d["C"], d["A"], d["theta"],
                             h, Bu, y, use_fast_exp=inp.get("fast_exp", 0))
    kmb.check(kmb.lib().kmb_blockscan_forward(C.byref(p), b, None), "blockscan forward")
    torch.cuda.synchronize()
    return h, Bu, y, p, d


CASES = [([6, 5], 8, 2, {}), ([24], 8, 2, {}), ([3, 4, 2], 6, 3, {}), ([5, 7], 7, 1, {}),
         ([4, 4], 8, 2, dict(fast_exp=True)), ([64, 64], 64, 2, {}), ([16, 32, 32], 64, 4, {})]


@pytest.mark.parametrize("dims,N,R,fl", CASES)
def test_blockscan_forward(kmb, cuda, dims, N, R, fl):
    batch = 2 if np.prod(dims) <= 4096 else 1
    inp = po.gen_blockscan(dims, N, R, batch=batch, seed=sum(dims) + N, **fl)
    h, Bu, y, _, _ = _fwd(kmb, cuda, inp)
    h, Bu, y = h.cpu().numpy(), Bu.cpu().numpy(), y.cpu().numpy()
    rh, rBu, ry = po.oracle_blockscan(inp)
    np.testing.assert_array_equal(np.isfinite(h), np.isfinite(rh))
    # B*u products are formed in the same order: identical
    np.testing.assert_allclose(Bu, rBu, rtol=1e-6, atol=1e-6)
    for g, r in ((h, rh), (y, ry)):
        scale = np.abs(r).max(axis=-1, keepdims=True)
        assert (np.abs(g - r) <= 1e-5 + 1e-4 * np.abs(r) + 1e-4 * scale).all()
    for b in range(batch):
        h64, y64 = po.blockscan_fwd64(inp, b)
        for g, r, ex in ((h[b], rh[b], h64), (y[b], ry[b], y64)):
            e_g = np.linalg.norm(g.astype(np.float64) - ex)
            e_r = np.linalg.norm(r.astype(np.float64) - ex)
            assert e_g <= max(4 * e_r, 1e-5 * np.linalg.norm(ex)) + 1e-30, (e_g, e_r, np.linalg.norm(ex))


@pytest.mark.parametrize("dims,N,R,fl", CASES[:5] + [([16, 16], 64, 2, {})])
def test_blockscan_backward(kmb, cuda, dims, N, R, fl):
    import torch
    from gpu_util import assert_grad_close
    batch = 2
    inp = po.gen_blockscan(dims, N, R, batch=batch, seed=7 + N, **fl)
    h, Bu, y, p, d = _fwd(kmb, cuda, inp)
    L = int(np.prod(dims))
    dy = np.random.default_rng(3).standard_normal((batch, L, R)).astype(np.float32)
    z = lambda *s: torch.zeros(s, device=cuda)
    g = dict(dB=z(batch, L, R * N), dC=z(batch, L, R * N), du=z(batch, L, R), ddt=z(batch, L),
             dlambda=z(batch, L), dA_log=z(N), dtheta=z(max(N // 2, 1)))
    gr = kmb.KMBlockScanGrads(**{k: v.data_ptr() for k, v in g.items()})
    dyt = torch.from_numpy(dy).to(cuda)
    kmb.check(kmb.lib().kmb_blockscan_backward(C.byref(p), batch, dyt.data_ptr(), C.byref(gr), None), "bwd")
    torch.cuda.synchronize()
    ref = po.oracle_blockscan_bwd(inp, h.cpu().numpy(), Bu.cpu().numpy(), dy)
    names = {"dB": "dB", "dC": "dC", "du": "du", "ddt": "ddt", "dlambda": "dlam", "dA_log": "dA", "dtheta": "dtheta"}
    for k, rk in names.items():
        assert_grad_close(g[k].cpu().numpy(), ref[rk], k)


@pytest.mark.parametrize("dims,N,R", [([64, 64], 64, 2), ([9, 13], 12, 1), ([16, 64], 64, 4), ([3, 8], 7, 2),
                                      ([8, 16], 16, 4), ([5, 8], 16, 2), ([4, 3], 2, 1), ([1, 9], 64, 2),
                                      ([7, 1], 16, 2), ([5, 40], 8, 4)])
def test_blockscan_strips_path(kmb, cuda, dims, N, R):
    """2D grids run a systolic strip forward: the grouped one (several CTAs per item)
    when N is even, else (and in mode 3) the one-CTA-per-item kernel, with rows
    staged through shared memory where the shape allows, else loaded directly.  The
    path is taken, and h and Bu equal the level-synchronous kernels bit for bit
    (same per-point arithmetic); y agrees to rounding (its sum over the states is
    ordered differently)."""
    import torch
    inp = po.gen_blockscan(dims, N, R, batch=2, seed=N + R)
    lib = kmb.lib()
    staged_ok = dims[1] % 8 == 0 and N % 8 == 0   # fp32 inputs at 64 x 64, N 64 exceed the stage budget
    out = {}
    try:
        for mode in (1, 3, 2, 0):
            lib.kmb_blockscan_set_strips(mode)
            h, Bu, y, _, _ = _fwd(kmb, cuda, inp)
            path = lib.kmb_blockscan_last_forward_path()
            assert lib.kmb_device_status(None) == 0
            if mode == 0:
                assert path == 0
            elif mode == 2:
                assert path == 1
            elif mode == 1 and N % 2 == 0:
                assert path == 3
            else:
                # staged when the shape allows and three staged rows per strip fit in shared memory
                assert path == (2 if dims in ([8, 16], [5, 8]) else 1 if not staged_ok else path) and path in (1, 2)
            out[mode] = (h.cpu(), Bu.cpu(), y.cpu())
    finally:
        lib.kmb_blockscan_set_strips(1)
    h0, b0, y0 = out[0]
    for mode in (1, 3, 2):
        h1, b1, y1 = out[mode]
        assert torch.equal(b1, b0)
        assert torch.equal(h1, h0)
        torch.testing.assert_close(y1, y0, rtol=1e-5, atol=1e-5 * float(y0.abs().max()))


@pytest.mark.parametrize("dims,N,R", [([64, 64], 64, 2), ([9, 13], 12, 1), ([16, 64], 64, 4), ([3, 8], 7, 2),
                                      ([5, 80], 8, 2), ([4, 3], 2, 1), ([2, 130], 64, 1), ([7, 1], 16, 2),
                                      ([1, 9], 64, 2)])
def test_blockscan_backward_strips_path(kmb, cuda, dims, N, R):
    """2D grids whose column strips fit in 8 warps take the systolic strip backward
    (others the level kernels); its gradients match the level kernels' to rounding
    (the per-point arithmetic is the same, the successor terms are summed in a
    different association)."""
    import torch
    batch = 2
    inp = po.gen_blockscan(dims, N, R, batch=batch, seed=N + 3 * R)
    lib = kmb.lib()
    L = int(np.prod(dims))
    dy = torch.from_numpy(np.random.default_rng(5).standard_normal((batch, L, R)).astype(np.float32)).to(cuda)
    gp = 1
    while gp < 8 and gp < (N + 1) // 2:
        gp *= 2
    strips_ok = N % 2 == 0 and (((dims[1] + 1) // 2) + 32 // gp - 1) // (32 // gp) <= 8
    out = {}
    try:
        for on in (1, 0):
            lib.kmb_blockscan_set_backward_strips(on)
            h, Bu, y, p, d = _fwd(kmb, cuda, inp)
            res = {}
            for ovw in (0, 1):
                # overwrite: the per-point outputs start as NaN and must be assigned, not accumulated
                z = lambda *s: torch.zeros(s, device=cuda)
                f = (lambda *s: torch.full(s, float("nan"), device=cuda)) if ovw else z
                g = dict(dB=f(batch, L, R * N), dC=f(batch, L, R * N), du=f(batch, L, R), ddt=f(batch, L),
                         dlambda=f(batch, L), dA_log=z(N), dtheta=z(max(N // 2, 1)))
                gr = kmb.KMBlockScanGrads(**{k: v.data_ptr() for k, v in g.items()})
                kmb.check(lib.kmb_blockscan_backward_ex(C.byref(p), batch, dy.data_ptr(), C.byref(gr), ovw, None),
                          "bwd")
                torch.cuda.synchronize()
                assert lib.kmb_device_status(None) == 0
                assert lib.kmb_blockscan_last_backward_path() == (1 if on and strips_ok else 0)
                res[ovw] = {k: v.cpu() for k, v in g.items()}
            for k in res[0]:
                assert torch.equal(res[0][k], res[1][k]), k
            out[on] = res[0]
    finally:
        lib.kmb_blockscan_set_backward_strips(1)
    for k in out[0]:
        ref = out[0][k]
        torch.testing.assert_close(out[1][k], ref, rtol=1e-4, atol=1e-5 * max(float(ref.abs().max()), 1e-30),
                                   msg=lambda m: f"{k}: {m}")
