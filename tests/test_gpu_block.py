"""GPU parity of the Mamba-3 block (projections + block scan + output
projection) through the C ABI: forward against the reference MambaBlock
forward (oracle/_ref, fp32) and the double-precision composition; backward
against the exact gradient (chain rule around the finite-difference-pinned
block-scan adjoint; the reference omits dW_in and the projection paths of
d_input)."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po

pytestmark = pytest.mark.gpu


def _setup(kmb, dev, dims, dim, N, R, batch, seed):
    import torch
    params = po.gen_block_params(dim, N, R, seed=seed)
    L = int(np.prod(dims))
    x = np.random.default_rng(seed + 1).standard_normal((batch, L, dim)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    W = {k: t(v) for k, v in params.items()}
    cfg = kmb.block_config(dims, dim, N, R)
    w = kmb.KMBlockWeights(**{k: W[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    nact = kmb.lib().kmb_block_activation_floats(C.byref(cfg), batch)
    act = torch.empty(nact, device=dev)
    xt = t(x)
    out = torch.empty_like(xt)
    kmb.check(kmb.lib().kmb_block_forward(C.byref(cfg), C.byref(w), xt.data_ptr(), out.data_ptr(), batch,
                                          act.data_ptr(), None), "block forward")
    torch.cuda.synchronize()
    return params, x, cfg, w, W, act, xt, out


@pytest.mark.parametrize("dims,dim,N,R", [([6, 5], 16, 8, 2), ([24], 16, 8, 2), ([3, 4, 2], 16, 6, 3),
                                          ([16, 16], 64, 64, 2), ([8, 16, 16], 64, 64, 4)])
def test_block_forward(kmb, cuda, dims, dim, N, R):
    params, x, cfg, w, W, act, xt, out = _setup(kmb, cuda, dims, dim, N, R, batch=2, seed=len(dims) + dim)
    out = out.cpu().numpy()
    for b in range(2):
        ref, _, _ = po.ref_block_run(dims, dim, N, R, params, x[b]) if po.have_ref() else (None, None, None)
        ex = po.block_fwd64(params, x[b], dims, N, R)
        e_g = np.linalg.norm(out[b] - ex)
        lim = 1e-5 * np.linalg.norm(ex)
        if ref is not None:
            from gpu_util import assert_close_strict
            lim = max(lim, 4 * np.linalg.norm(ref - ex))
            _, kap = po.perturbation_kappa(lambda params, x: po.block_fwd64(params, x, dims, N, R),
                                           dict(params=params, x=x[b]), n=6)
            assert_close_strict(out[b], ref, ex, kap, name=f"block out[{b}]")
        assert e_g <= lim + 1e-30, (e_g, lim)


@pytest.mark.parametrize("dims,dim,N,R", [([6, 5], 16, 8, 2), ([24], 16, 8, 2), ([3, 4, 2], 16, 6, 3),
                                          ([8, 8], 32, 16, 4)])
def test_block_backward(kmb, cuda, dims, dim, N, R):
    import torch
    from gpu_util import assert_grad_close
    batch = 2
    params, x, cfg, w, W, act, xt, out = _setup(kmb, cuda, dims, dim, N, R, batch=batch, seed=11 + dim)
    L = int(np.prod(dims))
    dout = np.random.default_rng(5).standard_normal((batch, L, dim)).astype(np.float32)
    G = {k: torch.zeros_like(v) for k, v in W.items()}
    g = kmb.KMBlockGrads(**{k: G[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    dx = torch.empty_like(xt)
    dt = torch.from_numpy(dout).to(cuda)
    kmb.check(kmb.lib().kmb_block_backward(C.byref(cfg), C.byref(w), xt.data_ptr(), dt.data_ptr(), dx.data_ptr(),
                                           C.byref(g), batch, act.data_ptr(), None), "block backward")
    torch.cuda.synchronize()
    ref = {k: 0.0 for k in kmb.BLOCK_FIELDS}
    dxs = []
    for b in range(batch):
        r = po.block_bwd_oracle(params, x[b], dout[b], dims, N, R)
        for k in kmb.BLOCK_FIELDS:
            ref[k] = ref[k] + r[k]
        dxs.append(r["dx"])
    for k in kmb.BLOCK_FIELDS:
        assert_grad_close(G[k].cpu().numpy(), ref[k], k)
    assert_grad_close(dx.cpu().numpy(), np.stack(dxs), "dx")


def _bf16_round(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


@pytest.mark.parametrize("dims,dim,N,R", [([6, 5], 32, 8, 2), ([16, 16], 64, 64, 2), ([64, 64], 512, 64, 2)])
def test_block_bf16_storage(kmb, cuda, dims, dim, N, R):
    """bf16 storage, fp32 state: against the double-precision
    block on bf16-rounded inputs and projection weights, 2e-2 normwise relative on
    the block's own contribution (out - x) and on every gradient."""
    import torch
    batch = 2 if np.prod(dims) <= 256 else 1
    params = po.gen_block_params(dim, N, R, seed=21)
    L = int(np.prod(dims))
    x = np.random.default_rng(22).standard_normal((batch, L, dim)).astype(np.float32)
    xb = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    W = {k: torch.from_numpy(v).to(cuda) for k, v in params.items()}
    cfg = kmb.block_config(dims, dim, N, R, bf16=True)
    w = kmb.KMBlockWeights(**{k: W[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    act = torch.empty(kmb.lib().kmb_block_activation_floats(C.byref(cfg), batch), device=cuda)
    out = torch.empty_like(xb)
    kmb.check(kmb.lib().kmb_block_forward(C.byref(cfg), C.byref(w), xb.data_ptr(), out.data_ptr(), batch,
                                          act.data_ptr(), None), "bf16 block forward")
    dout = np.random.default_rng(23).standard_normal((batch, L, dim)).astype(np.float32)
    db = torch.from_numpy(dout).to(cuda).to(torch.bfloat16)
    G = {k: torch.zeros_like(v) for k, v in W.items()}
    g = kmb.KMBlockGrads(**{k: G[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    dx = torch.empty_like(xb)
    kmb.check(kmb.lib().kmb_block_backward(C.byref(cfg), C.byref(w), xb.data_ptr(), db.data_ptr(), dx.data_ptr(),
                                           C.byref(g), batch, act.data_ptr(), None), "bf16 block backward")
    torch.cuda.synchronize()
    rp = dict(params)
    for k in ("W_in", "W_B", "W_C", "delta_proj", "lambda_proj"):
        rp[k] = _bf16_round(params[k])
    xr = xb.float().cpu().numpy()
    dr = db.float().cpu().numpy()
    outg = out.float().cpu().numpy()
    rel = lambda a, b: np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30)
    ref_g = {k: 0.0 for k in kmb.BLOCK_FIELDS}
    for b in range(batch):
        ex = po.block_fwd64(rp, xr[b], dims, N, R)
        assert rel(outg[b] - xr[b], ex - xr[b]) <= 2e-2
        r = po.block_bwd_oracle(rp, xr[b], dr[b], dims, N, R)
        for k in kmb.BLOCK_FIELDS:
            ref_g[k] = ref_g[k] + r[k]
        assert rel(dx[b].float().cpu().numpy(), r["dx"]) <= 2e-2
    for k in kmb.BLOCK_FIELDS:
        assert rel(G[k].cpu().numpy(), ref_g[k]) <= 2e-2, k


@pytest.mark.parametrize("dims,dim,N,R,keep_bu,alias", [([6, 5], 16, 8, 2, False, True), ([24], 16, 8, 1, True, False),
                                                        ([4, 4, 3], 32, 16, 2, False, False)])
def test_reference_block_abi(kmb, cuda, dims, dim, N, R, keep_bu, alias):
    """cuda_block_forward / cuda_block_backward (the reference's argument lists,
    cuda/mamba_block.cu:223-346) agree bit for bit with kmb_block_forward /
    kmb_block_backward at batch 1 with zero B / C biases, whether dt_exp is NULL
    (the reference's call) or kept, and with d_dx aliasing d_dy."""
    import torch
    params = po.gen_block_params(dim, N, R, seed=dim + N)
    params["b_B"] = np.zeros_like(params["b_B"])
    params["b_C"] = np.zeros_like(params["b_C"])
    L = int(np.prod(dims))
    NR = N * R
    rng = np.random.default_rng(3)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(cuda)
    W = {k: t(v) for k, v in params.items()}
    x = t(rng.standard_normal((L, dim)))
    dy = t(rng.standard_normal((L, dim)))
    lib = kmb.lib()
    # own ABI
    cfg = kmb.block_config(dims, dim, N, R)
    w = kmb.KMBlockWeights(**{k: W[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    act = torch.empty(lib.kmb_block_activation_floats(C.byref(cfg), 1), device=cuda)
    y_own = torch.empty_like(x)
    kmb.check(lib.kmb_block_forward(C.byref(cfg), C.byref(w), x.data_ptr(), y_own.data_ptr(), 1, act.data_ptr(),
                                    None), "block forward")
    G_own = {k: torch.zeros_like(v) for k, v in W.items()}
    g = kmb.KMBlockGrads(**{k: G_own[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    dx_own = torch.empty_like(x)
    kmb.check(lib.kmb_block_backward(C.byref(cfg), C.byref(w), x.data_ptr(), dy.data_ptr(), dx_own.data_ptr(),
                                     C.byref(g), 1, act.data_ptr(), None), "block backward")
    # reference ABI
    z = lambda *s: torch.zeros(*s, device=cuda)
    ws = dict(u_raw=z(L, R), u=z(L, R), dt_raw=z(L), dt=z(L), B_exp=z(L, NR), C_exp=z(L, NR),
              dt_exp=z(L, N) if keep_bu else None, h=z(L, N), y_scan=z(L, R), y_proj=z(L, dim), lam_raw=z(L),
              lam=z(L))
    p = lambda a: None if a is None else C.c_void_p(a.data_ptr())
    darr = kmb.dims_array(dims)
    y_ref = torch.empty_like(x)
    lib.cuda_block_forward.restype = None
    lib.cuda_block_forward(None, *[p(W[k]) for k in ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "theta",
                                                     "lambda_proj")],
                           p(x), p(y_ref), p(ws["u_raw"]), p(ws["u"]), p(ws["dt_raw"]), p(ws["dt"]), p(ws["B_exp"]),
                           p(ws["C_exp"]), p(ws["dt_exp"]), p(ws["h"]), p(ws["y_scan"]), p(ws["y_proj"]),
                           p(ws["lam_raw"]), p(ws["lam"]), L, N, dim, R, len(dims), C.cast(darr, C.POINTER(C.c_long)))
    torch.cuda.synchronize()
    assert kmb.last_error() == "", kmb.last_error()
    assert torch.equal(y_ref, y_own)
    torch.testing.assert_close(ws["y_proj"], y_own - x, rtol=0, atol=0)
    G_ref = {k: torch.zeros_like(v) for k, v in W.items()}
    dbuf = dy.clone()
    dx_ref = dbuf if alias else torch.empty_like(x)
    lib.cuda_block_backward.restype = None
    lib.cuda_block_backward(None, *[p(W[k]) for k in ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "theta",
                                                      "lambda_proj")],
                            p(x), p(ws["u_raw"]), p(ws["u"]), p(ws["dt_raw"]), p(ws["dt"]), p(ws["B_exp"]),
                            p(ws["C_exp"]), p(ws["dt_exp"]), p(ws["h"]), p(ws["y_scan"]), p(ws["lam"]), p(dbuf),
                            *[p(G_ref[k]) for k in ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "theta",
                                                    "lambda_proj")],
                            p(dx_ref), *([None] * 11), L, N, dim, R, len(dims), C.cast(darr, C.POINTER(C.c_long)))
    torch.cuda.synchronize()
    assert kmb.last_error() == "", kmb.last_error()
    for k in ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "theta", "lambda_proj"):
        assert torch.equal(G_ref[k], G_own[k]), k
    assert torch.equal(dx_ref, dx_own)


@pytest.mark.parametrize("dims,dim,N,R,batch", [([64, 64], 512, 64, 2, 2), ([5, 7], 64, 64, 2, 3),
                                                ([16, 16], 128, 64, 4, 2), ([4, 6], 64, 8, 1, 1)])
def test_block_tensor_core_projection(kmb, cuda, dims, dim, N, R, batch):
    """bf16 block forward: the tcgen05 projection with the fused epilogue against
    the cuBLAS bf16 GEMM + separate epilogue (same bf16 operands, fp32
    accumulation; only the summation order differs).  Covers a partial last
    row tile (BL % 128 != 0), the 256 + 16 column split (Rt = 260), two
    column ranges per row tile (Rt = 518 > 512), and the cuBLAS fallback when
    N R is not a multiple of 16."""
    import torch
    params = po.gen_block_params(dim, N, R, seed=5)
    L = int(np.prod(dims))
    x = torch.from_numpy(np.random.default_rng(6).standard_normal((batch, L, dim)).astype(np.float32))
    xb = x.to(cuda).to(torch.bfloat16)
    W = {k: torch.from_numpy(v).to(cuda) for k, v in params.items()}
    cfg = kmb.block_config(dims, dim, N, R, bf16=True)
    w = kmb.KMBlockWeights(**{k: W[k].data_ptr() for k in kmb.BLOCK_FIELDS})
    lib = kmb.lib()
    nact = lib.kmb_block_activation_floats(C.byref(cfg), batch)
    res = {}
    for tc in (1, 0):
        lib.kmb_block_set_tensor_cores(tc)
        act = torch.zeros(nact, device=cuda)
        out = torch.empty_like(xb)
        kmb.check(lib.kmb_block_forward(C.byref(cfg), C.byref(w), xb.data_ptr(), out.data_ptr(), batch,
                                        act.data_ptr(), None), "bf16 block forward")
        torch.cuda.synchronize()
        assert lib.kmb_device_status(None) == 0
        # N R % 16 != 0 has no tensor-core layout: the cuBLAS path runs either way
        assert lib.kmb_block_last_projection_path() == (tc if (N * R) % 16 == 0 else 0)
        # backward: dx = dout + dP Wcat on the tensor cores (residual fused) or through cuBLAS
        dout = torch.from_numpy(np.random.default_rng(7).standard_normal((batch, L, dim)).astype(np.float32))
        db = dout.to(cuda).to(torch.bfloat16)
        G = {k: torch.zeros_like(v) for k, v in W.items()}
        g = kmb.KMBlockGrads(**{k: G[k].data_ptr() for k in kmb.BLOCK_FIELDS})
        dx = torch.empty_like(xb)
        kmb.check(lib.kmb_block_backward(C.byref(cfg), C.byref(w), xb.data_ptr(), db.data_ptr(), dx.data_ptr(),
                                         C.byref(g), batch, act.data_ptr(), None), "bf16 block backward")
        torch.cuda.synchronize()
        assert lib.kmb_device_status(None) == 0
        assert lib.kmb_block_last_dx_path() == tc
        res[tc] = (out.float().cpu(), act.cpu(), dx.float().cpu(), {k: v.cpu() for k, v in G.items()})
    lib.kmb_block_set_tensor_cores(1)
    o1, a1, dx1, G1 = res[1]
    o0, a0, dx0, G0 = res[0]
    torch.testing.assert_close(dx1, dx0, rtol=1.6e-2, atol=1e-2)
    for k in kmb.BLOCK_FIELDS:
        rel = float(torch.linalg.norm(G1[k] - G0[k]) / max(float(torch.linalg.norm(G0[k])), 1e-30))
        assert rel <= 2e-2, (k, rel)
    BL, Rt, NR = batch * L, R + 2 + 2 * N * R, N * R
    # pre-activations of the u / dt / lambda columns (fp32, summation order only)
    P1 = a1[:BL * Rt].view(BL, Rt)[:, :R + 2]
    P0 = a0[:BL * Rt].view(BL, Rt)[:, :R + 2]
    torch.testing.assert_close(P1, P0, rtol=1e-4, atol=1e-4)
    # the bf16 scan inputs and the block output: within one bf16 rounding step
    torch.testing.assert_close(o1, o0, rtol=1.6e-2, atol=1e-2)
    assert torch.isfinite(o1).all()
