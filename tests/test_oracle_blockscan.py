"""CPU tests pinning the Mamba-3 block-scan (Scan-B) oracle.

* The fp32 restatement reproduces, bit for bit, the scan states and rank
  outputs the reference MambaBlock forward leaves in its workspace
  (src/mamba_block.c:384-470 via mamba_block_forward_ws, driven through the
  reference's public API in oracle/_ref) for 1D, 2D and 3D grids.
* The double-precision adjoint matches central finite differences of the
  double forward (the reference's own block backward averages predecessors
  and is not an exact gradient, src/mamba_block.c:640-695).
"""
import numpy as np
import pytest

from oracle import pyoracle as po


def _block_params(rng, dim, N, R):
    NR = N * R
    return dict(W_in=rng.uniform(-.3, .3, (R, dim)), W_out=rng.uniform(-.3, .3, (dim, R)), A_log=-np.ones(N),
                W_B=rng.uniform(-.3, .3, (NR, dim)), W_C=rng.uniform(-.3, .3, (NR, dim)),
                delta_proj=rng.normal(0, .5, dim), lambda_proj=rng.normal(0, .02, dim),
                b_B=rng.normal(0, .1, NR), b_C=rng.normal(0, .1, NR), theta=rng.uniform(0, 2 * np.pi / N, N // 2))


@pytest.mark.skipif(not po.have_ref(), reason="reference build not available")
@pytest.mark.parametrize("dims,N,R", [([6, 5], 8, 2), ([24], 8, 2), ([3, 4, 2], 6, 3), ([8, 8], 16, 4)])
def test_blockscan_restatement_bit_equal_reference(dims, N, R):
    rng = np.random.default_rng(sum(dims) + N)
    dim = 16
    params = _block_params(rng, dim, N, R)
    x = rng.standard_normal((int(np.prod(dims)), dim)).astype(np.float32)
    _, ws, _ = po.ref_block_run(dims, dim, N, R, params, x)
    inp = dict(dims=dims, N=N, R=R, batch=1, fast_exp=0, default_lambda=0.5, u=ws["u"][None], dt=ws["dt"][None],
               lam=ws["lam"][None], B=ws["B"][None], C=ws["C"][None], A=params["A_log"].astype(np.float32),
               theta=params["theta"].astype(np.float32))
    h, Bu, y = po.oracle_blockscan(inp)
    np.testing.assert_array_equal(h[0], ws["h"])
    np.testing.assert_array_equal(Bu[0], ws["Bu"])
    np.testing.assert_array_equal(y[0], ws["y"])


@pytest.mark.parametrize("dims,fast", [([4, 3], False), ([5], False), ([2, 3, 2], True)])
def test_blockscan_adjoint_matches_finite_differences(dims, fast):
    N, R = 6, 2
    inp = po.gen_blockscan(dims, N, R, batch=1, seed=3, fast_exp=fast)
    L = int(np.prod(dims))
    h64, _ = po.blockscan_fwd64(inp)
    _, Bu, _ = po.oracle_blockscan(inp)
    dy = np.random.default_rng(1).standard_normal((1, L, R)).astype(np.float32)
    g = po.oracle_blockscan_bwd(inp, h64[None].astype(np.float32), Bu, dy)

    def loss(over):
        _, yy = po.blockscan_fwd64(inp, 0, over)
        return float((yy * dy[0]).sum())

    eps = 1e-6
    for name, gname, src in (("u", "du", inp["u"][0]), ("dt", "ddt", inp["dt"][0]), ("lam", "dlam", inp["lam"][0]),
                             ("B", "dB", inp["B"][0]), ("C", "dC", inp["C"][0]), ("A", "dA", inp["A"]),
                             ("theta", "dtheta", inp["theta"])):
        base = src.astype(np.float64)
        gg = g[gname] if gname in ("dA", "dtheta") else g[gname][0]
        for idx in list(np.ndindex(base.shape))[::max(1, base.size // 9)]:
            pp, mm = base.copy(), base.copy()
            pp[idx] += eps
            mm[idx] -= eps
            fd = (loss({name: pp}) - loss({name: mm})) / (2 * eps)
            assert abs(fd - gg[idx]) <= 1e-4 * (abs(fd) + 1e-2), (name, idx, fd, gg[idx])


@pytest.mark.skipif(not po.have_ref(), reason="reference build not available")
@pytest.mark.parametrize("dims,N,R", [([6, 5], 8, 2), ([24], 8, 2), ([3, 4, 2], 6, 3)])
def test_block_forward_oracle_matches_reference(dims, N, R):
    dim = 16
    params = po.gen_block_params(dim, N, R, seed=sum(dims))
    x = np.random.default_rng(1).standard_normal((int(np.prod(dims)), dim)).astype(np.float32)
    out_ref, _, _ = po.ref_block_run(dims, dim, N, R, params, x)
    out64 = po.block_fwd64(params, x, dims, N, R)
    np.testing.assert_allclose(out64, out_ref, rtol=2e-5, atol=2e-5 * np.abs(out_ref).max())


@pytest.mark.parametrize("dims,N,R", [([3, 4], 4, 2), ([6], 4, 1)])
def test_block_adjoint_matches_finite_differences(dims, N, R):
    dim = 6
    params = po.gen_block_params(dim, N, R, seed=3)
    # keep the softplus away from the dt clamp so the gradient is smooth at the test point
    params["delta_proj"] = (params["delta_proj"] * 0.1).astype(np.float32)
    L = int(np.prod(dims))
    x = np.random.default_rng(2).standard_normal((L, dim)).astype(np.float32) * 0.5
    dout = np.random.default_rng(4).standard_normal((L, dim))
    g = po.block_bwd_oracle(params, x, dout, dims, N, R, dt_min=1e-4, dt_max=10.0)

    def loss(pp, xx):
        return float((po.block_fwd64(pp, xx, dims, N, R, dt_min=1e-4, dt_max=10.0) * dout).sum())

    eps = 1e-6
    for k in po.BLOCK_KEYS + ("dx",):
        base = (x if k == "dx" else params[k]).astype(np.float64)
        for idx in list(np.ndindex(base.shape))[::max(1, base.size // 5)]:
            pp, mm = base.copy(), base.copy()
            pp[idx] += eps
            mm[idx] -= eps
            if k == "dx":
                fd = (loss(params, pp) - loss(params, mm)) / (2 * eps)
            else:
                fd = (loss(dict(params, **{k: pp}), x) - loss(dict(params, **{k: mm}), x)) / (2 * eps)
            gg = g[k][idx]
            assert abs(fd - gg) <= 2e-4 * (abs(fd) + 1e-2), (k, idx, fd, gg)


@pytest.mark.skipif(not po.have_ref(), reason="reference build not available")
@pytest.mark.parametrize("dims,V,dim,N,R,nl", [([4, 8], 16, 16, 8, 2, 2), ([2, 3, 4], 24, 16, 6, 4, 2)])
def test_model_forward_oracle_matches_reference(dims, V, dim, N, R, nl):
    """The double composition (embedding -> blocks -> head) used as the model
    oracle reproduces the reference kmamba_forward (src/kmamba.c:626-660)."""
    params = po.gen_model_params(V, dim, N, R, nl, seed=3)
    tok = np.random.default_rng(1).integers(0, V, int(np.prod(dims))).astype(np.uint32)
    ref = po.ref_model_forward(dims, V, dim, N, R, nl, params, tok)
    h = params["embedding"].astype(np.float64)[tok]
    for i in range(nl):
        h = po.block_fwd64({k: params[f"layers.{i}.{k}"] for k in po.BLOCK_KEYS}, h, dims, N, R)
    logits = h @ params["head"].astype(np.float64)
    np.testing.assert_allclose(logits, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
