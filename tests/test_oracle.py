"""CPU tests: the oracle is pinned to the reference.

* the reference's own known-answer vectors (tests/unit/test_scan_nd.c:53-171,
  tests/unit/test_convnd_full.c:14-57, tests/unit/test_wavefront_nd.c:104-156);
* bit-equality of the restatement with the reference compiled in place
  (oracle/_ref), and with the committed golden fixtures made from it;
* the double-precision adjoint against central finite differences.
"""
import math

import numpy as np
import pytest

import make_golden as mg
from oracle import pyoracle as po


def _kat_inputs(nd):
    dims = [2] * nd
    P = 2 ** nd
    A = np.array([math.log(2.0), math.log(3.0)] if nd == 2 else [0.0] * 3, np.float32).reshape(nd, 1, 1)
    one = np.ones((1, P, 1), np.float32)
    return dict(dims=dims, D=1, M=1, batch=1, x=one, A=A, B=one.reshape(1, P, 1, 1).copy(),
                C=one.reshape(1, P, 1, 1).copy(), delta=np.ones((1, nd, P, 1), np.float32),
                theta=None, **{"lambda": None}, default_lambda=0.5, use_a_log_clamp=1,
                a_log_min=-1e-5, use_fast_exp=0)


# expected values from the reference tests/unit/test_scan_nd.c:63 and :121
KAT_2D = [1.0, 2.99998, 2.99998, 7.99989]
KAT_3D = [1.5, 4.49997, 4.49997, 11.99984, 4.49997, 11.99984, 11.99984, 38.99913]


@pytest.mark.parametrize("nd,expected", [(2, KAT_2D), (3, KAT_3D)])
def test_known_answer_scan(nd, expected):
    inp = _kat_inputs(nd)
    _, y = po.oracle_scannd(inp)
    np.testing.assert_allclose(y.reshape(-1), expected, atol=1e-5)
    if po.have_ref():
        _, yr = po.ref_scannd(inp)
        np.testing.assert_array_equal(y, yr)


def test_known_answer_conv():
    # reference tests/unit/test_convnd_full.c:19
    inp = dict(dims=[2, 2], D=1, K=2, batch=1,
               input=np.array([1, 2, 3, 4], np.float32).reshape(1, 4, 1),
               kernel=np.array([1, 2, 3, 4], np.float32).reshape(4, 1),
               bias=np.array([0.5], np.float32), dy=np.zeros((1, 4, 1), np.float32))
    out, *_ = po.conv_run(inp, "oracle", mode=1)
    np.testing.assert_allclose(out.reshape(-1), [4.5, 11.5, 14.5, 30.5], atol=1e-5)


@pytest.mark.parametrize("name", list(mg.SCAN_CASES))
def test_oracle_matches_reference_fixture(name):
    inp, h, y = mg.load_scan(name)
    h2, y2 = po.oracle_scannd(inp)
    np.testing.assert_array_equal(h2, h)
    np.testing.assert_array_equal(y2, y)


@pytest.mark.parametrize("name", list(mg.CONV_CASES))
def test_conv_oracle_matches_reference_fixture(name):
    inp, ref = mg.load_conv(name)
    for b in range(inp["batch"]):
        one = dict(inp, batch=1, input=inp["input"][b:b + 1], dy=inp["dy"][b:b + 1])
        o, di, dk, db = po.conv_run(one, "oracle")
        np.testing.assert_array_equal(o[0], ref["output"][b])
        np.testing.assert_array_equal(di[0], ref["dinput"][b])
        np.testing.assert_array_equal(dk, ref["dkernel"][b])
        np.testing.assert_array_equal(db, ref["dbias"][b])


@pytest.mark.skipif(not po.have_ref(), reason="reference build not available")
@pytest.mark.parametrize("dims,D,M,flags", [
    ([32, 32], 64, 16, dict(rope=True)),
    ([1024], 64, 16, {}),
    ([4, 5, 6], 6, 3, dict(rope=True, lam=True)),
])
def test_oracle_bit_equal_reference_live(dims, D, M, flags):
    inp = po.gen_scan(dims, D, M, batch=1, seed=5, **flags)
    h1, y1 = po.oracle_scannd(inp)
    h2, y2 = po.ref_scannd(inp)
    np.testing.assert_array_equal(h1, h2)
    np.testing.assert_array_equal(y1, y2)


@pytest.mark.parametrize("dims,rope,lam,fast,clamp", [
    ([5], False, False, False, False),
    ([4, 3], True, True, False, False),
    ([3, 2, 3], True, True, True, True),
    ([3, 4], False, True, False, False),
])
def test_adjoint_matches_finite_differences(dims, rope, lam, fast, clamp):
    D, M = 4, 3
    inp = po.gen_scan(dims, D, M, batch=1, seed=7, rope=rope, lam=lam, fast_exp=fast, clamp=clamp,
                      a_log_min=-2.0)
    rng = np.random.default_rng(0)
    P = int(np.prod(dims))
    dy = rng.standard_normal((1, P, D)).astype(np.float32)
    h64, _ = po.fwd64(inp)
    g = po.oracle_scannd_bwd(inp, h64[None].astype(np.float32), dy)

    def loss(over):
        _, y = po.fwd64(inp, over)
        return float((y * dy[0].astype(np.float64)).sum())

    eps = 1e-6
    checks = [("A", "dA", inp["A"]), ("B", "dB", inp["B"][0]), ("C", "dC", inp["C"][0]),
              ("delta", "ddelta", inp["delta"][0]), ("x", "dx", inp["x"][0])]
    if rope:
        checks.append(("theta", "dtheta", inp["theta"]))
    if lam:
        checks.append(("lambda", "dlambda", inp["lambda"][0]))
    for name, gname, src in checks:
        base = src.astype(np.float64)
        gg = g[gname] if gname in ("dA", "dtheta") else g[gname][0]
        for idx in list(np.ndindex(base.shape))[::max(1, base.size // 9)]:
            pp, mm = base.copy(), base.copy()
            pp[idx] += eps
            mm[idx] -= eps
            fd = (loss({name: pp}) - loss({name: mm})) / (2 * eps)
            assert abs(fd - gg[idx]) <= 1e-4 * (abs(fd) + 1e-2), (name, idx, fd, gg[idx])
