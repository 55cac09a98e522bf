"""Helpers for the GPU parity tests: move generator inputs to the device and
call the product library through its C ABI."""
import ctypes as C

import numpy as np
import torch

import bissimamba_b200 as kmb


def to_dev(inp, dev):
    out = dict(inp)
    for k in ("x", "A", "B", "C", "delta", "theta", "lambda"):
        if inp.get(k) is not None:
            out[k] = torch.from_numpy(np.ascontiguousarray(inp[k])).to(dev)
    return out


def scan_fwd(inp, dev, batch=None):
    """Run scannd_batched on device buffers; returns (h, y) numpy + path id."""
    d = to_dev(inp, dev)
    batch = batch or inp.get("batch", 1)
    P = int(np.prod(inp["dims"]))
    D, M = inp["D"], inp["M"]
    h = torch.full((batch, P, D, M), float("nan"), device=dev)
    y = torch.full((batch, P, D), float("nan"), device=dev)
    p = kmb.scan_params(inp["dims"], D, M, d["x"], d["A"], d["B"], d["C"], d["delta"], h, y,
                        theta=d.get("theta"), lam=d.get("lambda"),
                        default_lambda=inp.get("default_lambda", 0.5),
                        use_fast_exp=inp.get("use_fast_exp", 0),
                        use_a_log_clamp=inp.get("use_a_log_clamp", 0), a_log_min=inp.get("a_log_min", -1e-5))
    kmb.check(kmb.lib().scannd_batched(C.byref(p), batch), "scannd_batched")
    path = kmb.lib().kmb_last_forward_path()
    return h.cpu().numpy(), y.cpu().numpy(), path


def scan_bwd(inp, h, dy, dev, with_dx=True):
    d = to_dev(inp, dev)
    batch = inp.get("batch", 1)
    P = int(np.prod(inp["dims"]))
    D, M = inp["D"], inp["M"]
    nd = len(inp["dims"])
    ht = torch.from_numpy(np.ascontiguousarray(h)).to(dev)
    dyt = torch.from_numpy(np.ascontiguousarray(dy)).to(dev)
    g = {
        "dA": torch.zeros((nd, D, M), device=dev),
        "dB": torch.zeros((batch, P, D, M), device=dev),
        "dC": torch.zeros((batch, P, D, M), device=dev),
        "ddelta": torch.zeros((batch, nd, P, D), device=dev),
        "dlambda": torch.zeros((batch, P), device=dev),
        "dtheta": torch.zeros((max(D // 2, 1),), device=dev),
    }
    dx = torch.zeros((batch, P, D), device=dev)
    p = kmb.scan_params(inp["dims"], D, M, d["x"], d["A"], d["B"], d["C"], d["delta"], ht, dyt,
                        theta=d.get("theta"), lam=d.get("lambda"),
                        default_lambda=inp.get("default_lambda", 0.5),
                        use_fast_exp=inp.get("use_fast_exp", 0),
                        use_a_log_clamp=inp.get("use_a_log_clamp", 0), a_log_min=inp.get("a_log_min", -1e-5),
                        grads=g)
    kmb.check(kmb.lib().scannd_backward_batched(C.byref(p), batch, dx.data_ptr() if with_dx else None),
              "scannd_backward_batched")
    out = {k: v.cpu().numpy() for k, v in g.items()}
    out["dx"] = dx.cpu().numpy()
    return out


EPS32 = 2.0 ** -24


def _item(inp, b):
    out = dict(inp, batch=1)
    for k in ("x", "B", "C", "delta", "lambda"):
        if inp.get(k) is not None:
            out[k] = np.ascontiguousarray(inp[k][b:b + 1])
    return out


def assert_scan_close(h, y, inp, href=None, yref=None, rtol=1e-4, atol=1e-5, kappa=64.0, norm_factor=2.0):
    """Parity criterion for the Scan-A forward (h and y), per batch item:

    1. identical non-finite masks against the fp32 reference;
    2. elementwise: |g - ref| <= atol + rtol*|ref| + kappa*eps32*Hb, where Hb is
       the recurrence evaluated on absolute values (oracle_scannd_bound): the
       magnitude of every term feeding that entry, i.e. what fp32 rounding in
       any evaluation order scales with (cancellation makes |ref| << Hb);
    3. normwise against the exact double-precision result:
       ||g - exact|| <= max(norm_factor ||ref - exact||, 1e-5 ||exact||): the
       GPU result is within 1e-5 normwise relative of the exact value (10x
       inside the 1e-4 parity tolerance), or as accurate as the reference's own
       fp32 evaluation up to norm_factor (2 by default; CUDA expf is a 2-ulp
       function, glibc's is sub-ulp, and the recurrence compounds that).
    Returns (worst elementwise ratio, worst normwise ratio)."""
    from oracle import pyoracle as po
    if href is None:
        href, yref = po.oracle_scannd(inp)
    Hb, Yb = po.scannd_bound(inp)
    assert np.array_equal(np.isfinite(h), np.isfinite(href)), "non-finite mask of h differs"
    assert np.array_equal(np.isfinite(y), np.isfinite(yref)), "non-finite mask of y differs"
    worst_e, worst_n = 0.0, 0.0
    for g, r, bnd, name in ((h, href, Hb, "h"), (y, yref, Yb, "y")):
        f = np.isfinite(r) & np.isfinite(bnd)
        err = np.abs(g[f].astype(np.float64) - r[f])
        bound = atol + rtol * np.abs(r[f].astype(np.float64)) + kappa * EPS32 * bnd[f]
        if err.size:
            ratio = err / bound
            k = int(ratio.argmax())
            worst_e = max(worst_e, float(ratio[k]))
            assert ratio[k] <= 1.0, (f"{name}: elementwise err/bound {ratio[k]:.3g} at flat index {k}: "
                                     f"got {g[f][k]!r} ref {r[f][k]!r} bound-scale {bnd[f][k]:.3g}")
    batch = h.shape[0]
    for b in range(batch):
        one = _item(inp, b)
        if not np.isfinite(href[b]).all():
            continue
        h64, y64 = po.fwd64(one)
        for g, r, ex, name in ((h[b], href[b], h64, "h"), (y[b], yref[b], y64, "y")):
            e_g = np.linalg.norm(g.astype(np.float64).ravel() - ex.ravel())
            e_r = np.linalg.norm(r.astype(np.float64).ravel() - ex.ravel())
            lim = max(norm_factor * e_r, 1e-5 * np.linalg.norm(ex.ravel())) + 1e-30
            worst_n = max(worst_n, e_g / lim)
            assert e_g <= lim, (f"{name}[item {b}]: ||gpu-exact|| {e_g:.3g} > max({norm_factor}||ref-exact|| "
                                f"{e_r:.3g}, 1e-5||exact||)")
    return worst_e, worst_n


KAPPA_STRICT = 256.0


def strict_scan_check(h, y, inp, href=None, yref=None, rtol=1e-4, atol=1e-5):
    """The parity bound itself, elementwise, per entry of h and y:
    |g - ref| <= atol + rtol |ref| against the reference's fp32 result.

    Counted, per case (all returned; the caller asserts):
      n            finite entries compared;
      exempt       entries where the fp32 reference itself misses that bound
                   against the exact (double-precision) result;
      violations   non-exempt entries where the GPU misses it against the
                   reference;
      cond_viol    violations at entries with condition number
                   kappa = Hb / |ref| <= KAPPA_STRICT, Hb being the recurrence on
                   absolute values (the magnitude that any fp32 evaluation
                   order's rounding scales with): must be 0;
      gpu_miss / ref_miss  entries where the GPU / the reference misses the
                   bound against the exact result;
      worst        max err/bound over the entries with kappa <= KAPPA_STRICT;
      bitident     fraction of entries bit-identical to the reference."""
    from oracle import pyoracle as po
    if href is None:
        href, yref = po.oracle_scannd(inp)
    Hb, Yb = po.scannd_bound(inp)
    out = {"n": 0, "exempt": 0, "violations": 0, "cond_viol": 0, "gpu_miss": 0, "ref_miss": 0, "worst": 0.0,
           "bitident": 0.0}
    same = 0
    for b in range(h.shape[0]):
        one = _item(inp, b)
        h64, y64 = po.fwd64(one)
        for g, r, ex, bnd in ((h[b], href[b], h64, Hb[b]), (y[b], yref[b], y64, Yb[b])):
            assert np.array_equal(np.isfinite(g), np.isfinite(r)), "non-finite mask differs"
            g = g.astype(np.float64).ravel()
            r = r.astype(np.float64).ravel()
            ex = ex.ravel()
            bnd = bnd.ravel()
            f = np.isfinite(r) & np.isfinite(ex) & np.isfinite(bnd)
            g, r, ex, bnd = g[f], r[f], ex[f], bnd[f]
            tol_r = atol + rtol * np.abs(r)
            tol_e = atol + rtol * np.abs(ex)
            exempt = np.abs(r - ex) > tol_e
            ratio = np.abs(g - r) / tol_r
            viol = ratio > 1.0
            well = bnd <= KAPPA_STRICT * np.maximum(np.abs(r), atol)
            out["n"] += int(g.size)
            out["exempt"] += int(exempt.sum())
            out["violations"] += int((viol & ~exempt).sum())
            out["cond_viol"] += int((viol & well).sum())
            out["gpu_miss"] += int((np.abs(g - ex) > tol_e).sum())
            out["ref_miss"] += int(exempt.sum())
            if well.any():
                out["worst"] = max(out["worst"], float(ratio[well].max()))
            same += int((g == r).sum())
    out["bitident"] = same / max(out["n"], 1)
    return out


def assert_scan_strict(h, y, inp, href=None, yref=None, zero_exempt=False):
    """Asserts on strict_scan_check: no violation at any entry with
    kappa <= KAPPA_STRICT; the GPU misses the bound against the exact result
    at no more entries than 1.5x the reference's own misses (+16); with
    zero_exempt, no entry is exempt and no entry violates at all."""
    r = strict_scan_check(h, y, inp, href, yref)
    assert r["cond_viol"] == 0, f"strict parity on well-conditioned entries: {r}"
    assert r["gpu_miss"] <= 1.5 * r["ref_miss"] + 16, f"strict parity against the exact result: {r}"
    if zero_exempt:
        assert r["exempt"] == 0 and r["violations"] == 0, f"strict parity, every entry: {r}"
    return r


KAPPA_PERT = 16.0


def assert_close_strict(got, ref, exact, kappa, rtol=1e-4, atol=1e-5, name="", kappa_max=KAPPA_PERT):
    """Elementwise parity bound |g - ref| <= atol + rtol |ref| against the
    fp32 reference, asserted at every entry whose condition estimate kappa
    (oracle.pyoracle.perturbation_kappa: the sensitivity to fp32 rounding of
    the inputs) is <= kappa_max; at the ill-conditioned rest the GPU may miss
    the bound against the exact result no more often than 1.5x the reference
    itself (+16).  The input-perturbation estimate does not see the rounding
    inside a recurrence, hence the low threshold: at kappa <= 16 (six draws)
    the fp32 reference itself stays within 0.14 of the bound on the block
    shapes tested, and such entries are ~88 % of the outputs."""
    g = np.asarray(got, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    e = np.asarray(exact, np.float64).ravel()
    k = np.asarray(kappa, np.float64).ravel()
    assert np.array_equal(np.isfinite(g), np.isfinite(r)), f"{name}: non-finite mask differs"
    f = np.isfinite(r) & np.isfinite(e)
    g, r, e, k = g[f], r[f], e[f], k[f]
    well = k <= kappa_max
    ratio = np.abs(g - r) / (atol + rtol * np.abs(r))
    tol_e = atol + rtol * np.abs(e)
    out = {"n": int(g.size), "well": int(well.sum()), "cond_viol": int((ratio[well] > 1).sum()),
           "violations": int((ratio > 1).sum()), "gpu_miss": int((np.abs(g - e) > tol_e).sum()),
           "ref_miss": int((np.abs(r - e) > tol_e).sum()),
           "worst_well": float(ratio[well].max()) if well.any() else 0.0}
    assert out["cond_viol"] == 0, f"{name}: strict parity on well-conditioned entries: {out}"
    assert out["gpu_miss"] <= 1.5 * out["ref_miss"] + 16, f"{name}: strict parity against the exact result: {out}"
    return out


def assert_grad_close(got, ref, name, rtol=1e-3):
    """Gradients are compared against the double-precision adjoint:
    |g - g_ref| <= rtol * (|g_ref| + max|g_ref| * 1e-3)."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    assert np.array_equal(np.isfinite(got), np.isfinite(ref)), f"{name}: non-finite mask differs"
    f = np.isfinite(ref)
    if not f.any():
        return 0.0
    mx = np.abs(ref[f]).max()
    bound = rtol * (np.abs(ref[f]) + 1e-3 * mx) + 1e-30
    worst = float((np.abs(got[f] - ref[f]) / bound).max())
    assert worst <= 1.0, f"{name}: worst err/bound {worst:.3g} (max|ref| {mx:.3g})"
    return worst
