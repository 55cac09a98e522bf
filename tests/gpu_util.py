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


def assert_scan_close(h, y, href, yref, Cm, rtol=1e-4, atol=1e-5):
    """Parity criterion: identical non-finite masks; on finite entries
    |h - h_ref| <= atol + rtol |h_ref| and |y - y_ref| <= atol + rtol * sum_m |C h_ref|
    (the y bound uses the magnitude of the summed terms: y is a sum over M
    states whose rounding error scales with sum |C h|, not with |y|)."""
    assert np.array_equal(np.isfinite(h), np.isfinite(href)), "non-finite mask of h differs"
    assert np.array_equal(np.isfinite(y), np.isfinite(yref)), "non-finite mask of y differs"
    fh = np.isfinite(href)
    err_h = np.abs(h[fh].astype(np.float64) - href[fh])
    bound_h = atol + rtol * np.abs(href[fh].astype(np.float64))
    worst = float((err_h / bound_h).max()) if err_h.size else 0.0
    assert worst <= 1.0, f"h exceeds tolerance: worst err/bound {worst:.3g}"
    scale = np.abs(Cm.astype(np.float64) * href.astype(np.float64)).sum(-1)
    fy = np.isfinite(yref) & np.isfinite(scale)
    err_y = np.abs(y[fy].astype(np.float64) - yref[fy])
    bound_y = atol + rtol * scale[fy]
    worst_y = float((err_y / bound_y).max()) if err_y.size else 0.0
    assert worst_y <= 1.0, f"y exceeds tolerance: worst err/bound {worst_y:.3g}"
    return worst, worst_y


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
