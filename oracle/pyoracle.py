"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU checkers.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs import this module.  It loads:

* ``liboracle.so``           -- my C restatement (scannd_oracle.c, convnd_oracle.c)
* ``_ref/libkmamba_ref.so``  -- the reference's own CPU sources compiled in place
                               (built here from the read-only reference checkout;
                               the built file travels with the repo snapshot).

It also holds the seeded synthetic input generators (numpy), whose
distributions follow the BASELINE configs.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libkmamba_ref.so")
ORACLE_SO = os.path.join(HERE, "liboracle.so")


def _reference_dir():
    """Where the reference sources are: KMB_REFERENCE_DIR, else the
    `reference_path` that BASELINE.json records (absent on the GPU box, which
    uses the prebuilt _ref library)."""
    d = os.environ.get("KMB_REFERENCE_DIR")
    if d:
        return d
    try:
        import json
        with open(os.path.join(HERE, "..", "BASELINE.json")) as f:
            return json.load(f).get("reference_path") or ""
    except (OSError, ValueError):
        return ""


REF_SRC = _reference_dir()

_f = C.POINTER(C.c_float)
_l = C.POINTER(C.c_long)


class ScanNDParams(C.Structure):
    # identical field order to the reference include/scan_nd.h:40-69
    _fields_ = [
        ("max_ndims", C.c_long), ("max_state", C.c_long), ("use_fast_exp", C.c_int),
        ("dims", _l), ("ndims", C.c_long), ("D", C.c_long), ("M", C.c_long),
        ("x", _f), ("A", _f), ("B", _f), ("C", _f), ("delta", _f),
        ("h", _f), ("y", _f), ("theta", _f), ("lambda_", _f),
        ("default_lambda", C.c_float), ("use_a_log_clamp", C.c_int), ("a_log_min", C.c_float),
        ("dA", _f), ("dB", _f), ("dC", _f), ("ddelta", _f), ("dlambda", _f), ("dtheta", _f),
    ]


class ConvNDParams(C.Structure):
    # reference include/convnd.h:10-23
    _fields_ = [
        ("input", _f), ("kernel", _f), ("bias", _f), ("output", _f), ("dy", _f),
        ("dinput", _f), ("dkernel", _f), ("dbias", _f), ("dims", _l),
        ("ndims", C.c_long), ("D", C.c_long), ("K", C.c_long),
    ]


def build(force: bool = False) -> None:
    """Build liboracle.so (always possible) and _ref (only where the reference
    sources exist, i.e. not on the GPU box, which uses the prebuilt file)."""
    targets = []
    if force or not os.path.exists(ORACLE_SO):
        targets.append("oracle")
    if REF_SRC and os.path.isdir(REF_SRC) and (force or not os.path.exists(REF_SO)):
        targets.append("ref")
    if targets:
        subprocess.run(["make", "-s", "-C", HERE, f"REF={REF_SRC}"] + targets, check=True)


_libs: dict = {}


def _lib(name: str):
    if name not in _libs:
        build()
        path = ORACLE_SO if name == "oracle" else REF_SO
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = C.CDLL(path)
        if name == "oracle":
            for fn in ("oracle_scannd_fwd", "oracle_scannd_bwd"):
                getattr(lib, fn).restype = C.c_int
            lib.oracle_scannd_fwd.argtypes = [C.POINTER(ScanNDParams)]
            lib.oracle_scannd_bwd.argtypes = [C.POINTER(ScanNDParams), _f]
            lib.oracle_convnd_fwd.argtypes = [C.POINTER(ConvNDParams)]
            lib.oracle_convnd_bwd.argtypes = [C.POINTER(ConvNDParams)]
            lib.oracle_scannd_fwd_f64.restype = C.c_int
            lib.oracle_blockscan_fwd.argtypes = [C.POINTER(BlockScanArgs)]
            lib.oracle_blockscan_bwd.argtypes = [C.POINTER(BlockScanArgs), _f, C.POINTER(BlockScanGrads)]
            lib.oracle_scannd_bound.argtypes = [C.POINTER(ScanNDParams), C.POINTER(C.c_double),
                                                C.POINTER(C.c_double)]
        else:
            lib.shim_scannd_ref.argtypes = [C.POINTER(ScanNDParams)]
            lib.shim_scannd_ref_batched.argtypes = [C.POINTER(ScanNDParams), C.c_long]
            lib.shim_convnd.argtypes = [C.POINTER(ConvNDParams), C.c_int]
            lib.shim_set_threads.argtypes = [C.c_int]
            lib.scannd_validate.argtypes = [C.POINTER(ScanNDParams)]
        _libs[name] = lib
    return _libs[name]


def have_ref() -> bool:
    try:
        _lib("ref")
        return True
    except (FileNotFoundError, OSError, subprocess.CalledProcessError):
        return False


def set_threads(n: int) -> int:
    return _lib("ref").shim_set_threads(n)


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f)


def scan_params(inp: dict, h, y, grads: dict | None = None, keep=None) -> ScanNDParams:
    """Fill ScanNDParams from a dict of numpy arrays (single item)."""
    dims = np.ascontiguousarray(inp["dims"], dtype=np.int64)
    if keep is not None:
        keep.append(dims)
    p = ScanNDParams()
    p.max_ndims = 32
    p.max_state = 0
    p.use_fast_exp = int(inp.get("use_fast_exp", 0))
    p.dims = dims.ctypes.data_as(_l)
    p.ndims = len(dims)
    p.D = inp["D"]
    p.M = inp["M"]
    p.x, p.A, p.B, p.C, p.delta = (_fp(inp[k]) for k in ("x", "A", "B", "C", "delta"))
    p.h, p.y = _fp(h), _fp(y)
    p.theta = _fp(inp.get("theta"))
    p.lambda_ = _fp(inp.get("lambda"))
    p.default_lambda = inp.get("default_lambda", 0.5)
    p.use_a_log_clamp = int(inp.get("use_a_log_clamp", 0))
    p.a_log_min = inp.get("a_log_min", -1e-5)
    g = grads or {}
    for k in ("dA", "dB", "dC", "ddelta", "dlambda", "dtheta"):
        setattr(p, k, _fp(g.get(k)))
    return p


def _item(inp: dict, b: int) -> dict:
    """Single batch item view of a batched input dict."""
    out = dict(inp)
    for k in ("x", "B", "C", "delta", "lambda"):
        if inp.get(k) is not None and inp[k].ndim > _base_ndim(k):
            out[k] = np.ascontiguousarray(inp[k][b])
    return out


def _base_ndim(k):
    return {"x": 2, "B": 3, "C": 3, "delta": 3, "lambda": 1}[k]


def ref_scannd(inp: dict):
    """Reference scannd_ref (src/scan_nd.c:219-232) on each batch item -> (h, y)."""
    return _run_fwd(inp, lambda p: _lib("ref").shim_scannd_ref(C.byref(p)))


def oracle_scannd(inp: dict):
    """My fp32 restatement -> (h, y)."""
    return _run_fwd(inp, lambda p: _lib("oracle").oracle_scannd_fwd(C.byref(p)))


def _run_fwd(inp, call):
    batch = inp.get("batch", 1)
    P = int(np.prod(inp["dims"]))
    D, M = inp["D"], inp["M"]
    hs = np.zeros((batch, P, D, M), np.float32)
    ys = np.zeros((batch, P, D), np.float32)
    for b in range(batch):
        it = _item(inp, b) if batch > 1 or inp["x"].ndim == 3 else inp
        h = np.zeros((P, D, M), np.float32)
        y = np.zeros((P, D), np.float32)
        keep = []
        p = scan_params(it, h, y, keep=keep)
        rc = call(p)
        if rc != 0:
            raise RuntimeError(f"scan oracle rc={rc}")
        hs[b], ys[b] = h, y
    return hs, ys


def scannd_bound(inp: dict):
    """(Hb, Yb) float64 magnitude bounds of h and y (see oracle_scannd_bound)."""
    batch = inp.get("batch", 1)
    P = int(np.prod(inp["dims"]))
    D, M = inp["D"], inp["M"]
    Hb = np.zeros((batch, P, D, M))
    Yb = np.zeros((batch, P, D))
    lib = _lib("oracle")
    dp = C.POINTER(C.c_double)
    for b in range(batch):
        it = _item(inp, b) if batch > 1 or inp["x"].ndim == 3 else inp
        h = np.zeros((P, D, M), np.float32)
        y = np.zeros((P, D), np.float32)
        keep = []
        p = scan_params(it, h, y, keep=keep)
        hb = np.zeros((P, D, M))
        yb = np.zeros((P, D))
        rc = lib.oracle_scannd_bound(C.byref(p), hb.ctypes.data_as(dp), yb.ctypes.data_as(dp))
        if rc != 0:
            raise RuntimeError("bound failed")
        Hb[b], Yb[b] = hb, yb
    return Hb, Yb


def oracle_scannd_bwd(inp: dict, h, dy):
    """Exact adjoint (double inside) -> dict of gradients (dA/dtheta summed over batch)."""
    batch = inp.get("batch", 1)
    dims = inp["dims"]
    P = int(np.prod(dims))
    nd = len(dims)
    D, M = inp["D"], inp["M"]
    g = {
        "dA": np.zeros((nd, D, M), np.float32),
        "dB": np.zeros((batch, P, D, M), np.float32),
        "dC": np.zeros((batch, P, D, M), np.float32),
        "ddelta": np.zeros((batch, nd, P, D), np.float32),
        "dlambda": np.zeros((batch, P), np.float32),
        "dtheta": np.zeros((max(D // 2, 1),), np.float32),
        "dx": np.zeros((batch, P, D), np.float32),
    }
    for b in range(batch):
        it = _item(inp, b) if batch > 1 or inp["x"].ndim == 3 else inp
        gi = {k: np.zeros_like(g[k][b]) for k in ("dB", "dC", "ddelta", "dlambda")}
        gi["dA"] = g["dA"]
        gi["dtheta"] = g["dtheta"] if inp.get("theta") is not None else None
        hb = np.ascontiguousarray(h[b])
        dyb = np.ascontiguousarray(dy[b])
        keep = []
        p = scan_params(it, hb, dyb, gi, keep=keep)
        dx = np.zeros((P, D), np.float32)
        rc = _lib("oracle").oracle_scannd_bwd(C.byref(p), dx.ctypes.data_as(_f))
        if rc != 0:
            raise RuntimeError("oracle bwd failed")
        for k in ("dB", "dC", "ddelta", "dlambda"):
            g[k][b] = gi[k]
        g["dx"][b] = dx
    return g


def fwd64(inp: dict, over: dict | None = None):
    """Double-precision forward of one item, with optional float64 overrides."""
    d = {k: (None if inp.get(k) is None else np.asarray(inp[k], np.float64))
         for k in ("x", "A", "B", "C", "delta", "theta", "lambda")}
    if over:
        d.update(over)
    dims = np.ascontiguousarray(inp["dims"], np.int64)
    P = int(np.prod(dims))
    D, M = inp["D"], inp["M"]
    h = np.zeros(P * D * M)
    y = np.zeros(P * D)
    dp = C.POINTER(C.c_double)

    def ptr(a):
        return None if a is None else np.ascontiguousarray(a, np.float64).ctypes.data_as(dp)

    arrs = {k: (None if v is None else np.ascontiguousarray(v, np.float64)) for k, v in d.items()}
    lib = _lib("oracle")
    rc = lib.oracle_scannd_fwd_f64(
        dims.ctypes.data_as(_l), C.c_long(len(dims)), C.c_long(D), C.c_long(M),
        ptr(arrs["x"]), ptr(arrs["A"]), ptr(arrs["B"]), ptr(arrs["C"]), ptr(arrs["delta"]),
        ptr(arrs["theta"]), ptr(arrs["lambda"]), C.c_double(inp.get("default_lambda", 0.5)),
        C.c_int(int(inp.get("use_a_log_clamp", 0))), C.c_double(inp.get("a_log_min", -1e-5)),
        C.c_int(int(inp.get("use_fast_exp", 0))),
        h.ctypes.data_as(dp), y.ctypes.data_as(dp))
    assert rc == 0
    return h.reshape(P, D, M), y.reshape(P, D)


# ----------------------------------------------------------------- generators
def gen_scan(dims, D, M, batch=1, seed=0, rope=False, lam=False, fast_exp=False,
             clamp=False, a_log_min=-1e-5, default_lambda=0.5):
    """Seeded Scan-A inputs with the BASELINE config-0 distributions:
    x ~ N(0,1); delta = softplus(N(-4, 0.5)); A = -exp(U(0, ln 16));
    B, C ~ N(0, 1/16) drawn per (p, m) and broadcast over d; theta ~ U(-pi, pi);
    lambda ~ U(0, 1) when per-point lambda is on."""
    rng = np.random.default_rng(seed)
    dims = [int(v) for v in dims]
    P = int(np.prod(dims))
    nd = len(dims)
    f32 = np.float32
    x = rng.standard_normal((batch, P, D)).astype(f32)
    delta = np.log1p(np.exp(rng.normal(-4.0, 0.5, (batch, nd, P, D)))).astype(f32)
    A = (-np.exp(rng.uniform(0.0, np.log(16.0), (nd, D, M)))).astype(f32)
    Bpm = (rng.standard_normal((batch, P, 1, M)) * 0.25).astype(f32)
    Cpm = (rng.standard_normal((batch, P, 1, M)) * 0.25).astype(f32)
    B = np.ascontiguousarray(np.broadcast_to(Bpm, (batch, P, D, M)))
    Cm = np.ascontiguousarray(np.broadcast_to(Cpm, (batch, P, D, M)))
    out = dict(dims=dims, D=D, M=M, batch=batch, x=x, delta=delta, A=A, B=B, C=Cm,
               theta=None, use_fast_exp=int(fast_exp), use_a_log_clamp=int(clamp),
               a_log_min=a_log_min, default_lambda=default_lambda)
    out["lambda"] = None
    if rope:
        out["theta"] = rng.uniform(-np.pi, np.pi, (D // 2,)).astype(f32)
    if lam:
        out["lambda"] = rng.uniform(0.0, 1.0, (batch, P)).astype(f32)
    return out


def gen_conv(dims, D, K, batch=1, seed=0, bias=True):
    """convnd inputs: input ~ N(0,1); kernel ~ N(0, 1/K^nd); bias ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    P = int(np.prod(dims))
    V = K ** len(dims)
    f32 = np.float32
    return dict(
        dims=[int(v) for v in dims], D=D, K=K, batch=batch,
        input=rng.standard_normal((batch, P, D)).astype(f32),
        kernel=(rng.standard_normal((V, D)) / np.sqrt(V)).astype(f32),
        bias=(rng.standard_normal(D) * np.sqrt(0.02)).astype(f32) if bias else None,
        dy=rng.standard_normal((batch, P, D)).astype(f32),
    )


def _conv_params(inp, b, out, dinput=None, dkernel=None, dbias=None, keep=None):
    dims = np.ascontiguousarray(inp["dims"], np.int64)
    keep.append(dims)
    p = ConvNDParams()
    inb = np.ascontiguousarray(inp["input"][b])
    keep.append(inb)
    p.input = _fp(inb)
    p.kernel = _fp(inp["kernel"])
    p.bias = _fp(inp.get("bias"))
    p.output = _fp(out)
    dyb = np.ascontiguousarray(inp["dy"][b])
    keep.append(dyb)
    p.dy = _fp(dyb)
    p.dinput, p.dkernel, p.dbias = _fp(dinput), _fp(dkernel), _fp(dbias)
    p.dims = dims.ctypes.data_as(_l)
    p.ndims = len(dims)
    p.D = inp["D"]
    p.K = inp["K"]
    return p


def conv_run(inp, which="oracle", mode=3):
    """(output, dinput, dkernel summed over batch, dbias summed over batch)."""
    batch = inp["batch"]
    P = int(np.prod(inp["dims"]))
    D = inp["D"]
    V = inp["K"] ** len(inp["dims"])
    out = np.zeros((batch, P, D), np.float32)
    din = np.zeros((batch, P, D), np.float32)
    dk = np.zeros((V, D), np.float32)
    db = np.zeros((D,), np.float32)
    for b in range(batch):
        o = np.zeros((P, D), np.float32)
        di = np.zeros((P, D), np.float32)
        dki = np.zeros((V, D), np.float32)
        dbi = np.zeros((D,), np.float32)
        keep = []
        p = _conv_params(inp, b, o, di, dki, dbi if inp.get("bias") is not None else None, keep)
        if which == "oracle":
            lib = _lib("oracle")
            if mode & 1:
                assert lib.oracle_convnd_fwd(C.byref(p)) == 0
            if mode & 2:
                assert lib.oracle_convnd_bwd(C.byref(p)) == 0
        else:
            assert _lib("ref").shim_convnd(C.byref(p), mode) == 0
        out[b], din[b] = o, di
        dk += dki
        db += dbi
    return out, din, dk, db


# ------------------------------------------------------------- block scan (Scan-B)
class BlockScanArgs(C.Structure):
    _fields_ = [("ndims", C.c_long), ("dims", _l), ("L", C.c_long), ("N", C.c_long), ("R", C.c_long),
                ("u", _f), ("dt", _f), ("lam", _f), ("B", _f), ("C", _f), ("A", _f), ("theta", _f),
                ("default_lambda", C.c_float), ("fast_exp", C.c_int),
                ("h", _f), ("Bu", _f), ("y", _f)]


class BlockScanGrads(C.Structure):
    _fields_ = [(k, _f) for k in ("dB", "dC", "du", "ddt", "dlam", "dA", "dtheta")]


def gen_blockscan(dims, N, R, batch=1, seed=0, lam=True, fast_exp=False):
    """Scan-B inputs shaped like the block produces them: u = silu(.),
    dt in [dt_min, dt_max], lambda = sigmoid(.), B/C projections, A_log = -1
    plus noise, theta in [0, 2 pi / N)."""
    rng = np.random.default_rng(seed)
    L = int(np.prod(dims))
    f32 = np.float32
    z = rng.standard_normal((batch, L, R))
    out = dict(dims=[int(d) for d in dims], N=N, R=R, batch=batch, fast_exp=int(fast_exp),
               default_lambda=0.5,
               u=(z / (1 + np.exp(-z))).astype(f32),
               dt=np.clip(np.log1p(np.exp(rng.normal(-3.0, 1.0, (batch, L)))), 1e-3, 0.1).astype(f32),
               B=(rng.standard_normal((batch, L, R * N)) * 0.5).astype(f32),
               C=(rng.standard_normal((batch, L, R * N)) * 0.5).astype(f32),
               A=(-1.0 + 0.1 * rng.standard_normal(N)).astype(f32),
               theta=rng.uniform(0, 2 * np.pi / N, max(N // 2, 1)).astype(f32))
    out["lam"] = (1 / (1 + np.exp(-rng.standard_normal((batch, L))))).astype(f32) if lam else None
    return out


def _bs_args(inp, b, h, Bu, y, keep):
    dims = np.ascontiguousarray(inp["dims"], np.int64)
    keep.append(dims)
    a = BlockScanArgs()
    a.ndims = len(dims) if len(dims) > 1 else 1
    a.dims = dims.ctypes.data_as(_l)
    a.L = int(np.prod(dims))
    a.N, a.R = inp["N"], inp["R"]
    for k in ("u", "dt", "lam", "B", "C"):
        v = inp.get(k)
        if v is not None:
            v = np.ascontiguousarray(v[b])
            keep.append(v)
        setattr(a, k, _fp(v))
    a.A = _fp(inp["A"])
    a.theta = _fp(inp["theta"])
    a.default_lambda = inp.get("default_lambda", 0.5)
    a.fast_exp = inp.get("fast_exp", 0)
    a.h, a.Bu, a.y = _fp(h), _fp(Bu), _fp(y)
    return a


def oracle_blockscan(inp):
    """(h[b,L,N], Bu[b,L,N], y[b,L,R]) from the fp32 restatement."""
    lib = _lib("oracle")
    batch, L, N, R = inp["batch"], int(np.prod(inp["dims"])), inp["N"], inp["R"]
    H = np.zeros((batch, L, N), np.float32)
    BU = np.zeros((batch, L, N), np.float32)
    Y = np.zeros((batch, L, R), np.float32)
    for b in range(batch):
        keep = []
        a = _bs_args(inp, b, H[b], BU[b], Y[b], keep)
        assert lib.oracle_blockscan_fwd(C.byref(a)) == 0
    return H, BU, Y


def oracle_blockscan_bwd(inp, h, Bu, dy):
    """Exact adjoint (double inside); dA / dtheta summed over the batch."""
    lib = _lib("oracle")
    batch, L, N, R = inp["batch"], int(np.prod(inp["dims"])), inp["N"], inp["R"]
    g = dict(dB=np.zeros((batch, L, R * N), np.float32), dC=np.zeros((batch, L, R * N), np.float32),
             du=np.zeros((batch, L, R), np.float32), ddt=np.zeros((batch, L), np.float32),
             dlam=np.zeros((batch, L), np.float32), dA=np.zeros(N, np.float32),
             dtheta=np.zeros(max(N // 2, 1), np.float32))
    for b in range(batch):
        keep = []
        hb, bub = np.ascontiguousarray(h[b]), np.ascontiguousarray(Bu[b])
        a = _bs_args(inp, b, hb, bub, np.zeros((L, R), np.float32), keep)
        gg = BlockScanGrads()
        tmp = {k: np.ascontiguousarray(g[k][b]) for k in ("dB", "dC", "du", "ddt", "dlam")}
        for k, v in tmp.items():
            setattr(gg, k, _fp(v))
        gg.dA, gg.dtheta = _fp(g["dA"]), _fp(g["dtheta"])
        dyb = np.ascontiguousarray(dy[b], np.float32)
        assert lib.oracle_blockscan_bwd(C.byref(a), dyb.ctypes.data_as(_f), C.byref(gg)) == 0
        for k, v in tmp.items():
            g[k][b] = v
    return g


def blockscan_fwd64(inp, b=0, over=None):
    lib = _lib("oracle")
    d = {k: (None if inp.get(k) is None else np.asarray(inp[k], np.float64)) for k in ("u", "dt", "lam", "B", "C")}
    d = {k: (None if v is None else np.ascontiguousarray(v[b])) for k, v in d.items()}
    d["A"] = np.asarray(inp["A"], np.float64)
    d["theta"] = np.asarray(inp["theta"], np.float64)
    if over:
        d.update({k: np.ascontiguousarray(v, np.float64) for k, v in over.items()})
    dims = np.ascontiguousarray(inp["dims"], np.int64)
    L, N, R = int(np.prod(dims)), inp["N"], inp["R"]
    h = np.zeros(L * N)
    y = np.zeros(L * R)
    dp = C.POINTER(C.c_double)
    ptr = lambda a: None if a is None else a.ctypes.data_as(dp)
    rc = lib.oracle_blockscan_fwd64(C.c_long(len(dims)), dims.ctypes.data_as(_l), C.c_long(N), C.c_long(R),
                                    ptr(d["u"]), ptr(d["dt"]), ptr(d["lam"]), ptr(d["B"]), ptr(d["C"]),
                                    ptr(d["A"]), ptr(d["theta"]), C.c_double(inp.get("default_lambda", 0.5)),
                                    C.c_int(inp.get("fast_exp", 0)), h.ctypes.data_as(dp), y.ctypes.data_as(dp))
    assert rc == 0
    return h.reshape(L, N), y.reshape(L, R)


def ref_block_run(dims, dim, N, R, params, x, dt_min=1e-3, dt_max=0.1, default_lambda=0.5, fast_exp=0, dy=None):
    """The reference MambaBlock forward (and backward when dy is given) on one
    item: returns (out, ws dict, grads dict)."""
    lib = _lib("ref")
    L = int(np.prod(dims))
    NR = N * R
    dims_a = np.ascontiguousarray(dims, np.int64)
    order = ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "lambda_proj", "b_B", "b_C", "theta")
    parr = [np.ascontiguousarray(params[k], np.float32) for k in order]
    pp = (_f * 10)(*[a.ctypes.data_as(_f) for a in parr])
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros((L, dim), np.float32)
    ws = {k: np.zeros(s, np.float32) for k, s in (("u", (L, R)), ("dt", (L,)), ("lam", (L,)), ("B", (L, NR)),
                                                   ("C", (L, NR)), ("h", (L, N)), ("Bu", (L, N)), ("y", (L, R)))}
    wsp = (_f * 8)(*[ws[k].ctypes.data_as(_f) for k in ("u", "dt", "lam", "B", "C", "h", "Bu", "y")])
    gnames = ("g_A_log", "g_theta", "d_scan_B", "d_scan_C", "d_delta", "d_lambda", "g_W_out", "g_W_B",
              "g_W_C", "g_b_B", "g_b_C", "g_delta_proj", "g_lambda_proj")
    gshapes = ((N,), (max(N // 2, 1),), (L, NR), (L, NR), (L,), (L,), (dim, R), (NR, dim), (NR, dim), (NR,),
               (NR,), (dim,), (dim,))
    grads = {k: np.zeros(s, np.float32) for k, s in zip(gnames, gshapes)} if dy is not None else {}
    gp = (_f * 13)(*[grads[k].ctypes.data_as(_f) for k in gnames]) if dy is not None else None
    dyp = np.ascontiguousarray(dy, np.float32).ctypes.data_as(_f) if dy is not None else None
    lib.shim_block_run.restype = C.c_int
    rc = lib.shim_block_run(dims_a.ctypes.data_as(_l), C.c_long(len(dims)), C.c_long(dim), C.c_long(N), C.c_long(R),
                            pp, C.c_float(dt_min), C.c_float(dt_max), C.c_float(default_lambda), C.c_int(fast_exp),
                            x.ctypes.data_as(_f), out.ctypes.data_as(_f), wsp, dyp, gp)
    if rc != 0:
        raise RuntimeError("reference block run failed")
    return out, ws, grads


# ------------------------------------------------------------- Mamba-3 block
BLOCK_KEYS = ("W_in", "W_out", "A_log", "W_B", "W_C", "delta_proj", "lambda_proj", "b_B", "b_C", "theta")


def gen_block_params(dim, N, R, seed=0):
    """Random block parameters with the reference init scales (src/mamba_block.c:227-268):
    Xavier-uniform matrices, A_log = -1, theta in [0, 2 pi / N), delta / lambda
    projections small; biases small non-zero so their gradients are exercised."""
    rng = np.random.default_rng(seed)
    NR = N * R
    xav = lambda r, c: rng.uniform(-1, 1, (r, c)) * np.sqrt(6.0 / (r + c))
    p = dict(W_in=xav(R, dim), W_out=xav(dim, R), A_log=-np.ones(N) + 0.05 * rng.standard_normal(N),
             W_B=xav(NR, dim), W_C=xav(NR, dim), delta_proj=rng.normal(0, 0.5, dim),
             lambda_proj=rng.normal(0, 0.02, dim), b_B=rng.normal(0, 0.05, NR), b_C=rng.normal(0, 0.05, NR),
             theta=rng.uniform(0, 2 * np.pi / N, max(N // 2, 1)))
    return {k: v.astype(np.float32) for k, v in p.items()}


def _block_proj64(params, x, dt_min, dt_max):
    P = {k: np.asarray(v, np.float64) for k, v in params.items()}
    x = np.asarray(x, np.float64)
    zu = x @ P["W_in"].T
    u = zu / (1 + np.exp(-zu))
    zd = x @ P["delta_proj"]
    dt = np.clip(np.log1p(np.exp(zd)), dt_min, dt_max)
    zl = x @ P["lambda_proj"]
    lam = 1 / (1 + np.exp(-zl))
    B = x @ P["W_B"].T + P["b_B"]
    Cm = x @ P["W_C"].T + P["b_C"]
    return P, x, zu, u, zd, dt, zl, lam, B, Cm


def block_fwd64(params, x, dims, N, R, dt_min=1e-3, dt_max=0.1, default_lambda=0.5):
    """Double-precision block forward of one item x[L, dim] -> out[L, dim]."""
    P, x, zu, u, zd, dt, zl, lam, B, Cm = _block_proj64(params, x, dt_min, dt_max)
    inp = dict(dims=list(dims), N=N, R=R, default_lambda=default_lambda, fast_exp=0,
               u=u[None], dt=dt[None], lam=lam[None], B=B[None], C=Cm[None], A=P["A_log"], theta=P["theta"])
    h, y = blockscan_fwd64(inp)
    return x + y @ P["W_out"].T


def block_bwd_oracle(params, x, dout, dims, N, R, dt_min=1e-3, dt_max=0.1, default_lambda=0.5):
    """Exact gradient of block_fwd64 (chain rule around the exact block-scan
    adjoint): dict of parameter gradients and 'dx'.  One item."""
    P, x64, zu, u, zd, dt, zl, lam, B, Cm = _block_proj64(params, x, dt_min, dt_max)
    f = lambda a: np.ascontiguousarray(a, np.float32)
    inp = dict(dims=list(dims), N=N, R=R, batch=1, default_lambda=default_lambda, fast_exp=0,
               u=f(u[None]), dt=f(dt[None]), lam=f(lam[None]), B=f(B[None]), C=f(Cm[None]),
               A=f(P["A_log"]), theta=f(P["theta"]))
    h64, y64 = blockscan_fwd64(inp)
    _, Bu, _ = oracle_blockscan(inp)
    dout = np.asarray(dout, np.float64)
    dy = dout @ P["W_out"]
    g = oracle_blockscan_bwd(inp, f(h64[None]), Bu, f(dy[None]))
    s = 1 / (1 + np.exp(-zu))
    dzu = g["du"][0] * s * (1 + zu * (1 - s))
    sp = np.log1p(np.exp(zd))
    dzd = np.where((sp > dt_min) & (sp < dt_max), g["ddt"][0] / (1 + np.exp(-zd)), 0.0)
    dzl = g["dlam"][0] * lam * (1 - lam)
    dB, dC = g["dB"][0].astype(np.float64), g["dC"][0].astype(np.float64)
    out = dict(W_out=dout.T @ y64, W_in=dzu.T @ x64, delta_proj=dzd @ x64, lambda_proj=dzl @ x64,
               W_B=dB.T @ x64, W_C=dC.T @ x64, b_B=dB.sum(0), b_C=dC.sum(0),
               A_log=g["dA"].astype(np.float64), theta=g["dtheta"].astype(np.float64))
    out["dx"] = (dout + dzu @ P["W_in"] + np.outer(dzd, P["delta_proj"]) + np.outer(dzl, P["lambda_proj"])
                 + dB @ P["W_B"] + dC @ P["W_C"])
    return out


# ------------------------------------------------------------- model (config 4)
def model_tensor_names(nl):
    names = ["embedding", "head"]
    for i in range(nl):
        names += [f"layers.{i}.{k}" for k in BLOCK_KEYS]
    return names


def gen_model_params(V, dim, N, R, nl, seed=0):
    rng = np.random.default_rng(seed)
    lim_e = np.sqrt(6.0 / (V + dim))
    p = {"embedding": rng.uniform(-lim_e, lim_e, (V, dim)).astype(np.float32),
         "head": rng.uniform(-lim_e, lim_e, (dim, V)).astype(np.float32)}
    for i in range(nl):
        for k, v in gen_block_params(dim, N, R, seed=seed + 1 + i).items():
            p[f"layers.{i}.{k}"] = v
    return p


def ref_model_init(dims, V, dim, N, R, nl, seed, names, sizes):
    """The reference's kmamba_init(seed) (src/kmamba.c:453-466) -> {name: array}."""
    lib = _lib("ref")
    dims_a = np.asarray(dims, np.int64)
    outs = [np.zeros(n, np.float32) for n in sizes]
    names_a = (C.c_char_p * len(names))(*[n.encode() for n in names])
    ptrs = (C.c_void_p * len(names))(*[o.ctypes.data for o in outs])
    lib.shim_model_init_tensors.restype = C.c_int
    rc = lib.shim_model_init_tensors(dims_a.ctypes.data_as(_l), C.c_long(len(dims)), C.c_long(V), C.c_long(dim),
                                     C.c_long(N), C.c_long(R), C.c_long(nl), C.c_uint32(seed), names_a, ptrs,
                                     C.c_long(len(names)))
    if rc != 0:
        raise RuntimeError(f"shim_model_init_tensors rc={rc}")
    return dict(zip(names, outs))


def ref_model_forward(dims, V, dim, N, R, nl, params, tokens):
    """Reference kmamba_forward (CPU) logits[L, V] for one token sequence."""
    lib = _lib("ref")
    dims_a = np.ascontiguousarray(dims, np.int64)
    names = model_tensor_names(nl)
    arrs = [np.ascontiguousarray(params[n], np.float32) for n in names]
    cn = (C.c_char_p * len(names))(*[n.encode() for n in names])
    cd = (_f * len(names))(*[a.ctypes.data_as(_f) for a in arrs])
    L = int(np.prod(dims))
    tok = np.ascontiguousarray(tokens, np.uint32)
    logits = np.zeros((L, V), np.float32)
    lib.shim_model_forward.restype = C.c_int
    rc = lib.shim_model_forward(dims_a.ctypes.data_as(_l), C.c_long(len(dims)), C.c_long(V), C.c_long(dim),
                                C.c_long(N), C.c_long(R), C.c_long(nl), cn, cd, C.c_long(len(names)),
                                tok.ctypes.data_as(C.POINTER(C.c_uint32)), logits.ctypes.data_as(_f))
    if rc != 0:
        raise RuntimeError(f"reference model forward failed ({rc})")
    return logits


def model_logits64(dims, V, dim, N, R, nl, params, tokens, dt_min=1e-3, dt_max=0.1):
    """Double-precision logits[L, V] of one sequence (embedding, blocks, head)."""
    emb = np.asarray(params["embedding"], np.float64)
    tin = np.where(tokens >= V, 0, tokens).astype(np.int64)
    h = emb[tin]
    for i in range(nl):
        lp = {k: params[f"layers.{i}.{k}"] for k in BLOCK_KEYS}
        h = block_fwd64(lp, h, dims, N, R, dt_min, dt_max)
    return h @ np.asarray(params["head"], np.float64)


def perturbation_kappa(fn, arrays, n=2, eps=2.0 ** -24, seed=0, floor=1e-5):
    """Condition estimate per output entry of the double-precision map
    fn(**arrays): the change of each entry under a random relative
    perturbation of every input by eps (fp32 input rounding), over its
    magnitude: |f(x (1 + eps r)) - f(x)| / (eps max(|f(x)|, floor)), max over
    n draws.  Entries near cancellation have large values."""
    rng = np.random.default_rng(seed)
    base = np.asarray(fn(**arrays), np.float64)
    kap = np.zeros(base.shape)
    for _ in range(n):
        pert = {}
        for k, v in arrays.items():
            if isinstance(v, dict):
                pert[k] = {kk: np.asarray(vv, np.float64) * (1 + eps * rng.uniform(-1, 1, np.shape(vv)))
                           for kk, vv in v.items()}
            else:
                pert[k] = np.asarray(v, np.float64) * (1 + eps * rng.uniform(-1, 1, np.shape(v)))
        d = np.abs(np.asarray(fn(**pert), np.float64) - base)
        kap = np.maximum(kap, d / (eps * np.maximum(np.abs(base), floor)))
    return base, kap


def model_loss_and_grads(dims, V, dim, N, R, nl, params, batch_tokens, dt_min=1e-3, dt_max=0.1):
    """Mean cross-entropy over batch and positions and its exact gradient
    (double precision; embedding / blocks / head).  batch_tokens[B, L+1]."""
    B = batch_tokens.shape[0]
    L = int(np.prod(dims))
    grads = {k: np.zeros(v.shape) for k, v in params.items()}
    total = 0.0
    emb = params["embedding"].astype(np.float64)
    head = params["head"].astype(np.float64)
    for b in range(B):
        tin = batch_tokens[b, :L].astype(np.int64)
        tin = np.where(tin >= V, 0, tin)
        tgt = batch_tokens[b, 1:L + 1].astype(np.int64)
        hs = [emb[tin]]
        for i in range(nl):
            lp = {k: params[f"layers.{i}.{k}"] for k in BLOCK_KEYS}
            hs.append(block_fwd64(lp, hs[-1], dims, N, R, dt_min, dt_max))
        logits = hs[-1] @ head
        mx = logits.max(1, keepdims=True)
        lse = mx[:, 0] + np.log(np.exp(logits - mx).sum(1))
        total += float((lse - logits[np.arange(L), tgt]).sum())
        p = np.exp(logits - lse[:, None])
        p[np.arange(L), tgt] -= 1.0
        dl = p / (B * L)
        grads["head"] += hs[-1].T @ dl
        dh = dl @ head.T
        for i in reversed(range(nl)):
            lp = {k: params[f"layers.{i}.{k}"] for k in BLOCK_KEYS}
            g = block_bwd_oracle(lp, hs[i], dh, dims, N, R, dt_min, dt_max)
            for k in BLOCK_KEYS:
                grads[f"layers.{i}.{k}"] += g[k]
            dh = g["dx"]
        np.add.at(grads["embedding"], tin, dh)
    return total / (B * L), grads


def adamw_ref(p, g, m, v, lr, b1, b2, eps, wd, t):
    """reference kernels/optimizer_f32.c:82-105 in double."""
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    mh = m / (1 - b1 ** t)
    vh = v / (1 - b2 ** t)
    return p * (1 - lr * wd) - lr * mh / (np.sqrt(vh) + eps), m, v
