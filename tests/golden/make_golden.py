"""Generate the golden fixtures in this folder from the REFERENCE itself.

Runs the reference's own CPU code (compiled in place into oracle/_ref by
oracle/Makefile from the read-only reference checkout) on small seeded inputs
and stores inputs + outputs as .npz.  Re-run after changing a case:

    python tests/golden/make_golden.py

The fixtures let the GPU box (where the reference sources do not exist) check
parity against the reference's outputs, not only against the restatement.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import pyoracle as po  # noqa: E402

SCAN_CASES = {
    # name: (dims, D, M, batch, seed, flags)
    "scan_1d_small": ([64], 8, 4, 1, 11, {}),
    "scan_2d_rope_lam": ([6, 5], 6, 4, 2, 12, dict(rope=True, lam=True)),
    "scan_2d_rope_odd": ([5, 7], 5, 3, 1, 13, dict(rope=True)),
    "scan_3d_fast_clamp": ([3, 4, 2], 4, 4, 1, 14, dict(fast_exp=True, clamp=True, a_log_min=-2.0)),
    "scan_2d_tma_shape": ([8, 16], 16, 16, 1, 15, dict(rope=True, lam=True)),
    "scan_1d_tma_shape": ([64], 16, 16, 1, 16, dict(lam=True)),
}
CONV_CASES = {
    "conv_2d": ([6, 5], 8, 3, 2, 21),
    "conv_3d": ([3, 4, 5], 4, 3, 1, 22),
    "conv_2d_k2": ([4, 4], 3, 2, 1, 23),
}


def load_scan(name):
    """(inputs dict in the generator format, h_ref, y_ref)."""
    z = np.load(os.path.join(HERE, name + ".npz"))
    meta = eval(str(z["meta"]))  # written by main(): a dict of plain literals
    inp = dict(meta)
    for k in ("x", "delta", "A", "theta", "lambda"):
        inp[k] = z[k] if k in z.files else None
    D = meta["D"]
    for k in ("B", "C"):
        v = z[k]
        inp[k] = np.ascontiguousarray(np.broadcast_to(v, v.shape[:2] + (D,) + v.shape[3:]))
    return inp, z["h"], z["y"]


def load_conv(name):
    z = np.load(os.path.join(HERE, name + ".npz"))
    inp = dict(eval(str(z["meta"])))
    for k in ("input", "kernel", "bias", "dy"):
        inp[k] = z[k] if k in z.files else None
    return inp, {k: z[k] for k in ("output", "dinput", "dkernel", "dbias")}


def main():
    assert po.have_ref(), "oracle/_ref is needed (build it where the reference sources exist)"
    for name, (dims, D, M, batch, seed, flags) in SCAN_CASES.items():
        inp = po.gen_scan(dims, D, M, batch=batch, seed=seed, **flags)
        h, y = po.ref_scannd(inp)
        arrays = {k: v for k, v in inp.items() if isinstance(v, np.ndarray)}
        # B and C are drawn per (point, state) and broadcast over channels:
        # store one channel, load_scan() broadcasts it back
        arrays["B"] = np.ascontiguousarray(arrays["B"][:, :, :1, :])
        arrays["C"] = np.ascontiguousarray(arrays["C"][:, :, :1, :])
        meta = {k: v for k, v in inp.items() if not isinstance(v, np.ndarray) and v is not None}
        np.savez_compressed(os.path.join(HERE, name + ".npz"), h=h, y=y, meta=repr(meta), **arrays)
    for name, (dims, D, K, batch, seed) in CONV_CASES.items():
        inp = po.gen_conv(dims, D, K, batch=batch, seed=seed)
        out, din, dk, db = [], [], [], []
        for b in range(batch):  # the reference zeroes dkernel per call: keep per-item values
            one = dict(inp, batch=1, input=inp["input"][b:b + 1], dy=inp["dy"][b:b + 1])
            o, di, k, bb = po.conv_run(one, "ref")
            out.append(o[0]); din.append(di[0]); dk.append(k); db.append(bb)
        arrays = {k: v for k, v in inp.items() if isinstance(v, np.ndarray)}
        meta = {k: v for k, v in inp.items() if not isinstance(v, np.ndarray) and v is not None}
        np.savez_compressed(os.path.join(HERE, name + ".npz"), output=np.stack(out), dinput=np.stack(din),
                            dkernel=np.stack(dk), dbias=np.stack(db), meta=repr(meta), **arrays)
    print("wrote", len(SCAN_CASES) + len(CONV_CASES), "fixtures")


if __name__ == "__main__":
    main()
