"""CPU tests of the boundary: the C-ABI library loads, exports every symbol the
public headers declare, and its host-side logic (validation, wavefront plan)
matches the reference without touching a GPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from oracle import pyoracle as po

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        txt = open(os.path.join(ROOT, "include", h)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        txt = re.sub(r"typedef[^;]*;", "", txt)
        for m in re.finditer(r"([A-Za-z_][A-Za-z0-9_]*)\s*\([^;{]*\)\s*;", txt):
            names.add(m.group(1))
    return names


def test_library_exports_every_header_symbol(kmb):
    lib = kmb.lib()
    declared = _header_functions()
    assert declared, "no declarations parsed"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    assert declared <= set(kmb.EXPORTS), declared - set(kmb.EXPORTS)


def test_struct_layout_matches_reference_abi(kmb):
    # field offsets must equal the reference struct (same declaration order)
    for f1, f2 in zip(kmb.ScanNDParams._fields_, po.ScanNDParams._fields_):
        assert getattr(kmb.ScanNDParams, f1[0]).offset == getattr(po.ScanNDParams, f2[0]).offset
    assert C.sizeof(kmb.ScanNDParams) == C.sizeof(po.ScanNDParams)
    assert C.sizeof(kmb.ConvNDParams) == C.sizeof(po.ConvNDParams)


def test_validate_rejects_bad_dims(kmb):
    # reference tests/unit/test_scan_nd.c:18-51: dims {2, 0} is invalid
    lib = kmb.lib()
    buf = np.zeros(64, np.float32)
    p = kmb.scan_params([2, 0], 1, 1, buf, buf, buf, buf, buf, buf, buf)
    assert lib.scannd_validate(C.byref(p)) == 0
    p = kmb.scan_params([2, 2], 1, 1, buf, buf, buf, buf, buf, buf, buf)
    assert lib.scannd_validate(C.byref(p)) == 1
    p = kmb.scan_params([2, 2], 1, 1, buf, buf, None, buf, buf, buf, buf)
    assert lib.scannd_validate(C.byref(p)) == 0


def test_level_sizes(kmb):
    # reference tests/unit/test_wavefront_nd.c:104-156
    lib = kmb.lib()
    for dims, expected in (([3, 4], [1, 2, 3, 3, 2, 1]), ([2, 3, 2], [1, 3, 4, 3, 1])):
        d = kmb.dims_array(dims)
        assert lib.wavefront_nd_max_level(d, len(dims)) == len(expected) - 1
        got = [lib.wavefront_nd_level_size(d, len(dims), l) for l in range(len(expected))]
        assert got == expected


@pytest.mark.parametrize("dims", [[3, 4], [2, 3, 2], [5], [4, 1, 3, 2]])
def test_plan_matches_reference_plan(kmb, dims):
    lib = kmb.lib()
    d = kmb.dims_array(dims)
    plan = lib.km_wavefront_plan_create(d, len(dims), 4)
    assert plan
    ml = lib.wavefront_nd_max_level(d, len(dims))
    mine = []
    for l in range(ml + 1):
        n = lib.km_wavefront_plan_level_size(plan, l)
        offs = lib.km_wavefront_plan_level_offsets(plan, l)
        mine.append([offs[i] for i in range(n)])
    lib.km_wavefront_plan_free(plan)
    assert sorted(x for lv in mine for x in lv) == list(range(int(np.prod(dims))))
    if po.have_ref():
        ref = po._lib("ref")
        ref.km_wavefront_plan_create.restype = C.c_void_p
        ref.km_wavefront_plan_create.argtypes = [C.POINTER(C.c_long), C.c_long, C.c_long]
        ref.km_wavefront_plan_level_size.restype = C.c_long
        ref.km_wavefront_plan_level_size.argtypes = [C.c_void_p, C.c_long]
        ref.km_wavefront_plan_level_offsets.restype = C.POINTER(C.c_long)
        ref.km_wavefront_plan_level_offsets.argtypes = [C.c_void_p, C.c_long]
        ref.km_wavefront_plan_free.argtypes = [C.c_void_p]
        rp = ref.km_wavefront_plan_create(C.cast(d, C.POINTER(C.c_long)), len(dims), 4)
        theirs = []
        for l in range(ml + 1):
            n = ref.km_wavefront_plan_level_size(rp, l)
            offs = ref.km_wavefront_plan_level_offsets(rp, l)
            theirs.append([offs[i] for i in range(n)])
        ref.km_wavefront_plan_free(rp)
        assert mine == theirs


def test_kernel_volume(kmb):
    assert kmb.lib().convnd_kernel_volume(3, 3) == 27
    assert kmb.lib().convnd_kernel_volume(2, 2) == 4


def test_model_config_layout_matches_reference(kmb):
    if not po.have_ref():
        pytest.skip("reference build not available")
    ref = po._lib("ref")
    ref.shim_sizeof_kmamba_config.restype = C.c_size_t
    ref.shim_sizeof_mboptim_config.restype = C.c_size_t
    assert C.sizeof(kmb.KMambaConfig) == ref.shim_sizeof_kmamba_config()
    assert C.sizeof(kmb.MBOptimConfig) == ref.shim_sizeof_mboptim_config()
    c = kmb.KMambaConfig()
    kmb.lib().kmamba_config_set_defaults(C.byref(c))
    assert (c.dim, c.state_size, c.seq_len, c.n_layers, c.vocab_size) == (512, 64, 1024, 12, 32768)


@pytest.mark.parametrize("dims,V,dim,N,R,nl,seed", [([16, 32, 32], 256, 512, 64, 4, 2, 42),   # BASELINE config 4 shape
                                                    ([64, 64], 256, 512, 64, 2, 1, 42),       # config 3 block
                                                    ([6, 5], 37, 24, 6, 3, 2, 7)])
def test_kmamba_init_matches_reference(dims, V, dim, N, R, nl, seed):
    """kmamba_init(seed) gives the reference's weights bit for bit: every
    tensor from kmb_init_tensor (the host stream kmamba_init uploads) equals
    the reference's kmamba_init output (oracle/_ref, the reference sources)."""
    import ctypes as C
    from oracle import pyoracle as po
    if not po.have_ref():
        pytest.skip("reference build unavailable")
    import bissimamba_b200 as kmb
    cfg = kmb.model_config(dims, V, dim, N, R, nl)
    NR, TS = N * R, max(N // 2, 1)
    sizes = {"embedding": V * dim, "head": dim * V}
    for i in range(nl):
        for f, n in (("W_in", R * dim), ("W_out", dim * R), ("A_log", N), ("W_B", NR * dim), ("W_C", NR * dim),
                     ("delta_proj", dim), ("lambda_proj", dim), ("b_B", NR), ("b_C", NR), ("theta", TS)):
            sizes[f"layers.{i}.{f}"] = n
    names = list(sizes)
    ref = po.ref_model_init(dims, V, dim, N, R, nl, seed, names, [sizes[n] for n in names])
    for n in names:
        got = np.zeros(sizes[n], np.float32)
        assert kmb.lib().kmb_init_tensor(C.byref(cfg), seed, n.encode(), got.ctypes.data, got.size) == got.size, n
        assert np.array_equal(got.view(np.uint32), ref[n].view(np.uint32)), n
