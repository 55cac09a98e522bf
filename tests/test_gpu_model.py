"""GPU tests of the k-mamba model path (kmamba_create / kmamba_forward /
kmamba_train_batch, BASELINE config 4 at reduced size):
forward logits against the reference's own kmamba_forward (oracle/_ref), and
one training step's loss, gradients and AdamW update against the exact
double-precision gradient composed from the pinned block oracle."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as po

pytestmark = pytest.mark.gpu

SHAPES = [([4, 8], 16, 16, 8, 2, 2), ([2, 3, 4], 24, 16, 6, 4, 2)]


def _model(kmb, dims, V, dim, N, R, nl, params):
    cfg = kmb.model_config(dims, V, dim, N, R, nl)
    m = kmb.lib().kmamba_create(C.byref(cfg))
    assert m, kmb.last_error()
    for name, arr in params.items():
        a = np.ascontiguousarray(arr, np.float32)
        assert kmb.lib().kmamba_set_tensor(m, name.encode(), a.ctypes.data) == 0
    return m


@pytest.mark.parametrize("dims,V,dim,N,R,nl", SHAPES)
def test_model_forward_matches_reference(kmb, cuda, dims, V, dim, N, R, nl):
    params = po.gen_model_params(V, dim, N, R, nl, seed=3)
    m = _model(kmb, dims, V, dim, N, R, nl, params)
    L = int(np.prod(dims))
    tok = np.random.default_rng(1).integers(0, V, L).astype(np.uint32)
    logits = np.zeros((L, V), np.float32)
    assert kmb.lib().kmamba_forward(m, tok.ctypes.data, logits.ctypes.data) == 0, kmb.last_error()
    kmb.lib().kmamba_free(m)
    ref = po.ref_model_forward(dims, V, dim, N, R, nl, params, tok)
    from gpu_util import assert_close_strict
    ex, kap = po.perturbation_kappa(lambda params: po.model_logits64(dims, V, dim, N, R, nl, params, tok),
                                    dict(params=params), n=6)
    assert_close_strict(logits, ref, ex, kap, name="logits")


@pytest.mark.parametrize("dims,V,dim,N,R,nl", SHAPES)
def test_model_train_step_exact_gradient(kmb, cuda, dims, V, dim, N, R, nl):
    import torch
    from gpu_util import assert_grad_close
    params = po.gen_model_params(V, dim, N, R, nl, seed=5)
    m = _model(kmb, dims, V, dim, N, R, nl, params)
    L = int(np.prod(dims))
    B = 2
    tok = np.random.default_rng(2).integers(0, V, (B, L + 1)).astype(np.uint32)
    dtok = torch.from_numpy(tok.astype(np.int32)).to(cuda)
    loss = kmb.lib().kmb_model_forward_backward(m, dtok.data_ptr(), B, None)
    torch.cuda.synchronize()
    ref_loss, ref_g = po.model_loss_and_grads(dims, V, dim, N, R, nl, params, tok)
    assert abs(loss - ref_loss) <= 1e-4 * abs(ref_loss), (loss, ref_loss)
    n = C.c_size_t()
    gptr = kmb.lib().kmb_model_grad_arena(m, C.byref(n))
    garena = torch.as_tensor(kmb.DeviceArray(gptr, n.value), device=cuda).cpu().numpy()
    for name in ref_g:
        off, cnt = C.c_size_t(), C.c_size_t()
        assert kmb.lib().kmb_model_tensor_offset(m, name.encode(), C.byref(off), C.byref(cnt)) == 0
        got = garena[off.value:off.value + cnt.value].reshape(ref_g[name].shape)
        assert_grad_close(got, ref_g[name], name)
    # AdamW step (reference kernels/optimizer_f32.c:82-105) on the gradients just computed
    opt = kmb.MBOptimConfig()
    kmb.lib().kmamba_optim_config_set_defaults(C.byref(opt))
    assert kmb.lib().kmamba_enable_training(m, C.byref(opt), 2e-3, 0.05) == 0
    assert kmb.lib().kmb_model_optimizer_step(m, None) == 0
    torch.cuda.synchronize()
    for name in ("embedding", "head", "layers.0.W_B", f"layers.{nl - 1}.theta"):
        lr, wd = (2e-3, 0.05) if name in ("embedding", "head") else (opt.lr, opt.weight_decay)
        g = garena[0:0]
        off, cnt = C.c_size_t(), C.c_size_t()
        kmb.lib().kmb_model_tensor_offset(m, name.encode(), C.byref(off), C.byref(cnt))
        g = garena[off.value:off.value + cnt.value].astype(np.float64)
        p0 = params[name].astype(np.float64).ravel()
        exp, _, _ = po.adamw_ref(p0, g, 0.0, 0.0, lr, opt.mu, opt.beta2, opt.eps, wd, 1)
        got = np.ctypeslib.as_array(kmb.lib().kmamba_get_tensor(m, name.encode()), (cnt.value,)).copy()
        np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-7)
    kmb.lib().kmamba_free(m)


def test_train_batch_reduces_loss(kmb, cuda):
    dims, V, dim, N, R, nl = [4, 8], 16, 16, 8, 2, 2
    cfg = kmb.model_config(dims, V, dim, N, R, nl)
    m = kmb.lib().kmamba_create(C.byref(cfg))
    assert kmb.lib().kmamba_init(m, 42) == 0
    opt = kmb.MBOptimConfig()
    kmb.lib().kmamba_optim_config_set_defaults(C.byref(opt))
    opt.lr = 1e-2
    assert kmb.lib().kmamba_enable_training(m, C.byref(opt), 1e-2, 0.0) == 0
    tok = np.random.default_rng(0).integers(0, V, (4, 33)).astype(np.uint32)
    losses = [kmb.lib().kmamba_train_batch(m, tok.ctypes.data, 4) for _ in range(20)]
    assert np.isfinite(losses).all()
    assert losses[-1] < losses[0], losses
    assert kmb.lib().kmamba_step_count(m) == 20
    kmb.lib().kmamba_free(m)


def test_ser_save_load_round_trip(kmb, cuda, tmp_path):
    """kmamba_save_ser writes the reference's .ser layout (embedding, per-layer
    W_in .. theta, head) byte for byte as the reference's own kser writer does
    for the same tensors; kmamba_load_ser / kmb_load_ser_ex bring back a model
    whose logits equal the saved model's bit for bit (bf16 storage: to bf16)."""
    import sys
    sys.path.insert(0, __import__("os").path.dirname(__file__))
    from test_kser import FP32, BF16, KSerConfig, _bind, _write
    if not po.have_ref():
        pytest.skip("reference build unavailable")
    dims, V, dim, N, R, nl = [4, 8], 16, 16, 8, 2, 2
    params = po.gen_model_params(V, dim, N, R, nl, seed=11)
    m = _model(kmb, dims, V, dim, N, R, nl, params)
    L = int(np.prod(dims))
    tok = np.random.default_rng(4).integers(0, V, L).astype(np.uint32)
    ref_logits = np.zeros((L, V), np.float32)
    assert kmb.lib().kmamba_forward(m, tok.ctypes.data, ref_logits.ctypes.data) == 0
    cfg = kmb.model_config(dims, V, dim, N, R, nl)
    for dt in (FP32, BF16):
        ours = str(tmp_path / f"ours{dt}.ser")
        assert kmb.lib().kmamba_save_ser(m, ours.encode(), dt) == 0, kmb.last_error()
        # the same tensors through the reference's writer, in kmamba_save_ser's order and shapes
        sc = KSerConfig(vocab_size=V, dim=dim, state_size=N, n_layers=nl, seq_len=L, d_conv=cfg.d_conv,
                        expand_factor=cfg.expand_factor, dtype=dt, model_name=bytes(cfg.model_name))
        NR, TS = N * R, max(N // 2, 1)
        shapes = {"W_in": (R, dim), "W_out": (dim, R), "A_log": (N, 0), "W_B": (NR, dim), "W_C": (NR, dim),
                  "delta_proj": (dim, 0), "lambda_proj": (dim, 0), "b_B": (NR, 0), "b_C": (NR, 0), "theta": (TS, 0)}
        tens = [("embedding", params["embedding"], (V, dim, 0, 0), dt)]
        for i in range(nl):
            for f in shapes:
                tens.append((f"layers.{i}.{f}", np.ascontiguousarray(params[f"layers.{i}.{f}"], np.float32),
                             shapes[f] + (0, 0), dt))
        tens.append(("head", params["head"], (dim, V, 0, 0), dt))
        refp = str(tmp_path / f"ref{dt}.ser")
        _write(_bind(C.CDLL(po.REF_SO)), refp, sc, [], tens)
        assert open(ours, "rb").read() == open(refp, "rb").read()
        m2 = kmb.lib().kmb_load_ser_ex(ours.encode(), 2, C.byref(cfg))   # KM_SER_VERIFY
        assert m2, kmb.last_error()
        got = np.zeros((L, V), np.float32)
        assert kmb.lib().kmamba_forward(m2, tok.ctypes.data, got.ctypes.data) == 0
        kmb.lib().kmamba_free(m2)
        if dt == FP32:
            assert np.array_equal(got, ref_logits)
        else:
            np.testing.assert_allclose(got, ref_logits, rtol=0.05, atol=0.05 * np.abs(ref_logits).max())
    kmb.lib().kmamba_free(m)
