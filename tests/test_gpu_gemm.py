"""The tensor-core products of the block and the LM head (include/kmamba_gemm.h)
against float64 products of the same inputs.

fp32 kinds must reach fp32 accuracy: on every shape the worst error, relative
to sum_k |a_ik b_kj| (the scale a dot product's rounding error is bounded by),
stays within a small multiple of the CUDA-core fp32 kernel's own, which adds
in K order like the reference's SGEMM-free loops.  bf16 products are checked
against the float64 product of the bf16-rounded inputs (fp32 accumulation)."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SIMT, TF32X3, BF16X6, BF16X9 = 4, 1, 2, 3
DEFAULT_FLUSH = 8

# (M, N, K): block projection / dx / dWcat shapes at reduced batch, head shapes, ragged ones
SHAPES = [(1024, 260, 512), (2048, 512, 260), (260, 512, 4096), (512, 256, 64), (300, 100, 77),
          (128, 16, 8), (1000, 33, 200)]


def _run_f32(kmb, kind, trans, A, B, M, N, K, acc=None):
    D = acc.clone() if acc is not None else torch.full((M, N), float("nan"), device=A.device)
    lda, ldb = A.shape[1], B.shape[1]
    kmb.check(kmb.lib().kmb_gemm_f32(kind, trans, M, N, K, A.data_ptr(), lda, B.data_ptr(), ldb, D.data_ptr(), N,
                                     1 if acc is not None else 0, None), "kmb_gemm_f32")
    torch.cuda.synchronize()
    return D


def _err(D, ref, scale):
    return float((np.abs(D.cpu().double().numpy() - ref) / np.maximum(scale, 1e-30)).max())


def _bias(D, ref, scale):
    """mean signed error relative to sum |a b|: a truncating accumulator shows here"""
    return float(((D.cpu().double().numpy() - ref) / np.maximum(scale, 1e-30)).mean())


@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_f32_kinds_reach_fp32_accuracy(kmb, cuda, M, N, K, trans):
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    a = torch.randn((K, M) if trans else (M, K), generator=g)
    b = torch.randn((K, N) if trans else (N, K), generator=g)
    a64, b64 = a.double().numpy(), b.double().numpy()
    am, bm = (a64.T, b64) if trans else (a64, b64.T)
    ref = am @ bm
    scale = np.abs(am) @ np.abs(bm)
    A, B = a.to(cuda), b.to(cuda)
    errs = {}
    for flush in (1, 2, 8, 16):
        kmb.check(kmb.lib().kmb_gemm_set_f32_flush(flush), "flush")
        for kind in (SIMT, TF32X3, BF16X6, BF16X9):
            D = _run_f32(kmb, kind, trans, A, B, M, N, K)
            errs[kind, flush] = _err(D, ref, scale)
            errs[kind, flush, "bias"] = _bias(D, ref, scale)
            errs[kind, flush, "path"] = kmb.lib().kmb_gemm_last_path()
        print(f"\n[gemm f32] M={M} N={N} K={K} trans={trans} flush={flush} err,bias /2^-24: " +
              " ".join(f"{n}={errs[k, flush] * 2**24:.2f},{errs[k, flush, 'bias'] * 2**24:+.3f}"
                       f"(p{errs[k, flush, 'path']})" for n, k in
                       (("simt", SIMT), ("tf32x3", TF32X3), ("bf16x6", BF16X6), ("bf16x9", BF16X9))))
    kmb.check(kmb.lib().kmb_gemm_set_f32_flush(DEFAULT_FLUSH), "flush")
    base = max(errs[SIMT, 1], 2.0 ** -24)
    for kind in (BF16X6, BF16X9):
        # the default flush interval is within 2x of the fp32 FMA loop's error (below it on most shapes)
        assert errs[kind, DEFAULT_FLUSH] <= 2 * base, (kind, errs[kind, DEFAULT_FLUSH], base)
    # 3xTF32 keeps the tf32 rounding of its low pieces (about 2^-22 relative per product): 4 units more
    assert errs[TF32X3, DEFAULT_FLUSH] <= 2 * base + 4 * 2.0 ** -24, (errs[TF32X3, DEFAULT_FLUSH], base)


@pytest.mark.parametrize("trans", [0, 1])
def test_f32_tensor_core_path_taken_and_accumulate(kmb, cuda, trans):
    M, N, K = 512, 256, 512
    g = torch.Generator().manual_seed(5)
    a = torch.randn((K, M) if trans else (M, K), generator=g).to(cuda)
    b = torch.randn((K, N) if trans else (N, K), generator=g).to(cuda)
    c = torch.randn((M, N), generator=g).to(cuda)
    for kind in (TF32X3, BF16X6, BF16X9):
        D = _run_f32(kmb, kind, trans, a, b, M, N, K, acc=c)
        assert kmb.lib().kmb_gemm_last_path() == 1, kind
        ref = (a.double().T if trans else a.double()) @ (b.double() if trans else b.double().T) + c.double()
        assert torch.allclose(D.double(), ref, rtol=1e-5, atol=1e-4), kind


@pytest.mark.parametrize("trans", [0, 1])
@pytest.mark.parametrize("M,N,K", [(1024, 272, 512), (272, 512, 8192), (256, 64, 128), (100, 40, 72)])
def test_bf16_product(kmb, cuda, M, N, K, trans):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn((K, M) if trans else (M, K), generator=g).bfloat16()
    b = torch.randn((K, N) if trans else (N, K), generator=g).bfloat16()
    a64, b64 = a.double().numpy(), b.double().numpy()
    am, bm = (a64.T, b64) if trans else (a64, b64.T)
    ref, scale = am @ bm, np.abs(am) @ np.abs(bm)
    A, B = a.to(cuda), b.to(cuda)
    D = torch.full((M, N), float("nan"), device=cuda)
    kmb.check(kmb.lib().kmb_gemm_bf16(trans, M, N, K, A.data_ptr(), A.shape[1], B.data_ptr(), B.shape[1],
                                      D.data_ptr(), N, 0, None), "kmb_gemm_bf16")
    torch.cuda.synchronize()
    path = kmb.lib().kmb_gemm_last_path()
    err = _err(D, ref, scale)
    print(f"\n[gemm bf16] M={M} N={N} K={K} trans={trans} path={path} err/2^-24={err * 2**24:.2f}")
    assert err <= 64 * 2.0 ** -24, err
    if M % 8 == 0 and N % 8 == 0 and K % 8 == 0:
        assert path == 1
