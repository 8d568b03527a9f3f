"""The token-parallel path's tensor-core GEMM (qmk_gemm_bf16_nt, tcgen05 +
TMA) through its C ABI against a torch fp32 reference of the same product
(bf16 operands are exact in fp32; only the summation order differs)."""

import ctypes
import os

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

LIB = os.path.join(ROOT, "qwen_megakernel_b200", "libqwen_megakernel.so")


def _lib():
    lib = ctypes.CDLL(LIB)
    vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.qmk_gemm_bf16_nt.restype = i
    lib.qmk_gemm_bf16_nt.argtypes = [vp, ll, ll, i, vp, ll, ll, i, i, i, i, vp, ll, ll, ll, vp, vp]
    lib.qmk_get_last_error_message.restype = ctypes.c_char_p
    return lib


def _gemm(W, A, n, rows, k, batch=1, splits=1, ldw=None, lda=None, wbs=0, abs_=0):
    lib = _lib()
    ldw = ldw or k
    lda = lda or k
    C = torch.full((batch, splits, rows, n), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.qmk_gemm_bf16_nt(W.data_ptr(), ldw, wbs, n, A.data_ptr(), lda, abs_, rows, k, batch, splits,
                              C.data_ptr(), n, splits * rows * n, rows * n, status.data_ptr(),
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.qmk_get_last_error_message().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return C


def _check(got, ref):
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-5 * scale + 1e-6, f"max |gemm - ref| = {err} (scale {scale})"


@pytest.mark.parametrize("n,rows,k", [(1024, 8, 1024), (4096, 32, 1024), (1024, 100, 3072), (6144, 256, 1024),
                                      (1000, 300, 128), (128, 1000, 1000), (151936, 2, 1024)])
def test_gemm_matches_torch(n, rows, k):
    g = torch.Generator(device="cuda").manual_seed(n + rows + k)
    W = torch.randn(n, k, generator=g, device="cuda").to(torch.bfloat16)
    A = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    C = _gemm(W, A, n, rows, k)[0, 0]
    _check(C, A.float() @ W.float().T)


@pytest.mark.parametrize("splits", [2, 4, 8])
def test_gemm_split_k_partials_sum_to_product(splits):
    n, rows, k = 1024, 32, 2048
    g = torch.Generator(device="cuda").manual_seed(splits)
    W = torch.randn(n, k, generator=g, device="cuda").to(torch.bfloat16)
    A = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    C = _gemm(W, A, n, rows, k, splits=splits)[0]
    kc = k // splits
    for s in range(splits):  # every split holds exactly its K chunk's product
        ref = A[:, s * kc:(s + 1) * kc].float() @ W[:, s * kc:(s + 1) * kc].float().T
        _check(C[s], ref)
    _check(C.sum(0), A.float() @ W.float().T)


def test_gemm_batched_strided_with_padded_rows():
    """Batched over 8 heads with row strides beyond K (as the prompt
    attention uses it: W = the transposed V cache, K = positions)."""
    batch, n, rows, k, ld = 8, 128, 260, 200, 208
    g = torch.Generator(device="cuda").manual_seed(5)
    Wf = torch.randn(batch, n, ld, generator=g, device="cuda").to(torch.bfloat16)
    Af = torch.randn(batch, rows, ld, generator=g, device="cuda").to(torch.bfloat16)
    C = _gemm(Wf, Af, n, rows, k, batch=batch, ldw=ld, lda=ld, wbs=n * ld, abs_=rows * ld)[:, 0]
    ref = torch.einsum("brk,bnk->brn", Af[:, :, :k].float(), Wf[:, :, :k].float())
    _check(C, ref)


def test_gemm_rejects_misaligned_strides():
    lib = _lib()
    W = torch.zeros(128, 100, dtype=torch.bfloat16, device="cuda")
    C = torch.zeros(4, 128, device="cuda")
    rc = lib.qmk_gemm_bf16_nt(W.data_ptr(), 100, 0, 128, W.data_ptr(), 100, 0, 4, 99, 1, 1, C.data_ptr(), 128, 0, 0,
                              None, None)
    assert rc != 0  # row stride 100 elements = 200 bytes: not a multiple of 16
