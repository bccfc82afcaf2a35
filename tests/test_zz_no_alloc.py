"""ppdl_gemm_tf32x3_static — the tensor-core GEMM entry point that allocates
nothing, for callers that cannot hand it a workspace (a ggml custom-op hook
only sees its own tensors; ggml's allocator owns all other device memory).

Its split-weight workspace is a static device array of the library, shared
by every call and keeping the last call's contents, so the test makes two
calls in a row with different shapes and data and checks each result
against ppdl_gemm_tf32x3 (caller-provided workspace) and against a float64
matmul of the same operands, both under the GEMM tests' gate,
max|diff| / max|ref| <= 1e-5 (the two library paths run the same
arithmetic, so they agree far more closely).  This file is collected last
so that a run stopping at the first failure has run every other test; it
also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import ppdl

pytestmark = pytest.mark.gpu

RTOL = 1e-5
MAX_NK = 1 << 21


def _lib():
    L = ppdl.lib()
    common = [C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong, C.c_longlong, C.c_void_p]
    tail = [C.c_void_p, C.c_longlong, C.c_longlong, C.c_longlong, C.c_void_p]
    L.ppdl_gemm_tf32x3.argtypes = common + [C.c_void_p] + tail
    L.ppdl_gemm_tf32x3.restype = C.c_int
    L.ppdl_gemm_tf32x3_static.argtypes = common + tail
    L.ppdl_gemm_tf32x3_static.restype = C.c_int
    L.ppdl_op_device_error.restype = C.c_int
    return L


def _case(cuda, M, N, K, batch, a_m_major, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    lda = ((M if a_m_major else K) + 3) // 4 * 4
    rows = K if a_m_major else M
    A = torch.randn((batch, rows, lda), generator=g).to(cuda)
    B = (torch.randn((N, K), generator=g) / K ** 0.5).to(cuda)
    shape = (batch, N, M) if a_m_major else (batch, M, N)
    ldc = (1, M) if a_m_major else (N, 1)
    return A, B, shape, lda, rows, ldc


def _run_pair(L, cuda, M, N, K, batch, a_m_major, seed):
    A, B, shape, lda, rows, (ldc_m, ldc_n) = _case(cuda, M, N, K, batch, a_m_major, seed)
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(2 * N * K, device=cuda)
    want = torch.full(shape, float("nan"), device=cuda)
    got = torch.full(shape, float("nan"), device=cuda)
    st = L.ppdl_gemm_tf32x3(M, N, K, batch, A.data_ptr(), a_m_major, lda, rows * lda,
                            B.data_ptr(), ws.data_ptr(), want.data_ptr(), ldc_m, ldc_n, M * N,
                            stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    st = L.ppdl_gemm_tf32x3_static(M, N, K, batch, A.data_ptr(), a_m_major, lda, rows * lda,
                                   B.data_ptr(), got.data_ptr(), ldc_m, ldc_n, M * N, stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    assert L.ppdl_op_device_error() == 0
    want, got = want.cpu().numpy(), got.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= RTOL, err
    # float64 product of the same operands: A(m, k) per the layout, B [N][K]
    Ad = A.cpu().double()[:, :, :(M if a_m_major else K)]
    Am = Ad.transpose(1, 2) if a_m_major else Ad           # [batch][M][K]
    ref = Am @ B.cpu().double().T                          # [batch][M][N]
    if a_m_major:
        ref = ref.transpose(1, 2)                          # [batch][N][M]
    ref = ref.numpy()
    err64 = np.abs(got - ref).max() / np.abs(ref).max()
    assert err64 <= RTOL, err64
    return err


def test_static_workspace_gemm_matches_workspace_gemm_twice(cuda):
    L = _lib()
    # two calls in a row: the second reuses the array the first one filled,
    # with a different shape, layout and data
    _run_pair(L, cuda, 10000, 256, 704, 2, 1, seed=1)      # CHW conv layout
    _run_pair(L, cuda, 3000, 512, 256, 1, 0, seed=2)       # token-major linear layout


def test_static_workspace_rejects_oversized_weights(cuda):
    L = _lib()
    N, K = 2048, 2048                                      # 4M > 2M weights
    A = torch.zeros((K, 128), device=cuda)
    B = torch.zeros((N, K), device=cuda)
    Cc = torch.zeros((N, 128), device=cuda)
    st = L.ppdl_gemm_tf32x3_static(128, N, K, 1, A.data_ptr(), 1, 128, 128 * K, B.data_ptr(),
                                   Cc.data_ptr(), 1, 128, 0,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_ERR_SHAPE
    assert "static workspace" in ppdl.last_error()
    assert N * K > MAX_NK
