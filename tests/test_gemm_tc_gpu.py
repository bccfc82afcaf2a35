"""The FP32-faithful tensor-core GEMM (tcgen05 kind::tf32, 3xTF32 split)
through its C-ABI entry ppdl_gemm_tf32x3, against a float64 product.

The hot path's per-op gate is 1e-5 relative (max|diff| / max|ref|).  A
plain single-pass TF32 product misses it by ~2 orders of magnitude on these
data, so passing also shows that the hi/lo split is in effect.  Shapes cover
the conv layouts (A M-major: pixels contiguous, CHW), the linear layout (A
K-major), batching, and M / N / K tails of every tile size.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import ppdl

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _lib():
    L = ppdl.lib()
    L.ppdl_gemm_tf32x3.argtypes = [C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong, C.c_longlong,
                                                   C.c_void_p, C.c_void_p, C.c_void_p,
                                                   C.c_longlong, C.c_longlong, C.c_longlong,
                                                   C.c_void_p]
    L.ppdl_gemm_tf32x3.restype = C.c_int
    return L


def _gemm(cuda, M, N, K, batch, a_m_major, seed, lda_pad=0):
    rng = np.random.default_rng(seed)
    # leading dimension padded to 4 floats: TMA strides are 16-byte multiples
    lda = ((M if a_m_major else K) + 3) // 4 * 4 + lda_pad
    rows = K if a_m_major else M
    A = rng.standard_normal((batch, rows, lda), dtype=np.float32)
    B = (rng.standard_normal((N, K)) / np.sqrt(K)).astype(np.float32)
    if a_m_major:
        Am = A[:, :, :M].transpose(0, 2, 1)   # (batch, M, K)
    else:
        Am = A[:, :, :K]
    ref = np.einsum("zmk,nk->zmn", Am.astype(np.float64), B.astype(np.float64))
    dA = torch.from_numpy(A).to(cuda)
    dB = torch.from_numpy(B).to(cuda)
    ws = torch.empty(2 * N * K, device=cuda)
    # CHW-style output (m contiguous) for M-major A, row-major otherwise
    out = torch.full((batch, N, M) if a_m_major else (batch, M, N), float("nan"), device=cuda)
    ldc_m, ldc_n = (1, M) if a_m_major else (N, 1)
    L = _lib()
    st = L.ppdl_gemm_tf32x3(M, N, K, batch, dA.data_ptr(), int(a_m_major), lda, rows * lda,
                            dB.data_ptr(), ws.data_ptr(), out.data_ptr(), ldc_m, ldc_n, M * N,
                            torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    assert ppdl.lib().ppdl_op_last_error() is not None
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float64)
    if a_m_major:
        got = got.transpose(0, 2, 1)
    return got, ref


@pytest.mark.parametrize("M,N,K,batch", [
    (2500, 512, 1664, 1),    # st2 agg0
    (40000, 64, 336, 1),     # st0 agg0 (K tail: 336 = 10.5 x 32)
    (10000, 256, 704, 2),    # st1 agg0, two pages
    (130, 48, 36, 3),        # M, N and K tails, batch 3
    (2500, 48, 48, 36),      # Winograd plane GEMM shape
    (1000, 300, 32, 1),      # mask GEMM shape (N = 300 -> two 160 tiles)
])
def test_tc_gemm_m_major(cuda, M, N, K, batch):
    got, ref = _gemm(cuda, M, N, K, batch, 1, seed=M + N + K)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < RTOL, err


@pytest.mark.parametrize("M,N,K", [(3000, 256, 256), (300, 2048, 256), (300, 4, 256),
                                   (600, 512, 4), (77, 25, 256)])
def test_tc_gemm_k_major(cuda, M, N, K):
    got, ref = _gemm(cuda, M, N, K, 1, 0, seed=M * 7 + N)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < RTOL, err


# Large shapes (many tiles per SM, several k-blocks): an N tail of 44
# columns, an odd M with a partial last tile, both A layouts, a K tail,
# batches.
@pytest.mark.parametrize("M,N,K,batch,a_m_major", [
    (40000, 300, 128, 1, 1),   # N tail: 300 = 2 x 128 + 44
    (20037, 128, 160, 2, 1),   # odd M
    (40000, 256, 256, 1, 0),   # K-major A (token-major rows)
    (19000, 96, 232, 2, 0),    # K-major, N = 96, K tail (232 = 7.25 x 32)
])
def test_tc_gemm_large(cuda, M, N, K, batch, a_m_major):
    got, ref = _gemm(cuda, M, N, K, batch, a_m_major, seed=M + 3 * N + K)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < RTOL, err


# Narrow identity GEMMs of one or two k-blocks with at least four tiles per
# CTA run the alternate-tile epilogue (each epilogue warpgroup takes every
# other tile whole, with TMEM slots and barriers of its own): odd tile counts
# per CTA, M, N and K tails, both A layouts.
@pytest.mark.parametrize("M,N,K,batch,a_m_major", [
    (20000, 48, 48, 6, 1),     # the stage-0 Winograd plane GEMM shape, 942 tiles
    (19999, 40, 20, 5, 1),     # one k-block, N tail (40 of a 48-column tile), M tail
    (80000, 64, 64, 1, 0),     # K-major A, 64-column tiles, 625 tiles
    (30001, 32, 36, 3, 1),     # K tail: 36 = 32 + 4
])
def test_tc_gemm_alternate_tiles(cuda, M, N, K, batch, a_m_major):
    got, ref = _gemm(cuda, M, N, K, batch, a_m_major, seed=M + 5 * N + K)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < RTOL, err


def test_tc_gemm_rejects_unaligned_strides(cuda):
    L = _lib()
    A = torch.zeros(625 * 64, device=cuda)
    B = torch.zeros(32 * 64, device=cuda)
    ws = torch.zeros(2 * 32 * 64, device=cuda)
    Cc = torch.zeros(625 * 32, device=cuda)
    # a K-major A with lda = 66 floats (not a 16-byte multiple): no TMA
    # descriptor and no row-wise form for this layout, so a clear error (an
    # M-major A with lda = 625 is loaded row by row and accepted)
    st = L.ppdl_gemm_tf32x3(64, 32, 64, 1, A.data_ptr(), 0, 66, 66 * 64, B.data_ptr(),
                            ws.data_ptr(), Cc.data_ptr(), 32, 1, 0,
                            torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_ERR_SHAPE
    assert "TMA" in ppdl.last_error()
    # K not a multiple of 4: rejected for both layouts
    st = L.ppdl_gemm_tf32x3(625, 32, 63, 1, A.data_ptr(), 1, 625, 625 * 64, B.data_ptr(),
                            ws.data_ptr(), Cc.data_ptr(), 1, 625, 0,
                            torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_ERR_SHAPE


def test_presplit_gemm_matches_one_call(cuda):
    """ppdl_tf32_split + ppdl_gemm_tf32x3_presplit (weights split once, as at
    model load) give the same bits as ppdl_gemm_tf32x3."""
    import ctypes as C
    L = _lib()
    L.ppdl_tf32_split.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]
    L.ppdl_gemm_tf32x3_presplit.argtypes = ([C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong,
                                            C.c_longlong, C.c_void_p, C.c_void_p]
                                            + [C.c_longlong] * 3 + [C.c_void_p])
    M, N, K, B = 2500, 192, 320, 2
    g = torch.Generator().manual_seed(5)
    A = torch.randn((B, K, M), generator=g).to(cuda)
    W = (torch.randn((N, K), generator=g) / K ** 0.5).to(cuda)
    ws1, ws2 = torch.empty(2 * N * K, device=cuda), torch.empty(2 * N * K, device=cuda)
    c1, c2 = torch.empty((B, N, M), device=cuda), torch.empty((B, N, M), device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert L.ppdl_gemm_tf32x3(M, N, K, B, A.data_ptr(), 1, M, K * M, W.data_ptr(), ws1.data_ptr(),
                              c1.data_ptr(), 1, M, N * M, s) == ppdl.PPDL_OK
    assert L.ppdl_tf32_split(W.data_ptr(), N * K, ws2.data_ptr(), s) == ppdl.PPDL_OK
    assert L.ppdl_gemm_tf32x3_presplit(M, N, K, B, A.data_ptr(), 1, M, K * M, ws2.data_ptr(),
                                       c2.data_ptr(), 1, M, N * M, s) == ppdl.PPDL_OK
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("M,N,K,splits,act,use_res", [(2400, 256, 2048, 3, 0, True),
                                                      (300, 256, 2048, 3, 0, True),
                                                      (517, 96, 1000, 4, 1, False),
                                                      (130, 40, 64, 2, 2, True)])
def test_split_k_matches_float64(cuda, M, N, K, splits, act, use_res):
    """ppdl_gemm_tf32x3_split_k (the forward's path for the decoder's
    2048 -> 256 linear): K in `splits` ranges summed in order, then bias,
    activation and residual; against float64, and the same per-row result
    at 2400 and 300 rows (the split depends on K only)."""
    import ctypes as C
    L = ppdl.lib()
    L.ppdl_tf32_split.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]
    L.ppdl_gemm_tf32x3_split_k.argtypes = ([C.c_int] * 3 + [C.c_void_p, C.c_longlong]
                                           + [C.c_void_p] * 3 + [C.c_int, C.c_int]
                                           + [C.c_void_p] * 3)
    g = torch.Generator(device=cuda).manual_seed(M + K)
    A = torch.randn((M, K), generator=g, device=cuda)
    W = torch.randn((N, K), generator=g, device=cuda) / K ** 0.5
    b = torch.randn((N,), generator=g, device=cuda) * 0.1
    R = torch.randn((M, N), generator=g, device=cuda) if use_res else None
    ws = torch.empty(2 * N * K, device=cuda)
    work = torch.empty(splits * M * N, device=cuda)
    out = torch.full((M, N), float("nan"), device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert L.ppdl_tf32_split(W.data_ptr(), N * K, ws.data_ptr(), s) == 0
    st = L.ppdl_gemm_tf32x3_split_k(M, N, K, A.data_ptr(), K, ws.data_ptr(), b.data_ptr(),
                                    R.data_ptr() if use_res else None, act, splits,
                                    work.data_ptr(), out.data_ptr(), s)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    ref = A.double() @ W.double().T + b.double()
    if act == 1:
        ref = torch.relu(ref)
    elif act == 2:
        ref = ref * torch.sigmoid(ref)
    if use_res:
        ref = ref + R.double()
    err = float((out.double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-6, err
    if M == 2400:
        # the first 300 rows alone give the same bits
        out2 = torch.empty((300, N), device=cuda)
        work2 = torch.empty(splits * 300 * N, device=cuda)
        assert L.ppdl_gemm_tf32x3_split_k(300, N, K, A.data_ptr(), K, ws.data_ptr(), b.data_ptr(),
                                          R.data_ptr() if use_res else None, act, splits,
                                          work2.data_ptr(), out2.data_ptr(), s) == 0
        torch.cuda.synchronize()
        assert torch.equal(out2, out[:300])
