"""ppdl_conv2d_tf32x3 — direct convolution on the tensor-core GEMM with no
im2col buffer, the path of the forward's k3-s2 and k2 convs: the A operand
comes from TMA windows of the CHW input when its rows are 16-byte multiples
(W % 4 == 0), else from the converter warps' gather.

Checked against a float64 torch conv2d of the same seeded data (on the
CPU, or on the GPU in float64 for the config-2 sizes), under the
tensor-core GEMM tests' gate max|diff| / max|ref| <= 1e-5.  The cases cover
the reference's conv shapes of this kind (stem1: IC=3; stem2a/b: k2 with
padding only at the bottom/right; stem3; pand0/pand1: k3-s2 with 256
channels; the 625-pixel 1x1 convs), both A paths, output widths that are
and are not multiples of 4 (TMA or direct stores), channel tails, page
batches, more tiles than SMs, and the baseline's config-2 stride-2 shapes
at B = 1 and 8.  ppdl_gemm_tf32x3 on 25 x 25 CHW planes (one TMA row per
channel) is checked the same way.
"""
import ctypes as C

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import ppdl

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _lib():
    L = ppdl.lib()
    L.ppdl_conv2d_tf32x3.argtypes = (
        [C.c_void_p] + [C.c_int] * 4 + [C.c_longlong, C.c_void_p, C.c_void_p]
        + [C.c_int] * 7 + [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p])
    L.ppdl_conv2d_tf32x3.restype = C.c_int
    L.ppdl_conv2d_tf32x3_workspace.argtypes = [C.c_int] * 3
    L.ppdl_conv2d_tf32x3_workspace.restype = C.c_longlong
    return L


def _ref(x, w, b, S, P, OH, OW, act):
    # zero padding P at the top/left, whatever the bottom/right needs for OH x OW
    K = w.shape[-1]
    H, W = x.shape[-2:]
    pb = max(0, (OH - 1) * S + K - H - P)
    pr = max(0, (OW - 1) * S + K - W - P)
    xp = F.pad(x.double(), (P, pr, P, pb))
    y = F.conv2d(xp, w.double(), b.double(), stride=S)[:, :, :OH, :OW]
    if act == 1:
        y = torch.relu(y)
    elif act == 2:
        y = y * torch.sigmoid(y)
    return y


def _run(L, cuda, B, IC, H, W, OC, K, S, P, act, OH=None, OW=None, seed=0, ref_on_gpu=False):
    OH = OH or (H + 2 * P - K) // S + 1
    OW = OW or (W + 2 * P - K) // S + 1
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B, IC, H, W), generator=g)
    w = torch.randn((OC, IC, K, K), generator=g) / (IC * K * K) ** 0.5
    b = torch.randn((OC,), generator=g) * 0.1
    dx, dw, db = x.to(cuda), w.to(cuda), b.to(cuda)
    ws = torch.empty(L.ppdl_conv2d_tf32x3_workspace(IC, OC, K), device=cuda)
    y = torch.full((B, OC, OH, OW), float("nan"), device=cuda)
    st = L.ppdl_conv2d_tf32x3(dx.data_ptr(), B, IC, H, W, IC * H * W, dw.data_ptr(),
                              db.data_ptr(), OC, K, S, P, OH, OW, act, ws.data_ptr(),
                              y.data_ptr(), OC * OH * OW,
                              torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    if ref_on_gpu:
        want = _ref(dx, dw, db, S, P, OH, OW, act).cpu().numpy()
    else:
        want = _ref(x, w, b, S, P, OH, OW, act).numpy()
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= RTOL, err
    return err


@pytest.mark.parametrize("case", [
    # B, IC, H, W, OC, K, S, P, act, OH, OW          (model layer it stands for)
    (2, 3, 67, 67, 32, 3, 2, 1, 1, None, None),     # stem1 (K = 27 -> 28)
    (2, 32, 50, 50, 16, 2, 1, 0, 1, 50, 50),        # stem2a: k2, pad (0, 1)
    (2, 16, 50, 50, 32, 2, 1, 0, 1, 50, 50),        # stem2b
    (2, 64, 41, 41, 96, 3, 2, 1, 1, None, None),    # stem3 (odd size, N tail)
    (2, 256, 100, 100, 256, 3, 2, 1, 2, None, None),  # pand0 (tiles > SMs)
    (3, 256, 50, 50, 256, 3, 2, 1, 2, None, None),  # pand1
    (3, 100, 25, 25, 256, 1, 1, 0, 0, None, None),  # 625-pixel 1x1 (K tail)
    (2, 13, 25, 25, 40, 1, 1, 0, 1, None, None),    # 1x1, K = 13 -> 16
    (1, 8, 9, 7, 24, 3, 1, 1, 2, None, None),       # tiny k3-s1 (one tile)
    # TMA windows of the input (W % 4 == 0)
    (2, 3, 68, 68, 32, 3, 2, 1, 1, None, None),     # stem1: 3 of 32 window channels
    (2, 32, 52, 52, 16, 2, 1, 0, 1, 52, 52),        # stem2a: k2, pad (0, 1)
    (2, 16, 52, 52, 32, 2, 1, 0, 1, 52, 52),        # stem2b: 16 of 32 channels
    (2, 64, 40, 40, 96, 3, 2, 1, 1, None, None),    # stem3 (N tail)
    (2, 256, 100, 100, 256, 3, 2, 1, 2, None, None),  # pand0 (OW 50: direct stores)
    (1, 40, 36, 36, 48, 3, 2, 1, 0, None, None),    # channel tail 40 = 32 + 8, OW 18
    (2, 32, 64, 96, 64, 3, 1, 1, 1, None, None),    # k3-s1 window (P = 1, 4 rows)
    (3, 64, 132, 128, 40, 2, 1, 0, 2, 132, 128),    # row tiles past H, 3 pages
    (2, 8, 36, 36, 24, 3, 2, 1, 1, None, None),     # 8-channel windows, 3 columns per k-block
    (1, 12, 44, 44, 20, 2, 1, 0, 2, 44, 44),        # 16-channel windows (12 real)
])
def test_conv2d_gather_matches_float64(cuda, case):
    B, IC, H, W, OC, K, S, P, act, OH, OW = case
    _run(_lib(), cuda, B, IC, H, W, OC, K, S, P, act, OH, OW, seed=IC * 7 + OC)


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("case", [
    # config 2: k3-s2 200x200x128 -> 256 and 100x100x512 -> 512
    (128, 200, 200, 256),
    (512, 100, 100, 512),
])
def test_conv2d_config2_stride2_matches_float64(cuda, B, case):
    IC, H, W, OC = case
    _run(_lib(), cuda, B, IC, H, W, OC, 3, 2, 1, 1, seed=IC + B, ref_on_gpu=True)


@pytest.mark.parametrize("B,IC,OC,HW", [(2, 1024, 256, 25), (1, 2048, 256, 25),
                                        (3, 64, 96, 13)])
def test_gemm_on_unaligned_planes_matches_float64(cuda, B, IC, OC, HW):
    """ppdl_gemm_tf32x3 with an M-major A of 25 x 25 (13 x 13) CHW planes:
    lda = 625 (169) is no 16-byte multiple, so each k is one TMA row."""
    L = ppdl.lib()
    L.ppdl_gemm_tf32x3.argtypes = ([C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong,
                                   C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p]
                                   + [C.c_longlong] * 3 + [C.c_void_p])
    M = HW * HW
    g = torch.Generator().manual_seed(B * 100 + IC)
    x = torch.randn((B, IC, M), generator=g)
    w = torch.randn((OC, IC), generator=g) / IC ** 0.5
    dx, dw = x.to(cuda), w.to(cuda)
    ws = torch.empty(2 * OC * IC, device=cuda)
    y = torch.full((B, OC, M), float("nan"), device=cuda)
    st = L.ppdl_gemm_tf32x3(M, OC, IC, B, dx.data_ptr(), 1, M, IC * M, dw.data_ptr(),
                            ws.data_ptr(), y.data_ptr(), 1, M, OC * M,
                            torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    want = torch.einsum("nk,bkm->bnm", w.double(), x.double()).numpy()
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() / np.abs(want).max() <= RTOL


def test_conv2d_gather_rejects_bad_geometry(cuda):
    L = _lib()
    x = torch.zeros((1, 4, 8, 8), device=cuda)
    w = torch.zeros((8, 4, 3, 3), device=cuda)
    ws = torch.zeros(L.ppdl_conv2d_tf32x3_workspace(4, 8, 3), device=cuda)
    y = torch.zeros((1, 8, 8, 8), device=cuda)
    s = torch.cuda.current_stream().cuda_stream

    def call(K, S, P, OH, OW):
        return L.ppdl_conv2d_tf32x3(x.data_ptr(), 1, 4, 8, 8, 256, w.data_ptr(), None, 8, K, S,
                                    P, OH, OW, 0, ws.data_ptr(), y.data_ptr(), 512, s)

    assert call(3, 1, 3, 8, 8) == ppdl.PPDL_ERR_SHAPE      # P >= K
    assert call(1, 2, 0, 4, 4) == ppdl.PPDL_ERR_SHAPE      # strided 1x1
    assert call(3, 1, 1, 10, 8) == ppdl.PPDL_ERR_SHAPE     # window starts past the input
    assert "conv2d" in ppdl.last_error()
