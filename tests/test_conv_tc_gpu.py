"""ppdl_conv2d_tf32x3 — direct convolution on the tensor-core GEMM with the
A tile gathered from the CHW input (the forward's k3-s2 and k2 convs and
its 1x1 convs on 25x25 planes run through this kernel).

Checked against a float64 torch conv2d on the CPU of the same seeded data,
under the tensor-core GEMM tests' gate max|diff| / max|ref| <= 1e-5.  The
cases cover the reference's conv shapes of this kind (stem1: IC=3, so
IC*K*K = 27 is padded to 28; stem2a/b: k2 with padding only at the
bottom/right; pand0/pand1: k3-s2 with 256 channels; the 625-pixel 1x1
convs), K tails, N tails, page batches and more tiles than SMs.
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


def _run(L, cuda, B, IC, H, W, OC, K, S, P, act, OH=None, OW=None, seed=0):
    OH = OH or (H + 2 * P - K) // S + 1
    OW = OW or (W + 2 * P - K) // S + 1
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B, IC, H, W), generator=g)
    w = torch.randn((OC, IC, K, K), generator=g) / (IC * K * K) ** 0.5
    b = torch.randn((OC,), generator=g) * 0.1
    kp = (IC * K * K + 3) // 4 * 4
    dx, dw, db = x.to(cuda), w.to(cuda), b.to(cuda)
    ws = torch.empty(2 * OC * kp, device=cuda)
    y = torch.full((B, OC, OH, OW), float("nan"), device=cuda)
    st = L.ppdl_conv2d_tf32x3(dx.data_ptr(), B, IC, H, W, IC * H * W, dw.data_ptr(),
                              db.data_ptr(), OC, K, S, P, OH, OW, act, ws.data_ptr(),
                              y.data_ptr(), OC * OH * OW,
                              torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
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
])
def test_conv2d_gather_matches_float64(cuda, case):
    B, IC, H, W, OC, K, S, P, act, OH, OW = case
    _run(_lib(), cuda, B, IC, H, W, OC, K, S, P, act, OH, OW, seed=IC * 7 + OC)


def test_conv2d_gather_rejects_bad_geometry(cuda):
    L = _lib()
    x = torch.zeros((1, 4, 8, 8), device=cuda)
    w = torch.zeros((8, 4, 3, 3), device=cuda)
    ws = torch.zeros(2 * 8 * 36, device=cuda)
    y = torch.zeros((1, 8, 8, 8), device=cuda)
    s = torch.cuda.current_stream().cuda_stream

    def call(K, S, P, OH, OW):
        return L.ppdl_conv2d_tf32x3(x.data_ptr(), 1, 4, 8, 8, 256, w.data_ptr(), None, 8, K, S,
                                    P, OH, OW, 0, ws.data_ptr(), y.data_ptr(), 512, s)

    assert call(3, 1, 3, 8, 8) == ppdl.PPDL_ERR_SHAPE      # P >= K
    assert call(1, 2, 0, 4, 4) == ppdl.PPDL_ERR_SHAPE      # strided 1x1
    assert call(3, 1, 1, 10, 8) == ppdl.PPDL_ERR_SHAPE     # window starts past the input
    assert "conv2d" in ppdl.last_error()
