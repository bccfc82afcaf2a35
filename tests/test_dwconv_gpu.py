"""ppdl_depthwise_conv2d — the backbone's depthwise convs (ggml_conv_2d_dw_direct,
src/ppdoclayout.cpp:400-404): the stride-2 downsamples (K3, P1) and the 5x5
light-block convs (K5, P2).

Checked against a float64 torch grouped conv2d on the CPU of the same seeded
data.  The kernel accumulates K*K FP32 fmas per output, so the gate is
max|diff| / max|ref| <= 1e-6.  The cases cover the model's plane sizes
(200 -> 100, 100 -> 50, 50 -> 25 and 50x50 / 25x25 stride 1), the three
forms (whole plane in shared memory; bands of output rows for larger planes,
with a shorter last band; 32x32 tiles for rows too wide for a band, with
tiles cut by the plane edges), page batches, a NULL bias and every
activation.
"""
import ctypes as C

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import ppdl

pytestmark = pytest.mark.gpu

RTOL = 1e-6


def _lib():
    L = ppdl.lib()
    L.ppdl_depthwise_conv2d.argtypes = (
        [C.c_void_p] + [C.c_int] * 4 + [C.c_longlong, C.c_void_p, C.c_void_p]
        + [C.c_int] * 4 + [C.c_void_p, C.c_longlong, C.c_void_p])
    L.ppdl_depthwise_conv2d.restype = C.c_int
    return L


def _ref(x, w, b, S, P, act):
    y = F.conv2d(x.double(), w.double().unsqueeze(1), None if b is None else b.double(),
                 stride=S, padding=P, groups=x.shape[1])
    if act == 1:
        y = torch.relu(y)
    elif act == 2:
        y = y * torch.sigmoid(y)
    elif act == 3:
        y = 0.5 * y * (1 + torch.erf(y / 2 ** 0.5))
    return y


@pytest.mark.parametrize("case", [
    # B, C, H, W, K, S, P, act, bias     (model layer it stands for)
    (2, 16, 200, 200, 3, 2, 1, 0, True),   # st1.ds (128 ch at 200x200 in the model), bands
    (2, 32, 100, 100, 3, 2, 1, 0, True),   # st2.ds
    (3, 64, 50, 50, 3, 2, 1, 0, True),     # st3.ds
    (2, 48, 50, 50, 5, 1, 2, 0, True),     # st2 light blocks, 5x5
    (2, 64, 25, 25, 5, 1, 2, 0, True),     # st3 light blocks, 5x5
    (1, 8, 37, 45, 3, 1, 1, 1, True),      # odd sizes, ReLU
    (1, 8, 41, 33, 5, 2, 2, 2, False),     # 5x5 stride 2, SiLU, no bias
    (1, 4, 70, 70, 3, 1, 1, 3, True),      # GELU
    (1, 4, 150, 130, 3, 1, 1, 1, True),    # 5 bands of 30 rows
    (1, 3, 257, 300, 5, 1, 2, 3, True),    # 18 bands, 5x5, odd height
    (1, 3, 203, 191, 5, 2, 2, 0, False),   # bands, 5x5 stride 2
    (2, 5, 51, 47, 5, 1, 2, 1, True),      # odd W: 4-byte copies, scalar stores
    (1, 6, 30, 30, 3, 2, 1, 2, True),      # odd P (4-byte copies), SiLU
    (1, 2, 20, 1300, 5, 1, 2, 0, True),    # tiled form: 5 rows of 1300 exceed a band buffer
    (2, 2, 9, 2100, 3, 2, 1, 1, True),     # tiled form, stride 2, edge tiles
])
def test_depthwise_matches_float64(cuda, case):
    B, Cc, H, W, K, S, P, act, with_bias = case
    g = torch.Generator().manual_seed(Cc * 31 + H)
    x = torch.randn((B, Cc, H, W), generator=g)
    w = torch.randn((Cc, K, K), generator=g) / K
    b = torch.randn((Cc,), generator=g) * 0.1 if with_bias else None
    OH, OW = (H + 2 * P - K) // S + 1, (W + 2 * P - K) // S + 1
    dx, dw = x.to(cuda), w.to(cuda)
    db = b.to(cuda) if with_bias else None
    y = torch.full((B, Cc, OH, OW), float("nan"), device=cuda)
    L = _lib()
    st = L.ppdl_depthwise_conv2d(dx.data_ptr(), B, Cc, H, W, Cc * H * W, dw.data_ptr(),
                                 db.data_ptr() if with_bias else None, K, S, P, act,
                                 y.data_ptr(), Cc * OH * OW,
                                 torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    want = _ref(x, w, b, S, P, act).numpy()
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= RTOL, err


def test_depthwise_rejects_unsupported(cuda):
    L = _lib()
    x = torch.zeros((1, 2, 8, 8), device=cuda)
    w = torch.zeros((2, 7, 7), device=cuda)
    y = torch.zeros((1, 2, 8, 8), device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    assert L.ppdl_depthwise_conv2d(x.data_ptr(), 1, 2, 8, 8, 128, w.data_ptr(), None, 7, 1, 3, 0,
                                   y.data_ptr(), 128, s) == ppdl.PPDL_ERR_UNSUPPORTED
    assert L.ppdl_depthwise_conv2d(x.data_ptr(), 1, 2, 8, 8, 128, w.data_ptr(), None, 3, 1, 3, 0,
                                   y.data_ptr(), 128, s) == ppdl.PPDL_ERR_SHAPE  # P >= K
