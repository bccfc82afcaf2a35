"""ppdl_conv2d_direct — the direct FP32 convolution the forward uses for the
stem's narrow convs (src/ppdoclayout.cpp:618-631: stem1 3 -> 32 k3-s2-p1,
stem2a 32 -> 16 and stem2b 16 -> 32 k2 with padding (0, 1) from ggml_pad).

Checked against a float64 torch conv2d on the CPU of the same seeded data,
with the bottom/right zero padding that OH / OW imply.  Each output sums at
most 128 FP32 fmas, so the gate is max|diff| / max|ref| <= 1e-6.  The cases
cover the stem's three shapes at two pages, channel counts that leave part
of a 16-channel group unused, edge tiles, every activation, a NULL
bias, and the shapes outside the narrow form (rejected, not computed).
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
    L.ppdl_conv2d_direct.argtypes = (
        [C.c_void_p] + [C.c_int] * 4 + [C.c_longlong, C.c_void_p, C.c_void_p]
        + [C.c_int] * 7 + [C.c_void_p, C.c_longlong, C.c_void_p])
    L.ppdl_conv2d_direct.restype = C.c_int
    return L


def _ref(x, w, b, S, P, OH, OW, act):
    K = w.shape[-1]
    H, W = x.shape[-2:]
    pb = max(0, (OH - 1) * S + K - P - H)
    pr = max(0, (OW - 1) * S + K - P - W)
    xp = F.pad(x.double(), (P, pr, P, pb))
    y = F.conv2d(xp, w.double(), None if b is None else b.double(), stride=S)[:, :, :OH, :OW]
    if act == 1:
        y = torch.relu(y)
    elif act == 2:
        y = y * torch.sigmoid(y)
    elif act == 3:
        y = 0.5 * y * (1 + torch.erf(y / 2 ** 0.5))
    return y


def _run(cuda, B, IC, H, W, OC, K, S, P, OH, OW, act, with_bias, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B, IC, H, W), generator=g)
    w = torch.randn((OC, IC, K, K), generator=g) / (IC * K * K) ** 0.5
    b = torch.randn((OC,), generator=g) * 0.1 if with_bias else None
    dx, dw = x.to(cuda), w.to(cuda)
    db = b.to(cuda) if with_bias else None
    y = torch.full((B, OC, OH, OW), float("nan"), device=cuda)
    st = _lib().ppdl_conv2d_direct(dx.data_ptr(), B, IC, H, W, IC * H * W, dw.data_ptr(),
                                   db.data_ptr() if with_bias else None, OC, K, S, P, OH, OW,
                                   act, y.data_ptr(), OC * OH * OW,
                                   torch.cuda.current_stream().cuda_stream)
    return st, x, w, b, y


@pytest.mark.parametrize("case", [
    # B, IC, H, W, OC, K, S, P, OH, OW, act, bias    (layer it stands for)
    (2, 3, 800, 800, 32, 3, 2, 1, 400, 400, 1, True),   # stem1
    (2, 32, 400, 400, 16, 2, 1, 0, 400, 400, 1, True),  # stem2a, padding (0, 1)
    (2, 16, 400, 400, 32, 2, 1, 0, 400, 400, 1, True),  # stem2b
    (1, 5, 37, 61, 20, 3, 1, 1, 37, 61, 2, False),      # 20 channels: 4 of the second group, SiLU
    (3, 7, 45, 33, 9, 2, 2, 1, 23, 17, 3, True),        # 9 of 16 channels, k2-s2, GELU
    (1, 14, 19, 70, 32, 3, 2, 0, 9, 34, 0, True),       # IC*K*K = 126, no activation
])
def test_direct_matches_float64(cuda, case):
    B, IC, H, W, OC, K, S, P, OH, OW, act, with_bias = case
    st, x, w, b, y = _run(cuda, B, IC, H, W, OC, K, S, P, OH, OW, act, with_bias, IC * 7 + H)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    want = _ref(x, w, b, S, P, OH, OW, act).numpy()
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= RTOL, err


def test_direct_rejects_wide_convs(cuda):
    # 33 output channels, 144 products per output, K = 5: not the narrow form
    for OC, IC, K in ((33, 3, 3), (16, 16, 3), (8, 1, 5)):
        st, *_ = _run(cuda, 1, IC, 16, 16, OC, K, 1, 1, 16 - K + 3, 16 - K + 3, 0, True, 1)
        assert st == ppdl.PPDL_ERR_UNSUPPORTED, (OC, IC, K)
    st, *_ = _run(cuda, 1, 3, 16, 16, 8, 3, 1, 3, 16, 16, 0, True, 1)  # P >= K
    assert st == ppdl.PPDL_ERR_SHAPE
