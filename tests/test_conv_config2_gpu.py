"""Config 2 of the baseline (the conv sweep, B in {1, 8}) through the C ABI
entry points that run the forward's conv kernels, against a float64 conv of
the same data computed on the GPU (cuDNN, double precision).

  3x3 stride-1 (Winograd F(4,3): input transform, 36-plane 3xTF32 GEMM,
  output transform): ppdl_conv3x3_wg4_tf32x3 at 200^2 x 128 -> 128,
  100^2 x 256 -> 256, 50^2 x 512 -> 512, 25^2 x 1024 -> 1024;
  1x1 (3xTF32 GEMM writing CHW): ppdl_gemm_tf32x3 at 100^2 x 512 -> 256,
  50^2 x 1024 -> 256, 25^2 x 2048 -> 256 (the 625-pixel planes load one
  TMA row per channel).
The k3-s2 shapes of config 2 are in test_conv_tc_gpu.py.  Data as the
baseline states: activations N(0, 1), Kaiming weights, bias N(0, 0.1),
ReLU.  Gate: max|diff| / max|ref| <= 1e-5.
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
    L.ppdl_conv3x3_wg4_tf32x3.argtypes = (
        [C.c_void_p] + [C.c_int] * 4 + [C.c_longlong, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p])
    L.ppdl_conv3x3_wg4_tf32x3.restype = C.c_int
    L.ppdl_conv3x3_wg4_workspace.argtypes = [C.c_int] * 5
    L.ppdl_conv3x3_wg4_workspace.restype = C.c_longlong
    L.ppdl_gemm_tf32x3.argtypes = ([C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong,
                                   C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p]
                                   + [C.c_longlong] * 3 + [C.c_void_p])
    L.ppdl_gemm_tf32x3.restype = C.c_int
    return L


def _data(cuda, B, IC, H, W, OC, K, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    x = torch.randn((B, IC, H, W), generator=g, device=cuda)
    w = torch.randn((OC, IC, K, K), generator=g, device=cuda) * (2.0 / (IC * K * K)) ** 0.5
    b = torch.randn((OC,), generator=g, device=cuda) * 0.1
    return x, w, b


def _check(got, want):
    got = got.double()
    assert torch.isfinite(got).all()
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err <= RTOL, err


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("IC,HW", [(128, 200), (256, 100), (512, 50), (1024, 25)])
def test_conv3x3_winograd_config2(cuda, B, IC, HW):
    L = _lib()
    OC = IC
    x, w, b = _data(cuda, B, IC, HW, HW, OC, 3, seed=IC * 10 + B)
    work = torch.empty(L.ppdl_conv3x3_wg4_workspace(B, IC, OC, HW, HW), device=cuda)
    y = torch.full((B, OC, HW, HW), float("nan"), device=cuda)
    st = L.ppdl_conv3x3_wg4_tf32x3(x.data_ptr(), B, IC, HW, HW, IC * HW * HW, w.data_ptr(),
                                   b.data_ptr(), OC, 1, work.data_ptr(), y.data_ptr(),
                                   OC * HW * HW, torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    want = torch.relu(F.conv2d(x.double(), w.double(), b.double(), padding=1))
    torch.cuda.synchronize()
    _check(y, want)


@pytest.mark.parametrize("B", [1, 8])
@pytest.mark.parametrize("IC,HW", [(512, 100), (1024, 50), (2048, 25)])
def test_conv1x1_config2(cuda, B, IC, HW):
    L = _lib()
    OC, M = 256, HW * HW
    x, w, _ = _data(cuda, B, IC, HW, HW, OC, 1, seed=IC * 10 + B + 1)
    ws = torch.empty(2 * OC * IC, device=cuda)
    y = torch.full((B, OC, HW, HW), float("nan"), device=cuda)
    st = L.ppdl_gemm_tf32x3(M, OC, IC, B, x.data_ptr(), 1, M, IC * M, w.data_ptr(),
                            ws.data_ptr(), y.data_ptr(), 1, M, OC * M,
                            torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    want = F.conv2d(x.double(), w.double())
    torch.cuda.synchronize()
    _check(y, want)


def test_conv3x3_winograd_rejects_bad_arguments(cuda):
    L = _lib()
    x = torch.zeros((1, 6, 8, 8), device=cuda)
    w = torch.zeros((4, 6, 3, 3), device=cuda)
    y = torch.zeros((1, 4, 8, 8), device=cuda)
    work = torch.zeros(L.ppdl_conv3x3_wg4_workspace(1, 8, 4, 8, 8), device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    # IC = 6 is not a multiple of 4
    assert L.ppdl_conv3x3_wg4_tf32x3(x.data_ptr(), 1, 6, 8, 8, 384, w.data_ptr(), None, 4, 0,
                                     work.data_ptr(), y.data_ptr(), 256, s) == ppdl.PPDL_ERR_SHAPE
    assert "conv3x3" in ppdl.last_error()
    assert L.ppdl_conv3x3_wg4_workspace(0, 8, 4, 8, 8) == 0
