"""ppdl_attention_f32 — the fused attention core of the forward (the
reference's ggml_mul_mat(k, q) -> ggml_scale -> ggml_soft_max ->
ggml_mul_mat(v) per head of 32 dims, src/ppdoclayout.cpp:572-587).

Checked against float64 torch on the CPU of the same seeded data: the
decoder's self-attention shape (T = 300, 8 heads, q|k stacked in rows of
512, v / o in rows of 256) at 8 pages with all keys in one tile (T <= 320),
AIFI's 625 tokens through 64-key tiles, and ragged lengths (the last 32-query block partly empty, T below one block, T not a
multiple of 4).  Gate: max|diff| <= 2e-6 on O(1) outputs (FP32 dot products
of 32 dims and sums over at most 625 keys).
"""
import ctypes as C

import numpy as np
import pytest
import torch

import ppdl

pytestmark = pytest.mark.gpu


def _lib():
    L = ppdl.lib()
    L.ppdl_attention_f32.argtypes = ([C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_longlong, C.c_int,
                                     C.c_longlong, C.c_float, C.c_void_p])
    L.ppdl_attention_f32.restype = C.c_int
    return L


@pytest.mark.parametrize("B,T,heads", [(8, 300, 8), (2, 625, 8), (3, 37, 8), (1, 5, 2),
                                       (2, 318, 4)])
def test_attention_matches_float64(cuda, B, T, heads):
    g = torch.Generator().manual_seed(T * 13 + heads)
    D = heads * 32
    qk = torch.randn((B, T, 2 * D), generator=g)  # q | k side by side, as the forward
    v = torch.randn((B, T, D), generator=g)
    dqk, dv = qk.to(cuda), v.to(cuda)
    o = torch.full((B, T, D), float("nan"), device=cuda)
    scale = 1.0 / np.sqrt(32.0)
    st = _lib().ppdl_attention_f32(dqk.data_ptr(), dqk.data_ptr() + 4 * D, dv.data_ptr(),
                                   o.data_ptr(), B, T, heads, 2 * D, T * 2 * D, D, T * D, scale,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_OK, ppdl.last_error()
    torch.cuda.synchronize()
    q = qk[..., :D].double().reshape(B, T, heads, 32).transpose(1, 2)
    k = qk[..., D:].double().reshape(B, T, heads, 32).transpose(1, 2)
    vv = v.double().reshape(B, T, heads, 32).transpose(1, 2)
    p = torch.softmax(q @ k.transpose(-1, -2) * scale, dim=-1)
    want = (p @ vv).transpose(1, 2).reshape(B, T, D).numpy()
    got = o.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - want).max() <= 2e-6, np.abs(got - want).max()


def test_attention_rejects_misaligned_rows(cuda):
    x = torch.zeros(4096, device=cuda)
    st = _lib().ppdl_attention_f32(x.data_ptr(), x.data_ptr() + 4, x.data_ptr(), x.data_ptr(), 1,
                                   10, 1, 66, 660, 32, 320, 0.1,
                                   torch.cuda.current_stream().cuda_stream)
    assert st == ppdl.PPDL_ERR_SHAPE
