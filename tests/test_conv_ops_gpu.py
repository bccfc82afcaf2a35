"""CUDA parity of the conv family through the operator C ABI (op ids 3, 4,
10, 11, 12 of include/ppdl_ops.h) against the CPU oracle.

The oracle's direct conv accumulates in double, so it is an
algorithm-independent reference for the GEMM, implicit-GEMM and Winograd
paths; the Winograd stages are additionally compared stage by stage with the
oracle's restatement of the reference transforms.  Ops 3 and 12 run on the
3xTF32 tensor-core GEMM (weights split into the library's static array in
chunks; cases below exceed one chunk), op 12 with IC not a multiple of 4
on the SIMT GEMM.  Gate: the hot path's
per-op FP32 relative error, max|diff| / max|ref| <= 1e-5.
"""
import numpy as np
import pytest
import torch

import ppdl

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _wr(w):
    """torch-order weight [OC][IC][K][K] -> the reference's .wr (K*K, IC, OC)
    row-major (src/ppdoclayout.cpp:273-280)."""
    OC, IC, K, _ = w.shape
    return np.ascontiguousarray(w.transpose(2, 3, 1, 0).reshape(K * K, IC, OC))


@pytest.mark.parametrize("B,IC,OC,H,W", [(1, 48, 64, 25, 25), (2, 37, 19, 13, 11),
                                          (1, 512, 256, 50, 50),
                                          # 3.1M weights > the 2^21 split array: N chunks
                                          (2, 2048, 1536, 13, 13)])
def test_op3_conv1x1(cuda, orc, B, IC, OC, H, W):
    rng = np.random.default_rng(B * 1000 + IC)
    x = rng.standard_normal((B, IC, H, W), dtype=np.float32)
    w = (rng.standard_normal((OC, IC, 1, 1)) / np.sqrt(IC)).astype(np.float32)
    y = torch.empty((B, OC, H, W), device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_CONV, y, [_t(x, cuda), _t(_wr(w), cuda)], params=[1, 0]))
    torch.cuda.synchronize()
    zb = np.zeros(OC, np.float32)
    for b in range(B):
        ref = orc.conv2d(x[b], w, zb, 1, 0)
        assert rel_err(y[b].cpu().numpy(), ref) < RTOL


@pytest.mark.parametrize("K,S,P,act", [(3, 2, 1, 1), (2, 1, 0, 1), (3, 1, 1, 2), (1, 1, 0, 0),
                                       (3, 2, 1, 0)])
def test_op4_direct_conv(cuda, orc, K, S, P, act):
    rng = np.random.default_rng(K * 100 + S * 10 + act)
    B, IC, OC, H, W = 2, 19, 23, 17, 14
    x = rng.standard_normal((B, IC, H, W), dtype=np.float32)
    w = (rng.standard_normal((OC, IC, K, K)) / np.sqrt(IC * K * K)).astype(np.float32)
    b = (0.1 * rng.standard_normal(OC)).astype(np.float32)
    OH, OW = (H + 2 * P - K) // S + 1, (W + 2 * P - K) // S + 1
    y = torch.empty((B, OC, OH, OW), device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_CONVDIRECT, y, [_t(x, cuda), _t(_wr(w), cuda), _t(b, cuda)],
                              params=[K | (S << 8) | (P << 16) | (act << 24)]))
    torch.cuda.synchronize()
    for i in range(B):
        ref = orc.conv2d(x[i], w, b, S, P, act=act)
        assert rel_err(y[i].cpu().numpy(), ref) < RTOL


def _winograd_ops(cuda, xp_b, wg4, bias, TW, TH, OW, OH, act):
    """op 10 -> op 12 -> op 11 on device, returning every stage."""
    B, IC = xp_b.shape[0], xp_b.shape[1]
    OC, T = wg4.shape[2], TW * TH
    dt = torch.empty((B, 36, IC, T), device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_WG4_INPUT, dt, [_t(xp_b, cuda)], params=[T, TH]))
    yt = torch.empty((B, 36, OC, T), device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_WG4_MADD, yt, [dt, _t(wg4, cuda)]))
    y = torch.empty((B, OC, OH, OW), device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_WG4_OUTPUT, y, [yt, _t(bias, cuda)], params=[act, TW]))
    torch.cuda.synchronize()
    return dt.cpu().numpy(), yt.cpu().numpy(), y.cpu().numpy()


def test_winograd_known_answer_f43(cuda, orc):
    """bench/wg_test.cu:89-167 re-targeted to F(4,3), through ops 10/12/11."""
    IW, IH, IC, OC = 10, 9, 3, 2
    TW, TH = (IW + 3) // 4, (IH + 3) // 4
    IWp, IHp = 4 * TW + 2, 4 * TH + 2
    i = np.arange(IWp * IHp * IC, dtype=np.float32)
    xp = (np.sin(np.float32(0.7) * i) * np.float32(0.5)).astype(np.float32).reshape(IC, IHp, IWp)
    j = np.arange(9 * IC * OC, dtype=np.float32)
    w = (np.cos(np.float32(0.3) * j) * np.float32(0.4)).astype(np.float32).reshape(OC, IC, 3, 3)
    b = (np.float32(0.1) * np.arange(OC, dtype=np.float32)).astype(np.float32)
    ref = np.zeros((OC, IH, IW))
    for oc in range(OC):
        for y in range(IH):
            for x in range(IW):
                ref[oc, y, x] = b[oc] + np.sum(xp[:, y:y + 3, x:x + 3].astype(np.float64) * w[oc])
    wg4 = orc.wg4_filter(w)
    _, _, got = _winograd_ops(cuda, xp[None], wg4, b, TW, TH, IW, IH, 0)
    assert rel_err(got[0], ref) < RTOL


@pytest.mark.parametrize("H,W,IC,OC,act", [(25, 25, 64, 64, 2), (50, 50, 48, 48, 1),
                                           (13, 11, 7, 5, 0), (100, 100, 128, 96, 1),
                                           # 36 x 256 x 256 > the 2^21 split array: plane chunks
                                           (25, 25, 256, 256, 1)])
def test_winograd_stages_vs_oracle(cuda, orc, H, W, IC, OC, act):
    rng = np.random.default_rng(H * W + IC)
    B = 2
    x = rng.standard_normal((B, IC, H, W), dtype=np.float32)
    w = (rng.standard_normal((OC, IC, 3, 3)) * np.sqrt(2.0 / (9 * IC))).astype(np.float32)
    b = (0.1 * rng.standard_normal(OC)).astype(np.float32)
    TW, TH = (W + 3) // 4, (H + 3) // 4
    xp = np.zeros((B, IC, 4 * TH + 2, 4 * TW + 2), np.float32)
    xp[:, :, 1:H + 1, 1:W + 1] = x
    wg4 = orc.wg4_filter(w)
    dt, yt, y = _winograd_ops(cuda, xp, wg4, b, TW, TH, W, H, act)
    for i in range(B):
        dt_ref = orc.wg4_input(xp[i], TW, TH)
        assert rel_err(dt[i], dt_ref) < 1e-6
        yt_ref = orc.wg4_madd(dt_ref, wg4)
        assert rel_err(yt[i], yt_ref) < RTOL
        assert rel_err(y[i], orc.conv2d(x[i], w, b, 1, 1, act=act)) < RTOL


def test_conv_op_errors(cuda):
    x = torch.zeros((1, 4, 8, 8), device=cuda)
    y = torch.zeros((1, 5, 8, 8), device=cuda)
    w = torch.zeros((9, 4, 5), device=cuda)
    # legacy K==3 channel-last form of op 3 is not provided
    assert ppdl.op_launch(ppdl.OP_CONV, y, [x, w], params=[3 | (1 << 8), 1]) == \
        ppdl.PPDL_ERR_UNSUPPORTED
    # op 4 with a (K,S,PAD) the reference does not accept
    assert ppdl.op_launch(ppdl.OP_CONVDIRECT, y, [x, w, torch.zeros(5, device=cuda)],
                          params=[5 | (1 << 8) | (2 << 16)]) == ppdl.PPDL_ERR_SHAPE
    # op 10 with a tile grid larger than the padded input
    dt = torch.zeros((1, 36, 4, 16), device=cuda)
    assert ppdl.op_launch(ppdl.OP_WG4_INPUT, dt, [x], params=[16, 4]) == ppdl.PPDL_ERR_SHAPE
