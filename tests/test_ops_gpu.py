"""CUDA parity of the decoder / selection ops through the operator C ABI
(include/ppdl_ops.h, ppdl_op_launch), against the golden fixtures made by
the reference's own CPU ops and against the pinned oracle.

Tolerances: mask->box and top-300 are integer/index work and must be
bit-exact (top-300) or equal to 1 ulp of logf (mask->box); MSDA is f32
with the reference's tap order, so it is held to 1e-6 absolute on O(1)
data (the per-op gate of the hot path is 1e-5 relative).
"""
import numpy as np
import pytest
import torch

import cases
import ppdl

pytestmark = pytest.mark.gpu


def _dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _msda(cuda, val, off, awr, ref, B, nq, canon=False):
    out = torch.empty((B, nq, 256), dtype=torch.float32, device=cuda)
    srcs = [_dev(val, cuda), _dev(off, cuda), _dev(awr, cuda)]
    if not canon:
        srcs.append(_dev(ref, cuda))
    st = ppdl.op_launch(ppdl.OP_MSDEF, out, srcs, params=[1 if canon else 0],
                        dst_ne=[256, nq, B], src_ne=[[256, 13125, B], [192, nq, B], [96, nq, B],
                                                     [4, nq, B]])
    ppdl.check(st)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("seed", [11, 12])
def test_msdeform_vs_golden(cuda, golden_dir, seed):
    g = np.load(f"{golden_dir}/msdeform_s{seed}.npz")
    val, off, awr, ref = cases.msdeform_inputs(seed)
    assert cases.digest(val, off, awr, ref) == str(g["digest"])
    got = _msda(cuda, val, off, awr, ref, 1, 300)[0]
    np.testing.assert_allclose(got, g["out"], rtol=0, atol=1e-6)


def test_msdeform_batched_ragged_nq(cuda, orc):
    """B = 3 pages, nq = 37 (not a multiple of the 2-query block)."""
    rng = np.random.default_rng(7)
    B, nq = 3, 37
    val = rng.standard_normal((B, 13125, 256), dtype=np.float32)
    off = (rng.standard_normal((B, nq, 192), dtype=np.float32) * 3).astype(np.float32)
    awr = rng.standard_normal((B, nq, 96), dtype=np.float32)
    ref = rng.uniform(0, 1, (B, nq, 4)).astype(np.float32)
    got = _msda(cuda, val, off, awr, ref, B, nq)
    np.testing.assert_allclose(got, orc.msdeform(val, off, awr, ref), rtol=0, atol=1e-6)


def test_msdeform_canonical_config1(cuda, orc):
    """Config 1 form: value N(0,1), loc U[0,1], weights softmax(N(0,1))."""
    rng = np.random.default_rng(1)
    B, nq = 2, 300
    val = rng.standard_normal((B, 13125, 8, 32), dtype=np.float32)
    loc = rng.uniform(0, 1, (B, nq, 8, 3, 4, 2)).astype(np.float32)
    lg = rng.standard_normal((B, nq, 8, 12)).astype(np.float32)
    w = np.exp(lg - lg.max(-1, keepdims=True))
    w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
    got = _msda(cuda, val, loc.reshape(B, nq, 192), w.reshape(B, nq, 96), None, B, nq, canon=True)
    exp = orc.msdeform_canon(val, loc, w)
    np.testing.assert_allclose(got, exp, rtol=0, atol=1e-6)


def test_msdeform_canonical_config1_b32(cuda, orc):
    """Config 1 at the benchmarked size, B = 32 pages (bench.py's msda
    workload recipe: value N(0,1), loc U[0,1], weights softmax(N(0,1)))."""
    rng = np.random.default_rng(32)
    B, nq = 32, 300
    val = rng.standard_normal((B, 13125, 8, 32), dtype=np.float32)
    loc = rng.uniform(0, 1, (B, nq, 8, 3, 4, 2)).astype(np.float32)
    lg = rng.standard_normal((B, nq, 8, 12)).astype(np.float32)
    w = np.exp(lg - lg.max(-1, keepdims=True))
    w = (w / w.sum(-1, keepdims=True)).astype(np.float32)
    got = _msda(cuda, val, loc.reshape(B, nq, 192), w.reshape(B, nq, 96), None, B, nq, canon=True)
    exp = orc.msdeform_canon(val, loc, w)
    np.testing.assert_allclose(got, exp, rtol=0, atol=1e-6)


def test_mask_box_vs_golden(cuda, golden_dir):
    g = np.load(f"{golden_dir}/mask_box_s21.npz")
    ml = cases.mask_box_inputs(21)
    out = torch.empty((300, 4), dtype=torch.float32, device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_MASKBOX, out, [_dev(ml, cuda)]))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    np.testing.assert_allclose(got, g["out"], rtol=2e-7, atol=0)
    # the integer box behind the logits is exact: identical after sigmoid
    np.testing.assert_array_equal(np.isfinite(got), np.isfinite(g["out"]))


def test_mask_box_batched(cuda, orc):
    ml = np.stack([cases.mask_box_inputs(21)[:50], cases.mask_box_inputs(22)[:50]])
    out = torch.empty((2, 50, 4), dtype=torch.float32, device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_MASKBOX, out, [_dev(ml, cuda)]))
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), orc.mask_box(ml), rtol=2e-7, atol=0)


@pytest.mark.parametrize("seed", [31, 32])
def test_topk_vs_golden(cuda, golden_dir, seed):
    g = np.load(f"{golden_dir}/topk300_s{seed}.npz")
    lg = cases.topk_inputs(seed)
    out = torch.empty((300,), dtype=torch.int32, device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_TOPK, out, [_dev(lg, cuda)]))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), g["out"])


def test_topk_mass_ties_and_extremes(cuda, orc):
    # the selection is a radix select over (max-logit bits, index) keys: a page
    # where every token ties (the winners are the 300 lowest indices), one with
    # a few hundred ties straddling the 300th place, one with +-inf and the
    # largest/smallest finite logits
    a = np.full_like(cases.topk_inputs(31), 0.25)
    b = cases.topk_inputs(32)
    b[::40] = 3.0                      # 329 tokens tie at the top
    c = cases.topk_inputs(33)
    c[5, 3] = np.inf
    c[77] = -np.inf
    c[100, 0] = np.finfo(np.float32).max
    c[101, 1] = -np.finfo(np.float32).max
    lg = np.stack([a, b, c]).astype(np.float32)
    out = torch.empty((3, 300), dtype=torch.int32, device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_TOPK, out, [_dev(lg, cuda)]))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    np.testing.assert_array_equal(got, orc.topk(lg))
    np.testing.assert_array_equal(got[0], np.arange(300))


def test_topk_batched_with_signed_zero_ties(cuda, orc):
    lg = np.stack([cases.topk_inputs(31), cases.topk_inputs(32)])
    lg[0, 200:260] = -0.0
    lg[0, 260:300] = 0.0      # -0 and +0 tie; ties go to the lower index
    lg[0] = np.minimum(lg[0], 0.0)
    out = torch.empty((2, 300), dtype=torch.int32, device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_TOPK, out, [_dev(lg, cuda)]))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), orc.topk(lg))


def test_bias_act_and_copy(cuda):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((2, 5, 7, 9), dtype=np.float32)  # B,C,H,W
    b = rng.standard_normal(5, dtype=np.float32)
    xt, bt = _dev(x, cuda), _dev(b, cuda)
    for act in (0, 1, 2):
        y = torch.empty_like(xt)
        ppdl.check(ppdl.op_launch(ppdl.OP_BIASACT, y, [xt, bt], params=[act]))
        v = torch.from_numpy(x) + torch.from_numpy(b)[None, :, None, None]
        ref = {0: v, 1: torch.relu(v), 2: v / (1 + torch.exp(-v))}[act]
        torch.cuda.synchronize()
        np.testing.assert_allclose(y.cpu().numpy(), ref.numpy(), rtol=1e-6, atol=1e-7)
    y = torch.empty(1001, device=cuda)
    src = torch.arange(1001, dtype=torch.float32, device=cuda)
    ppdl.check(ppdl.op_launch(ppdl.OP_COPY, y, [src]))
    torch.cuda.synchronize()
    assert torch.equal(y, src)


def test_silu_quotient_is_correctly_rounded(cuda):
    """SiLU as every epilogue applies it, x / (1 + exp(-x)) with a
    branch-free quotient, equals the same formula on the device with IEEE
    division (torch: the same expf, then a correctly rounded divide) bit for
    bit: 16M values over [-110, 40] (the overflow of exp(-x) below -88.7
    included), the ranges near 0 and the powers of two."""
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.cat([torch.rand(1 << 24, generator=g, device=cuda) * 150.0 - 110.0,
                   torch.randn(1 << 20, generator=g, device=cuda),
                   torch.randn(1 << 20, generator=g, device=cuda) * 1e-30,
                   2.0 ** torch.arange(-126, 7, device=cuda, dtype=torch.float32),
                   -(2.0 ** torch.arange(-126, 7, device=cuda, dtype=torch.float32)),
                   torch.tensor([0.0, -0.0, 17.0, 88.7, -88.7, -89.0, -1e4], device=cuda)])
    y = torch.empty_like(x)
    zero = torch.tensor([-0.0], device=cuda)  # x + (-0) == x, signed zeros included
    ppdl.check(ppdl.op_launch(ppdl.OP_BIASACT, y, [x, zero], params=[2]))
    ref = x / (1 + torch.exp(-x))
    torch.cuda.synchronize()
    bad = (y.view(torch.int32) != ref.view(torch.int32)).nonzero().flatten()
    assert bad.numel() == 0, (x[bad[:5]].tolist(), y[bad[:5]].tolist(), ref[bad[:5]].tolist())


def test_errors_are_status_codes(cuda):
    out = torch.empty((300, 3), device=cuda)
    ml = torch.zeros((300, 40000), device=cuda)
    assert ppdl.op_launch(ppdl.OP_MASKBOX, out, [ml]) == ppdl.PPDL_ERR_SHAPE
    assert "mask_box" in ppdl.last_error()
    assert ppdl.op_launch(ppdl.OP_WG_INPUT, out, [ml]) == ppdl.PPDL_ERR_UNSUPPORTED
    assert ppdl.op_launch(99, out, [ml]) == ppdl.PPDL_ERR_UNSUPPORTED
    assert not ppdl.op_supported(99)
    assert ppdl.op_supported(ppdl.OP_MSDEF)
