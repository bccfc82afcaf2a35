"""The CPU oracle, pinned before anything is compared against it.

* golden fixtures made by the reference's own CPU ops (tests/golden/) —
  bit-exact;
* the reference ops themselves, when they were compiled from a reference
  checkout into oracle/_ref/ (skipped elsewhere) — bit-exact on fresh seeds;
* the reference's Winograd known-answer test (bench/wg_test.cu:89-167:
  10x9 input, IC=3, OC=2, sin/cos data, pipeline vs direct correlation),
  re-targeted from F(2,3) to F(4,3) with the tolerance tightened from 1e-3
  absolute to 1e-5 relative.
"""
import numpy as np
import pytest

import cases
import oracle


def _load(golden_dir, name):
    return np.load(f"{golden_dir}/{name}")


@pytest.mark.parametrize("seed", [11, 12])
def test_msdeform_golden(orc, golden_dir, seed):
    g = _load(golden_dir, f"msdeform_s{seed}.npz")
    val, off, awr, ref = cases.msdeform_inputs(seed)
    assert cases.digest(val, off, awr, ref) == str(g["digest"]), "input regeneration drifted"
    out = orc.msdeform(val, off[None], awr[None], ref[None])[0]
    np.testing.assert_array_equal(out, g["out"])


def test_mask_box_golden(orc, golden_dir):
    g = _load(golden_dir, "mask_box_s21.npz")
    ml = cases.mask_box_inputs(21)
    assert cases.digest(ml) == str(g["digest"])
    np.testing.assert_array_equal(orc.mask_box(ml[None])[0], g["out"])


@pytest.mark.parametrize("seed", [31, 32])
def test_topk_golden(orc, golden_dir, seed):
    g = _load(golden_dir, f"topk300_s{seed}.npz")
    lg = cases.topk_inputs(seed)
    assert cases.digest(lg) == str(g["digest"])
    np.testing.assert_array_equal(orc.topk(lg[None])[0], g["out"])


def test_canonical_msda_equals_in_model_form(orc):
    """ref = (0, 0, 8, 8) makes the in-model location equal the offset
    exactly (src/ppdoclayout.cpp:174-175), so both forms must agree
    bit-for-bit when the canonical weights are the in-model softmax."""
    rng = np.random.default_rng(5)
    val = rng.standard_normal((1, 13125, 256), dtype=np.float32)
    loc = rng.uniform(-0.05, 1.05, (1, 300, 192)).astype(np.float32)
    awr = rng.standard_normal((1, 300, 96), dtype=np.float32)
    ref = np.tile(np.array([0, 0, 8, 8], np.float32), (1, 300, 1))
    a = awr.reshape(1, 300, 8, 12)
    e = np.exp((a - a.max(-1, keepdims=True)).astype(np.float32)).astype(np.float32)
    s = np.zeros(e.shape[:-1], np.float32)
    for i in range(12):  # the reference's sequential sum
        s = (s + e[..., i]).astype(np.float32)
    w = (e / s[..., None]).astype(np.float32)
    got_in = orc.msdeform(val, loc, awr, ref)
    got_can = orc.msdeform_canon(val, loc, np.ascontiguousarray(w))
    # expf of numpy and of libm may differ in the last ulp; everything
    # downstream of the weights is the same arithmetic
    np.testing.assert_allclose(got_can, got_in, rtol=0, atol=2e-6)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference checkout not built here")
@pytest.mark.parametrize("seed", [101, 102, 103])
def test_oracle_matches_reference_ops(orc, seed):
    r = oracle.ref()
    val, off, awr, ref = cases.msdeform_inputs(seed)
    np.testing.assert_array_equal(orc.msdeform(val, off[None], awr[None], ref[None])[0],
                                  r.msdeform(val, off, awr, ref, nth=4))
    ml = cases.mask_box_inputs(seed)
    np.testing.assert_array_equal(orc.mask_box(ml[None])[0], r.mask_box(ml, nth=4))
    lg = cases.topk_inputs(seed)
    np.testing.assert_array_equal(orc.topk(lg[None])[0], r.topk300(lg))


def _wg_kat_case():
    """bench/wg_test.cu:89-110 data, on the F(4,3) tile grid."""
    IW, IH, IC, OC = 10, 9, 3, 2
    TW, TH = (IW + 3) // 4, (IH + 3) // 4
    IW_p, IH_p = 4 * TW + 2, 4 * TH + 2
    i = np.arange(IW_p * IH_p * IC, dtype=np.float32)
    xp = (np.sin(np.float32(0.7) * i) * np.float32(0.5)).astype(np.float32).reshape(IC, IH_p, IW_p)
    j = np.arange(9 * IC * OC, dtype=np.float32)
    w = (np.cos(np.float32(0.3) * j) * np.float32(0.4)).astype(np.float32).reshape(OC, IC, 3, 3)
    b = (np.float32(0.1) * np.arange(OC, dtype=np.float32)).astype(np.float32)
    return xp, w, b, IW, IH, TW, TH


def test_winograd_f43_known_answer(orc):
    xp, w, b, IW, IH, TW, TH = _wg_kat_case()
    # direct correlation over the padded frame (wg_test.cu:127-139), in double
    ref = np.zeros((w.shape[0], IH, IW), np.float64)
    for oc in range(w.shape[0]):
        for y in range(IH):
            for x in range(IW):
                ref[oc, y, x] = b[oc] + np.sum(xp[:, y:y + 3, x:x + 3].astype(np.float64) *
                                               w[oc].astype(np.float64))
    dt = orc.wg4_input(xp, TW, TH)
    wg4 = orc.wg4_filter(w)
    yt = orc.wg4_madd(dt, wg4)
    out = orc.wg4_output(yt, b, TW, IW, IH, 0)
    err = np.abs(out - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


def test_winograd_matrices_are_an_exact_f43(orc):
    """A^T [(G g) * (B^T d)] reproduces the 4-output 3-tap correlation in
    float64 for any d, g: the matrices define F(4,3) (patch:141-146 claims
    1e-13 in float64 for their solve)."""
    B = orc.wg4_matrix(0).astype(np.float64)
    G = orc.wg4_matrix(1).astype(np.float64)
    A = orc.wg4_matrix(2).astype(np.float64)
    rng = np.random.default_rng(0)
    for _ in range(4):
        d = rng.standard_normal(6)
        g = rng.standard_normal(3)
        y = A.T @ ((G @ g) * (B @ d))
        direct = np.array([np.dot(d[i:i + 3], g) for i in range(4)])
        np.testing.assert_allclose(y, direct, rtol=0, atol=2e-6)


def test_conv2d_oracle_against_numpy(orc):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 11, 13), dtype=np.float32)
    w = rng.standard_normal((4, 5, 3, 3), dtype=np.float32)
    b = rng.standard_normal(4, dtype=np.float32)
    got = orc.conv2d(x, w, b, stride=2, pad=1, act=1)
    xp = np.pad(x.astype(np.float64), ((0, 0), (1, 1), (1, 1)))
    OH, OW = (11 + 2 - 3) // 2 + 1, (13 + 2 - 3) // 2 + 1
    ref = np.zeros((4, OH, OW))
    for oy in range(OH):
        for ox in range(OW):
            patch = xp[:, 2 * oy:2 * oy + 3, 2 * ox:2 * ox + 3]
            ref[:, oy, ox] = np.tensordot(w.astype(np.float64), patch, 3) + b
    np.testing.assert_allclose(got, np.maximum(ref, 0), rtol=1e-6, atol=1e-6)


def test_postprocess_semantics(orc):
    rng = np.random.default_rng(9)
    logits = rng.standard_normal((300, 25), dtype=np.float32)
    logits[3, 4] = logits[7, 1] = 5.0          # tie -> lower flat index first
    boxes = rng.uniform(0.1, 0.9, (300, 4)).astype(np.float32)
    order = rng.standard_normal((300 * 300,), dtype=np.float32)
    maskl = rng.standard_normal((300, 40000), dtype=np.float32)
    dets, masks, sel = orc.postprocess(logits, boxes, order, maskl, 1000, 700)
    assert sel[0] == 3 * 25 + 4 and sel[1] == 7 * 25 + 1
    scores = 1 / (1 + np.exp(-logits.astype(np.float64)))
    assert np.all(np.diff(dets[:, 1]) <= 0)
    np.testing.assert_allclose(dets[:, 1], scores.reshape(-1)[sel], rtol=1e-6)
    q = sel // 25
    np.testing.assert_array_equal(masks, (maskl[q] > 0).astype(np.int32))
    assert set(np.unique(dets[:, 6]).astype(int)) <= set(range(300))


def test_host_constants(orc):
    pos = orc.pos_embed()
    assert pos.shape == (625, 256)
    np.testing.assert_allclose(pos[0, 64:128], 1.0)          # cos(0)
    np.testing.assert_allclose(pos[25 * 3 + 2, 0], np.sin(3.0), rtol=1e-6)
    vm = orc.valid_mask()
    assert vm.shape == (13125,) and set(np.unique(vm)) <= {0.0, 1.0}
    # anchor centres (x + 0.5) / W must lie strictly inside (0.01, 0.99):
    # the outer ring of the 100^2 and 50^2 levels drops out
    assert vm.sum() == 13125 - (4 * 100 - 4) - (4 * 50 - 4)
