"""End-to-end parity: the B200 forward through the public C ABI
(ppdl_infer_batch / ppdl_infer / ppdl_dump_raw) against the CPU restatement
of the reference graph (oracle/model_ref.py), on seeded synthetic pages and
seeded random weights.

Gates (the hot path's end-to-end contract):
  * identical labels and top-300 selection for detections whose score
    margin to their neighbours exceeds 1e-4;
  * score diff < 1e-4, box diff <= 0.01 px;
  * mask IoU >= 0.99;
  * identical reading order for detections with score >= 0.3.
"""
import os

import numpy as np
import pytest

import ppdl
import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    d = os.environ.get("PPDL_SYNTH_DIR") or str(tmp_path_factory.mktemp("synth"))
    return synth.cached_gguf(0, d)


@pytest.fixture(scope="module")
def ref_model(gguf_path):
    from oracle import model_ref
    return model_ref.RefModel(model_ref.load_gguf(gguf_path))


@pytest.fixture(scope="module")
def pages():
    return [(synth.synth_page(100 + i), hw) for i, hw in enumerate([(1000, 700), (800, 800)])]


@pytest.fixture(scope="module")
def ref_out(ref_model, pages):
    return [ref_model.forward(img, h, w) for img, (h, w) in pages]


@pytest.fixture(scope="module")
def gpu_out(cuda, gguf_path, pages, tmp_path_factory):
    ctx = ppdl.Context(gguf_path, max_batch=2)
    imgs = np.stack([p[0] for p in pages])
    hw = np.array([p[1] for p in pages], np.int32)
    outs = ctx.infer_batch(imgs, hw)
    d = tmp_path_factory.mktemp("raw")
    assert ctx.dump_raw(str(d) + "/p0_") == 0
    raw = {k: np.fromfile(str(d) + f"/p0_{k}.bin",
                          dtype=np.int32 if k in ("sel", "topk") else np.float32)
           for k in ("logits", "boxes", "order", "sel", "topk")}
    ctx.close()
    return outs, raw


def _margin_ok(scores, i, tol=1e-4):
    lo = scores[i + 1] if i + 1 < len(scores) else -1.0
    hi = scores[i - 1] if i > 0 else 2.0
    return hi - scores[i] > tol and scores[i] - lo > tol


def test_raw_outputs_page0(gpu_out, ref_out):
    _, raw = gpu_out
    r = ref_out[0]
    # Decoder queries are the encoder's top-300 tokens in score order.  Two
    # FP32 implementations may order near-tied tokens differently (the test
    # pages hold gaps of ~1e-6 inside the top 300), which permutes decoder
    # rows; self-attention is permutation-equivariant, so rows are matched by
    # token.  Allowed: the same 300 tokens, displaced only where the oracle's
    # encoder scores of the two tokens differ by less than TIE.
    TIE = 1e-5
    gt, rt = raw["topk"], np.asarray(r["topk"], np.int64)
    assert set(gt.tolist()) == set(rt.tolist()), "top-300 token sets differ"
    for i in np.nonzero(gt != rt)[0]:
        assert abs(r["enc_max"][gt[i]] - r["enc_max"][rt[i]]) < TIE, f"query {i} reordered"
    gpos = {int(t): i for i, t in enumerate(gt)}
    idx = np.array([gpos[int(t)] for t in rt])
    lg = raw["logits"].reshape(300, 25)[idx]
    s_gpu, s_ref = 1 / (1 + np.exp(-lg.astype(np.float64))), 1 / (1 + np.exp(-r["logits"].astype(np.float64)))
    assert np.abs(s_gpu - s_ref).max() < 1e-4, np.abs(s_gpu - s_ref).max()
    assert np.abs(raw["boxes"].reshape(300, 4)[idx] - r["boxes"]).max() * 1000 <= 0.01
    od = raw["order"].reshape(300, 300)[idx][:, idx].reshape(-1)
    assert np.abs(od - r["order"]).max() / max(np.abs(r["order"]).max(), 1) < 1e-4


def _check_page(dets, masks, r, min_checked=30):
    """The end-to-end gates of one page against the oracle's result r;
    returns the number of rows held to the per-row gates (rows whose score
    margins to both neighbours exceed 1e-4 — a property of the page)."""
    rd, rm = r["dets"], r["masks"].reshape(300, 200, 200)
    scores = rd[:, 1]
    n_checked = 0
    for i in range(300):
        if not _margin_ok(scores, i):
            continue
        n_checked += 1
        assert dets[i, 0] == rd[i, 0], f"label row {i}"
        assert abs(dets[i, 1] - rd[i, 1]) < 1e-4, f"score row {i}"
        # box diff in pixels of the original image
        assert np.abs(dets[i, 2:6] - rd[i, 2:6]).max() <= 0.01, f"box row {i}"
        a, b = masks[i] != 0, rm[i] != 0
        union = np.logical_or(a, b).sum()
        iou = np.logical_and(a, b).sum() / union if union else 1.0
        assert iou >= 0.99, f"mask IoU row {i}: {iou}"
        if rd[i, 1] >= 0.3:
            assert dets[i, 6] == rd[i, 6], f"reading order row {i}"
    assert n_checked >= min_checked, n_checked
    # the whole score column regardless of margins
    assert np.abs(dets[:, 1] - rd[:, 1]).max() < 1e-4
    return n_checked


@pytest.mark.parametrize("page", [0, 1])
def test_dets_and_masks(gpu_out, ref_out, pages, page):
    outs, _ = gpu_out
    dets, masks = outs[page]
    _check_page(dets, masks, ref_out[page])


def test_batch8_bench_pages_graph_replay(cuda, gguf_path, ref_model):
    """The benchmarked configuration: a context of capacity 8 (as bench.py's
    forward workload), the 8 pages bench.py times on rank 0 (seeds
    1000..1007, 800 x 800), run twice — the first call eager, the second a
    replay of the captured CUDA graph — and every page of the replay held
    to the end-to-end gates; eager and replay agree bit for bit.  Random
    weights leave some pages with many near-tied scores, so the rows with
    clear margins are counted over the batch (at least 5 per page, 120 in
    all) rather than 30 per page."""
    B = 8
    ctx = ppdl.Context(gguf_path, max_batch=B)
    imgs = np.stack([synth.synth_page(1000 + i) for i in range(B)])
    hw = np.full((B, 2), 800, np.int32)
    eager = ctx.infer_batch(imgs, hw)
    replay = ctx.infer_batch(imgs, hw)
    ctx.close()
    total = 0
    for i in range(B):
        np.testing.assert_array_equal(eager[i][0], replay[i][0])
        np.testing.assert_array_equal(eager[i][1], replay[i][1])
        r = ref_model.forward(imgs[i], 800, 800)
        total += _check_page(replay[i][0], replay[i][1], r, min_checked=5)
    assert total >= 120, total


def test_batch32_stress_pages_match_batch8(cuda, gguf_path):
    """Config 4's batch size: a context of capacity 32 (as bench.py's stress
    workload) takes 32 pages through the pipelined API, and every page's dets
    and packed masks equal those of the same page in a capacity-8 context
    (the size the oracle gates above hold), so the parity carries over to the
    stress configuration.  The results match bit for bit: the GEMMs' tiles
    cut across pages' rows, never through a dot product, and no reduction
    order depends on the batch."""
    import torch
    imgs = np.stack([synth.synth_page(2000 + i) for i in range(32)])
    hw = np.array([[800, 800] if i % 3 else [1000, 700] for i in range(32)], np.int32)
    c32 = ppdl.Context(gguf_path, max_batch=32)
    buf = torch.from_numpy(imgs).pin_memory().numpy()
    r32 = [(d.copy(), b.copy()) for d, b in c32.wait(c32.submit(buf, hw), 32)]
    c32.close()
    c8 = ppdl.Context(gguf_path, max_batch=8)
    for b0 in range(0, 32, 8):
        bb = torch.from_numpy(np.ascontiguousarray(imgs[b0:b0 + 8])).pin_memory().numpy()
        r8 = c8.wait(c8.submit(bb, np.ascontiguousarray(hw[b0:b0 + 8])), 8)
        for k in range(8):
            np.testing.assert_array_equal(r32[b0 + k][0], r8[k][0])
            np.testing.assert_array_equal(r32[b0 + k][1], r8[k][1])
    c8.close()


def test_pipelined_batches_with_packed_masks(cuda, gguf_path, pages, gpu_out):
    """ppdl_submit_batch / ppdl_wait_batch: three batches in a row from
    pinned host memory, two in flight; every result equals ppdl_infer_batch's
    (dets bit for bit, masks after unpacking the bits, also through the C
    expansion ppdl_expand_mask_bits); a ticket two submissions old is
    reported as overwritten."""
    import ctypes as C
    import torch
    ctx = ppdl.Context(gguf_path, max_batch=2)
    base = np.stack([p[0] for p in pages])
    hw = np.array([p[1] for p in pages], np.int32)
    order = [[0, 1], [1, 0], [0, 1]]
    bufs = [torch.from_numpy(np.ascontiguousarray(base[o])).pin_memory().numpy() for o in order]
    hws = [np.ascontiguousarray(hw[o]) for o in order]
    t0 = ctx.submit(bufs[0], hws[0])
    t1 = ctx.submit(bufs[1], hws[1])
    r0 = ctx.wait(t0, 2)
    t2 = ctx.submit(bufs[2], hws[2])
    r1 = ctx.wait(t1, 2)
    r2 = ctx.wait(t2, 2)
    with pytest.raises(RuntimeError):
        ctx.wait(t0, 2)  # slot reused by t2
    want = gpu_out[0]
    for o, r in zip(order, (r0, r1, r2)):
        for k, page in enumerate(o):
            dets, bits = r[k]
            np.testing.assert_array_equal(dets, want[page][0])
            np.testing.assert_array_equal(ppdl.unpack_mask_bits(bits), want[page][1] != 0)
    L = ppdl.lib()
    L.ppdl_expand_mask_bits.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    bits = np.ascontiguousarray(r2[0][1])
    m32 = np.empty((300, 200, 200), np.int32)
    L.ppdl_expand_mask_bits(bits.ctypes.data, m32.ctypes.data, 300)
    np.testing.assert_array_equal(m32, want[0][1])
    ctx.close()


def test_single_page_api_matches_batch(cuda, gguf_path, pages, gpu_out):
    ctx = ppdl.Context(gguf_path, max_batch=1)
    img, (h, w) = pages[0]
    dets, masks, ms = ctx.infer(img, h, w)
    dets2, _, _ = ctx.infer(img, h, w)  # graph replay path
    ctx.close()
    np.testing.assert_array_equal(dets, dets2)
    bd, bm = gpu_out[0][0]
    np.testing.assert_allclose(dets, bd, rtol=0, atol=1e-5)
    assert ms > 0


def test_bad_arguments(cuda, gguf_path):
    import ctypes as C
    L = ppdl.lib()
    res = ppdl.Result()
    assert L.ppdl_infer(None, None, 800, 800, C.byref(res)) == 1
    ctx = ppdl.Context(gguf_path)
    img = np.zeros((3, 800, 800), np.float32)
    assert L.ppdl_infer(ctx.ctx, img.ctypes.data, 0, 800, C.byref(res)) == 1
    assert L.ppdl_infer(ctx.ctx, img.ctypes.data, 800, -5, C.byref(res)) == 1
    ctx.close()
    assert L.ppdl_init(b"/nonexistent/model.gguf", 1) is None
    assert L.ppdl_init(gguf_path.encode(), 0) is None  # no CPU backend in this build


def test_zero_copy_views_and_profiles(cuda, gguf_path, pages, gpu_out):
    """infer_batch(copy=False) returns views of the context's pinned result
    buffers with the same values as the copies; the per-step profile and the
    lane timeline cover the same steps, every lane's steps end in stream
    order, and the side lanes (value projections; k/v, mask-feature head,
    reading-order head) are used."""
    import torch
    ctx = ppdl.Context(gguf_path, max_batch=2)
    imgs = torch.from_numpy(np.stack([p[0] for p in pages])).pin_memory().numpy()
    hw = np.array([p[1] for p in pages], np.int32)
    views = ctx.infer_batch(imgs, hw, copy=False)
    for (d, m), (bd, bm) in zip(views, gpu_out[0]):
        np.testing.assert_array_equal(d, bd)
        np.testing.assert_array_equal(m, bm)
    steps = ctx.profile_steps(2)
    tl = ctx.profile_timeline(2)
    ctx.close()
    assert len(tl) == len(steps) > 300
    assert {lane for _, lane in tl} == {0, 1, 2}
    assert all(np.isfinite(e) and e > 0 for e, _ in tl)
    assert all(s[2] > 0 for s in steps)
    last = {}
    for e, lane in tl:
        assert e >= last.get(lane, 0.0)
        last[lane] = e
