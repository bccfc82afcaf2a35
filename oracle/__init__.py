"""ctypes bindings for the CPU checkers (TEST INFRASTRUCTURE ONLY).

``oracle`` wraps ``lib/libppdl_oracle.so`` (the C restatement in
``ppdl_oracle.c``); ``ref`` wraps ``_ref/librefops.so`` (the reference's own
CPU ops compiled from its sources, present only where the reference checkout
was available at build time).  Only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg import this package, and only as the checker or
the timed CPU arm; the product library never touches it.

All arrays are numpy, C-contiguous; shapes follow the C docs in
ppdl_oracle.c.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "lib", "libppdl_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "librefops.so")

NQ, NC, DM, NH, HD = 300, 25, 256, 8, 32
NTOK, MASK_HW = 13125, 200
MASK_PIX = MASK_HW * MASK_HW
LVL_HW = ((100, 100), (50, 50), (25, 25))
LVL_START = (0, 10000, 12500)

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int32)


def _f(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_fp)


def _i(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


def build(ref_dir: str | None = None) -> None:
    """Compile the checkers in-tree (make -C oracle)."""
    import subprocess
    cmd = ["make", "-s", "-C", HERE]
    if ref_dir and os.path.isdir(ref_dir):
        cmd.append(f"REF={ref_dir}")
    subprocess.run(cmd, check=True)


class _Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        self.lib = C.CDLL(path)

    # -- MSDA ---------------------------------------------------------------
    def msdeform(self, val, off, awr, ref):
        """In-model MSDA; val [B,13125,256], off [B,nq,192], awr [B,nq,96],
        ref [B,nq,4] -> [B,nq,256]."""
        B, nq = off.shape[0], off.shape[1]
        out = np.zeros((B, nq, DM), np.float32)
        self.lib.oracle_msdeform(_f(val), _f(off), _f(awr), _f(ref), _f(out), nq, B)
        return out

    def msdeform_canon(self, val, loc, w):
        """Canonical MSDA; val [B,13125,8,32], loc [B,nq,8,3,4,2], w [B,nq,8,12]."""
        B, nq = loc.shape[0], loc.shape[1]
        out = np.zeros((B, nq, DM), np.float32)
        self.lib.oracle_msdeform_canon(_f(val), _f(loc), _f(w), _f(out), nq, B)
        return out

    def mask_box(self, ml):
        """ml [B,nq,40000] -> [B,nq,4] inverse-sigmoid cxcywh."""
        B, nq = ml.shape[0], ml.shape[1]
        out = np.zeros((B, nq, 4), np.float32)
        self.lib.oracle_mask_box(_f(ml), _f(out), nq, B)
        return out

    def topk(self, lg, nq=NQ):
        """lg [B,ntok,nc] -> [B,nq] int32."""
        B, ntok, nc = lg.shape
        out = np.zeros((B, nq), np.int32)
        self.lib.oracle_topk(_f(lg), _i(out), ntok, nc, nq, B)
        return out

    # -- Winograd F(4,3) --------------------------------------------------------
    def wg4_matrix(self, which):
        """0 -> B4 (6x6), 1 -> G4 (6x3), 2 -> A4 (6x4)."""
        self.lib.oracle_wg4_matrix.restype = _fp
        p = self.lib.oracle_wg4_matrix(which)
        n, shape = {0: (36, (6, 6)), 1: (18, (6, 3)), 2: (24, (6, 4))}[which]
        return np.ctypeslib.as_array(p, (n,)).copy().reshape(shape)

    def wg4_filter(self, w):
        OC, IC = w.shape[0], w.shape[1]
        out = np.zeros((36, IC, OC), np.float32)
        self.lib.oracle_wg4_filter(_f(w), _f(out), IC, OC)
        return out

    def wg4_input(self, xp, TW, TH):
        IC, IH, IW = xp.shape
        out = np.zeros((36, IC, TW * TH), np.float32)
        self.lib.oracle_wg4_input(_f(xp), _f(out), IW, IH, IC, TW, TH)
        return out

    def wg4_madd(self, dt, wg4):
        _, IC, T = dt.shape
        OC = wg4.shape[2]
        out = np.zeros((36, OC, T), np.float32)
        self.lib.oracle_wg4_madd(_f(dt), _f(wg4), _f(out), T, IC, OC)
        return out

    def wg4_output(self, yt, bias, TW, OW, OH, act):
        _, OC, T = yt.shape
        out = np.zeros((OC, OH, OW), np.float32)
        self.lib.oracle_wg4_output(_f(yt), _f(bias), _f(out), T, TW, OC, OW, OH, act)
        return out

    def conv2d(self, x, w, b, stride, pad, groups=1, act=0):
        """x [IC,IH,IW], w [OC,IC/groups,K,K] -> [OC,OH,OW] (double accumulate)."""
        IC, IH, IW = x.shape
        OC, _, K, _ = w.shape
        OH = (IH + 2 * pad - K) // stride + 1
        OW = (IW + 2 * pad - K) // stride + 1
        out = np.zeros((OC, OH, OW), np.float32)
        self.lib.oracle_conv2d(_f(x), _f(w), _f(b), _f(out), IC, IH, IW, OC, K, stride, pad,
                               groups, act)
        return out

    # -- host constants / postprocess -----------------------------------------
    def pos_embed(self):
        out = np.zeros((625, DM), np.float32)
        self.lib.oracle_pos_embed(_f(out))
        return out

    def valid_mask(self):
        out = np.zeros((NTOK,), np.float32)
        self.lib.oracle_valid_mask(_f(out))
        return out

    def postprocess(self, logits, boxes, order, maskl, ori_h, ori_w, with_masks=True):
        dets = np.zeros((NQ, 7), np.float32)
        sel = np.zeros((NQ,), np.int32)
        masks = np.zeros((NQ, MASK_PIX), np.int32) if with_masks else None
        self.lib.oracle_postprocess(
            _f(logits), _f(boxes), _f(order),
            _f(maskl) if with_masks else None, int(ori_h), int(ori_w),
            _f(dets), _i(masks) if with_masks else None, _i(sel))
        return dets, masks, sel


class _Ref:
    """The reference's own CPU custom ops (batch 1, nq = 300)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)

    def msdeform(self, val, off, awr, ref, nth=1):
        out = np.zeros((NQ, DM), np.float32)
        self.lib.ref_msdeform(_f(val), _f(off), _f(awr), _f(ref), _f(out), nth)
        return out

    def mask_box(self, ml, nth=1):
        out = np.zeros((NQ, 4), np.float32)
        self.lib.ref_mask_box(_f(ml), _f(out), nth)
        return out

    def topk300(self, lg):
        out = np.zeros((NQ,), np.int32)
        self.lib.ref_topk300(_f(lg), _i(out))
        return out


_oracle = None


def oracle() -> _Oracle:
    global _oracle
    if _oracle is None:
        _oracle = _Oracle()
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> _Ref:
    return _Ref()
