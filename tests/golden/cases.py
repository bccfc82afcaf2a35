"""Seeded input generators for the golden operator fixtures.

The fixtures under tests/golden/ hold only the seed, a sha256 of the
regenerated inputs and the reference's outputs: the inputs (13-48 MB per
case) are rebuilt here from numpy's PCG64 stream, and the checksum proves the
rebuild matches the inputs the reference saw.

Each generator mirrors the shapes of the reference op it feeds
(src/ppdoclayout.cpp:73-198) and plants the edge cases that op has: sample
points out of bounds and exactly on pixel centres (MSDA), empty / single
pixel / full / zero-valued masks (mask->box), and exact ties (top-300).
"""
from __future__ import annotations

import hashlib

import numpy as np

NQ, NC, DM, NTOK, MASK_HW = 300, 25, 256, 13125, 200


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def msdeform_inputs(seed: int):
    """value [13125,256], off [300,192], awr [300,96], ref [300,4]."""
    rng = np.random.default_rng(seed)
    val = rng.standard_normal((NTOK, DM), dtype=np.float32)
    off = (rng.standard_normal((NQ, 192), dtype=np.float32) * 2.0).astype(np.float32)
    awr = rng.standard_normal((NQ, 96), dtype=np.float32)
    ref = np.empty((NQ, 4), np.float32)
    ref[:, 0:2] = rng.uniform(0.02, 0.98, (NQ, 2)).astype(np.float32)
    ref[:, 2:4] = rng.uniform(0.01, 0.8, (NQ, 2)).astype(np.float32)
    # edge rows: boxes hugging the borders with large offsets (points leave
    # the map on every side), and points landing exactly on pixel centres
    # (fractional part 0 -> zero-weight corners that the op skips)
    ref[0] = (0.0, 0.0, 1.0, 1.0)
    ref[1] = (1.0, 1.0, 1.0, 1.0)
    off[0:2] *= 4.0
    ref[2] = (0.5, 0.5, 0.0, 0.0)        # every point at the box centre
    ref[3] = (0.005, 0.995, 0.0, 0.0)    # centre between the pixel grid and the border
    ref[4] = (0.0, 0.0, 8.0, 8.0)        # loc == offset exactly (canonical form)
    off[4] = rng.integers(0, 25, 192).astype(np.float32) / 25.0 + 0.02  # on pixel centres of level 2
    return val, off, awr, ref


def mask_box_inputs(seed: int):
    """mask logits [300, 40000]: rectangles of positives on a negative field."""
    rng = np.random.default_rng(seed)
    ml = -rng.uniform(0.01, 3.0, (NQ, MASK_HW, MASK_HW)).astype(np.float32)
    for q in range(NQ):
        kind = q % 10
        if kind == 0:
            continue                                   # empty -> box 0
        if kind == 1:
            y, x = rng.integers(0, MASK_HW, 2)
            ml[q, y, x] = 0.5                          # single pixel
            continue
        if kind == 2:
            ml[q] = np.abs(ml[q]) + 0.1                # full mask
            continue
        if kind == 3:
            ml[q, rng.integers(0, MASK_HW), :] = 0.0   # exact zeros are not > 0
            ml[q, :, rng.integers(0, MASK_HW)] = -0.0
            y, x = rng.integers(0, MASK_HW, 2)
            ml[q, y, x] = 1e-30                        # tiny positive counts
            continue
        y0, x0 = rng.integers(0, MASK_HW, 2)
        y1 = min(MASK_HW, y0 + int(rng.integers(1, 120)))
        x1 = min(MASK_HW, x0 + int(rng.integers(1, 120)))
        ml[q, y0:y1, x0:x1] = rng.uniform(0.01, 3.0, (y1 - y0, x1 - x0))
        if kind >= 8:                                  # scattered extra positives
            n = int(rng.integers(1, 20))
            ml[q, rng.integers(0, MASK_HW, n), rng.integers(0, MASK_HW, n)] = 2.0
    return ml.reshape(NQ, MASK_HW * MASK_HW)


def topk_inputs(seed: int):
    """class logits [13125, 25] quantised to 1/16 so many token maxima tie."""
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((NTOK, NC), dtype=np.float32) * 2.0
    lg = (np.round(lg * 16.0) / 16.0).astype(np.float32)
    lg[100:140] = 9.0        # a block of exact ties at the very top
    lg[5000, 3] = 12.0
    lg[7] = -lg[7]
    return lg
