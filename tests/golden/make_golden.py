"""Regenerate the golden operator fixtures from the reference's own CPU ops.

Run in a checkout that has the reference sources (the fixtures are committed,
so this is only needed to refresh them):

    make -C oracle REF=<reference checkout>
    python tests/golden/make_golden.py

It loads oracle/_ref/librefops.so — op_msdeform, op_mask_box and op_topk300
compiled unmodified from the reference (src/ppdoclayout.cpp:73-198) — runs
them on the seeded inputs of cases.py and stores the seed, the input digest
and the outputs as .npz files beside this script.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

import cases  # noqa: E402
import oracle  # noqa: E402

MSDA_SEEDS = (11, 12)
MASKBOX_SEEDS = (21,)
TOPK_SEEDS = (31, 32)


def main():
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref/librefops.so missing: make -C oracle REF=<reference>")
    r = oracle.ref()
    for s in MSDA_SEEDS:
        val, off, awr, ref = cases.msdeform_inputs(s)
        out = r.msdeform(val, off, awr, ref, nth=8)
        np.savez_compressed(os.path.join(HERE, f"msdeform_s{s}.npz"), seed=s,
                            digest=cases.digest(val, off, awr, ref), out=out)
    for s in MASKBOX_SEEDS:
        ml = cases.mask_box_inputs(s)
        out = r.mask_box(ml, nth=8)
        np.savez_compressed(os.path.join(HERE, f"mask_box_s{s}.npz"), seed=s,
                            digest=cases.digest(ml), out=out)
    for s in TOPK_SEEDS:
        lg = cases.topk_inputs(s)
        out = r.topk300(lg)
        np.savez_compressed(os.path.join(HERE, f"topk300_s{s}.npz"), seed=s,
                            digest=cases.digest(lg), out=out)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
