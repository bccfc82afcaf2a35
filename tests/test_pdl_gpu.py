"""Programmatic dependent launch changes no result.

Every kernel of the library is launched with programmatic stream
serialization and waits for the grid before it (griddepcontrol.wait) ahead
of its first global access.  A kernel that touched memory before that wait
would race with its predecessor; such a race shows up as a difference
between the forward with the attribute and without it (PPDL_PDL=0, read once
per process, hence the child processes).  The forward has no atomics or
order-dependent reductions, so the two must agree bit for bit: dets, packed
masks and the raw encoder/decoder outputs of two pages, the graph replayed
several times.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

CHILD = r"""
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/ppdoclayout-ggml_b200")
import ppdl, synth
ctx = ppdl.Context(sys.argv[2], max_batch=2)
imgs = np.stack([synth.synth_page(300), synth.synth_page(301)])
hw = np.array([[800, 800], [1000, 700]], np.int32)
outs = None
for _ in range(4):  # the first call captures the graph, the others replay it
    outs = ctx.infer_batch(imgs, hw)
assert ctx.dump_raw(sys.argv[3] + "_") == 0
np.savez(sys.argv[3] + ".npz", d0=outs[0][0], m0=outs[0][1] != 0, d1=outs[1][0],
         m1=outs[1][1] != 0)
ctx.close()
"""


def _run(gguf, out, pdl):
    env = dict(os.environ)
    env["PPDL_PDL"] = "1" if pdl else "0"
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT, gguf, out], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]


def test_forward_identical_with_and_without_pdl(cuda, tmp_path):
    gguf = synth.cached_gguf(0, os.environ.get("PPDL_SYNTH_DIR") or str(tmp_path))
    a, b = str(tmp_path / "pdl"), str(tmp_path / "nopdl")
    _run(gguf, a, True)
    _run(gguf, b, False)
    za, zb = np.load(a + ".npz"), np.load(b + ".npz")
    for k in ("d0", "m0", "d1", "m1"):
        np.testing.assert_array_equal(za[k], zb[k], err_msg=k)
    for k in ("logits", "boxes", "order", "sel", "topk"):
        ra = np.fromfile(f"{a}_{k}.bin", dtype=np.uint8)
        rb = np.fromfile(f"{b}_{k}.bin", dtype=np.uint8)
        assert ra.size > 0 and np.array_equal(ra, rb), k
