"""Seeded synthetic PP-DocLayoutV3 weights (GGUF) and pages.

No real checkpoint is available, so weights are generated with the shapes
the reference's graph builder reads (src/ppdoclayout.cpp:388-882) under the
tensor names its converter writes (scripts/convert.py:17-67): BN-folded
F32 conv weights (ggml ne (KW,KH,IC,OC) = torch [OC][IC][KH][KW]) + bias,
Linear weight ne (in,out) = torch [out][in] + bias, LayerNorm weight/bias.

Architecture (HGNetV2-L backbone + hybrid encoder + 6-layer decoder):
  stem 3->32 (k3 s2) | 32->16->32 (k2, k2) | pool | 64->32 (k3 s2) | 32->48
  stage0 mid 48  out 128  1 block         (k3 layers)
  stage1 mid 96  out 512  1 block         (dw k3 s2 downsample, k3 layers)
  stage2 mid 192 out 1024 3 blocks light  (1x1 + dw k5 layers, residual b1/b2)
  stage3 mid 384 out 2048 1 block light
  encoder hidden 256, AIFI FFN 1024, CSP blocks with 3 RepVGG bottlenecks,
  mask-feature head 64 -> 32; decoder FFN 2048, 300 queries, 8 heads,
  3 levels x 4 points, 25 classes.
The FFN widths are not pinned by the reference sources (its GEMM
micro-bench uses 2048 for the decoder FFN, bench/gemm_bench.cu:99); the
product, the oracle and the tests all read them from the same GGUF.

Init: Kaiming-normal convs (fan-in, gain by the following activation),
Xavier-normal linears, small normal biases, LayerNorm gains near 1; BN is
already folded (weight + bias only).
"""
from __future__ import annotations

import os
from collections import OrderedDict

import numpy as np

HG_STAGES = (
    # name, in_ch, mid, out, blocks, light, downsample
    ("st0", 48, 48, 128, 1, False, False),
    ("st1", 128, 96, 512, 1, False, True),
    ("st2", 512, 192, 1024, 3, True, True),
    ("st3", 1024, 384, 2048, 1, True, True),
)
AIFI_FFN = 1024
DEC_FFN = 2048


def manifest() -> "OrderedDict[str, tuple]":
    """name -> (kind, torch-order shape[, activation]); kind in
    conv/dwconv/linear/ln/bias.  The activation after a conv picks its init
    gain (relu/silu 2, none 1, "half" 0.5 for the two summed RepVGG branches)
    so activations stay O(1) through the network, which is what the folded
    BatchNorm of a trained checkpoint achieves."""
    m: "OrderedDict[str, tuple]" = OrderedDict()

    def conv(name, ic, oc, k, act="relu"):
        m[name + ".weight"] = ("conv", (oc, ic, k, k), act)
        m[name + ".bias"] = ("bias", (oc,))

    def dw(name, c, k, act="none"):
        m[name + ".weight"] = ("dwconv", (c, 1, k, k), act)
        m[name + ".bias"] = ("bias", (c,))

    def lin(name, i, o):
        m[name + ".weight"] = ("linear", (o, i))
        m[name + ".bias"] = ("bias", (o,))

    def ln(name, d=256):
        m[name + ".weight"] = ("ln", (d,))
        m[name + ".bias"] = ("bias", (d,))

    conv("stem1", 3, 32, 3)
    conv("stem2a", 32, 16, 2)
    conv("stem2b", 16, 32, 2)
    conv("stem3", 64, 32, 3)
    conv("stem4", 32, 48, 1)
    for st, cin, mid, cout, nb, light, ds in HG_STAGES:
        if ds:
            dw(f"{st}.ds", cin, 3)
        for b in range(nb):
            bin_ = cin if b == 0 else cout
            cur = bin_
            for l in range(6):
                p = f"{st}.b{b}.l{l}"
                if light:
                    conv(p + ".c1", cur, mid, 1, "none")
                    dw(p + ".c2", mid, 5, "relu")
                else:
                    conv(p, cur, mid, 3)
                cur = mid
            cat = bin_ + 6 * mid
            conv(f"{st}.b{b}.agg0", cat, cout // 2, 1)
            conv(f"{st}.b{b}.agg1", cout // 2, cout, 1)
    conv("enc_in0", 512, 256, 1, "none")
    conv("enc_in1", 1024, 256, 1, "none")
    conv("enc_in2", 2048, 256, 1, "none")
    for n in ("q", "k", "v", "o"):
        lin(f"aifi.{n}", 256, 256)
    ln("aifi.ln1")
    ln("aifi.ln2")
    lin("aifi.fc1", 256, AIFI_FFN)
    lin("aifi.fc2", AIFI_FFN, 256)
    conv("lat0", 256, 256, 1, "silu")
    conv("lat1", 256, 256, 1, "silu")
    for blk in ("fpn0", "fpn1", "pan0", "pan1"):
        conv(f"{blk}.c1", 512, 256, 1, "silu")
        conv(f"{blk}.c2", 512, 256, 1, "silu")
        for i in range(3):
            conv(f"{blk}.bn{i}.c1", 256, 256, 3, "half")
            conv(f"{blk}.bn{i}.c2", 256, 256, 1, "half")
    conv("pand0", 256, 256, 3, "silu")
    conv("pand1", 256, 256, 3, "silu")
    conv("mh0.0", 256, 64, 3, "silu")
    conv("mh1.0", 256, 64, 3, "silu")
    conv("mh2.0", 256, 64, 3, "silu")
    conv("mh2.2", 64, 64, 3, "silu")
    conv("mh.out", 64, 64, 3, "silu")
    conv("mlat", 128, 64, 3, "silu")
    conv("mout.base", 64, 64, 3, "silu")
    conv("mout.conv", 64, 32, 1, "none")
    for i in range(3):
        conv(f"dec_in{i}", 256, 256, 1, "none")
    lin("enc_out.l", 256, 256)
    ln("enc_out.ln")
    lin("score_head", 256, 25)
    lin("mq.0", 256, 256)
    lin("mq.1", 256, 256)
    lin("mq.2", 256, 32)
    lin("qpos.0", 4, 512)
    lin("qpos.1", 512, 256)
    for i in range(6):
        d = f"dec{i}"
        for n in ("q", "k", "v", "o"):
            lin(f"{d}.sa.{n}", 256, 256)
        ln(f"{d}.ln1")
        ln(f"{d}.ln2")
        ln(f"{d}.ln3")
        lin(f"{d}.ca.so", 256, 192)
        lin(f"{d}.ca.aw", 256, 96)
        lin(f"{d}.ca.vp", 256, 256)
        lin(f"{d}.ca.op", 256, 256)
        lin(f"{d}.fc1", 256, DEC_FFN)
        lin(f"{d}.fc2", DEC_FFN, 256)
    lin("bbox_head.0", 256, 256)
    lin("bbox_head.1", 256, 256)
    lin("bbox_head.2", 256, 4)
    ln("dec_norm")
    lin("order5", 256, 256)
    lin("gp", 256, 128)
    return m


def make_weights(seed: int = 0) -> "OrderedDict[str, np.ndarray]":
    rng = np.random.default_rng(seed)
    out: "OrderedDict[str, np.ndarray]" = OrderedDict()
    gain = {"relu": 2.0, "silu": 2.0, "none": 1.0, "half": 0.5}
    for name, spec in manifest().items():
        kind, shape = spec[0], spec[1]
        if kind in ("conv", "dwconv"):
            fan_in = shape[1] * shape[2] * shape[3]
            g = gain[spec[2]]
            if name.endswith(".agg1.weight") and (".b1." in name or ".b2." in name):
                g *= 0.5  # the block output is added to a residual of equal variance
            a = rng.standard_normal(shape) * np.sqrt(g / fan_in)
        elif kind == "linear":
            a = rng.standard_normal(shape) * np.sqrt(2.0 / (shape[0] + shape[1]))
        elif kind == "ln":
            a = 1.0 + 0.05 * rng.standard_normal(shape)
        elif name == "enc_out.l.bias":
            # masked (border) memory tokens are exactly zero; a zero bias maps
            # them to the LayerNorm offset, i.e. low class logits, as a trained
            # model's two-stage selection does
            a = np.zeros(shape)
        else:
            a = 0.05 * rng.standard_normal(shape)
        out[name] = a.astype(np.float32)
    return out


def write_gguf(path: str, seed: int = 0) -> str:
    """Write the seeded weights as an F32 GGUF in the converter's layout
    (scripts/convert.py:132-143)."""
    import gguf
    w = make_weights(seed)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    wr = gguf.GGUFWriter(path, "pp-doclayout-v3")
    wr.add_description(f"PP-DocLayoutV3 F32, BN folded, synthetic seed {seed}")
    wr.add_uint32("ppdlv3.d_model", 256)
    wr.add_uint32("ppdlv3.decoder_layers", 6)
    wr.add_uint32("ppdlv3.num_queries", 300)
    wr.add_uint32("ppdlv3.num_classes", 25)
    for name in sorted(w):
        wr.add_tensor(name, np.ascontiguousarray(w[name]))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    return path


def cached_gguf(seed: int = 0, cache_dir: str | None = None) -> str:
    """Path of the seeded GGUF, generated on first use."""
    cache_dir = cache_dir or os.environ.get("PPDL_SYNTH_DIR") or os.path.join(
        os.path.expanduser("~"), ".cache", "ppdl_b200")
    path = os.path.join(cache_dir, f"ppdlv3_synth_s{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_gguf(tmp, seed)
        os.replace(tmp, path)
    return path


def synth_page(seed: int) -> np.ndarray:
    """Config 0 page: 3x800x800 CHW f32 in [0,1] — white background, 20-60
    dark rectangles U[0,0.3] with sides of 10-400 px, N(0,0.01) noise."""
    rng = np.random.default_rng(seed)
    img = np.ones((3, 800, 800), np.float32)
    for _ in range(int(rng.integers(20, 61))):
        h, w = rng.integers(10, 401, 2)
        y, x = rng.integers(0, 800 - h + 1), rng.integers(0, 800 - w + 1)
        img[:, y:y + h, x:x + w] = rng.uniform(0.0, 0.3, (3, 1, 1)).astype(np.float32)
    img += rng.normal(0.0, 0.01, img.shape).astype(np.float32)
    return np.clip(img, 0.0, 1.0).astype(np.float32)
