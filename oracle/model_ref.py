"""CPU restatement of the whole PP-DocLayoutV3 forward (TEST INFRASTRUCTURE).

Follows the reference graph builder of caojiachen1/ppdoclayout-ggml
(src/ppdoclayout.cpp:388-882) and its host postprocess (:927-993) node by
node, in FP32 on the CPU with torch ops as the dense kernels (conv2d,
matmul, layer_norm, interpolate).  The hot-path operators — MSDeformAttn,
mask->box, top-300, the host constants and the postprocess — go through
the C restatement in ppdl_oracle.c, which is pinned bit-exactly against the
reference's own CPU ops (tests/test_oracle.py).

The reference ggml runtime itself cannot be built here (its ggml submodule
is absent), so the dense parts of this restatement are unpinned: they follow
the op semantics of ggml as documented in each helper below.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import oracle as _oracle

NQ, NC, DM, NH, HD = 300, 25, 256, 8, 32


def load_gguf(path: str) -> dict:
    """GGUF tensors as torch float32 in torch order (reversed ggml ne)."""
    import gguf
    r = gguf.GGUFReader(path)
    out = {}
    for t in r.tensors:
        shape = [int(x) for x in reversed(list(t.shape))]
        a = np.asarray(t.data, dtype=np.float32).reshape(shape)
        out[t.name] = torch.from_numpy(a.copy())
    return out


LVL = ((100, 100, 0), (50, 50, 10000), (25, 25, 12500))


def msdeform_t(value, off, awr, ref):
    """Torch restatement of op_msdeform (src/ppdoclayout.cpp:142-198) in the
    dtype of its inputs (used for the float64 oracle): value [13125,256],
    off [nq,192], awr [nq,96], ref [nq,4] -> [nq,256]."""
    nq = off.shape[0]
    w = torch.softmax(awr.reshape(nq, NH, 12), dim=-1)
    off = off.reshape(nq, NH, 3, 4, 2)
    v = value.reshape(-1, NH, HD)
    out = torch.zeros((nq, NH, HD), dtype=value.dtype)
    hidx = torch.arange(NH).view(1, NH, 1)
    for l, (W, H, st) in enumerate(LVL):
        lx = ref[:, 0].view(nq, 1, 1) + off[:, :, l, :, 0] / 4 * ref[:, 2].view(nq, 1, 1) * 0.5
        ly = ref[:, 1].view(nq, 1, 1) + off[:, :, l, :, 1] / 4 * ref[:, 3].view(nq, 1, 1) * 0.5
        fx, fy = lx * W - 0.5, ly * H - 0.5
        x0, y0 = torch.floor(fx), torch.floor(fy)
        tx, ty = fx - x0, fy - y0
        x0, y0 = x0.long(), y0.long()
        wl = w[:, :, l * 4:(l + 1) * 4]
        for k in range(4):
            dx, dy = k & 1, k >> 1
            cw = (tx if dx else 1 - tx) * (ty if dy else 1 - ty)
            xx, yy = x0 + dx, y0 + dy
            ok = (xx >= 0) & (xx < W) & (yy >= 0) & (yy < H) & (cw != 0)
            tok = (st + yy.clamp(0, H - 1) * W + xx.clamp(0, W - 1))       # [nq, NH, 4]
            rows = v[tok, hidx.expand_as(tok)]                               # [nq, NH, 4, HD]
            coef = (wl * cw * ok).unsqueeze(-1)
            out += (coef * rows).sum(2)
    return out.reshape(nq, DM)


def mask_box_t(ml):
    """op_mask_box (src/ppdoclayout.cpp:98-140) in torch: [nq,40000] -> [nq,4]."""
    pos = (ml > 0).reshape(-1, 200, 200)
    out = torch.zeros((pos.shape[0], 4), dtype=ml.dtype)
    ar = torch.arange(200, dtype=ml.dtype)
    for q in range(pos.shape[0]):
        ys, xs = pos[q].any(1), pos[q].any(0)
        if not bool(xs.any()):
            b = torch.zeros(4, dtype=ml.dtype)
        else:
            b = torch.stack([ar[xs].min(), ar[ys].min(), ar[xs].max() + 1, ar[ys].max() + 1]) / 200
        c = torch.stack([(b[0] + b[2]) * 0.5, (b[1] + b[3]) * 0.5, b[2] - b[0], b[3] - b[1]])
        c = c.clamp(0, 1)
        out[q] = torch.log(c.clamp(min=1e-5) / (1 - c).clamp(min=1e-5))
    return out


def topk_t(lg, nq=NQ):
    """op_topk300 (src/ppdoclayout.cpp:73-96): stable descending sort of the
    per-token max logit, ties to the lower index."""
    mx = lg.max(dim=1).values
    return torch.sort(-mx, stable=True).indices[:nq].numpy().astype(np.int32)


class RefModel:
    """Forward of one page: image [3,800,800] -> raw outputs + dets.

    dtype=torch.float32 is the FP32 restatement (dense ops in torch FP32,
    hot-path ops through the pinned C restatement); dtype=torch.float64
    evaluates the same graph in double precision (hot-path ops through the
    torch restatements above) as an exact-arithmetic reference; the discrete
    postprocess runs on its outputs rounded to FP32."""

    def __init__(self, weights: dict, threads: int | None = None, dtype=torch.float32):
        self.dtype = dtype
        self.w = {k: v.to(dtype) for k, v in weights.items()}
        if threads:
            torch.set_num_threads(threads)
        o = _oracle()
        self.o = o
        self.pos = torch.from_numpy(o.pos_embed()).to(dtype)
        self.valid = torch.from_numpy(o.valid_mask()).to(dtype)
        if dtype == torch.float64:   # the constants in float64 math (:887-923)
            om = 1.0 / np.power(10000.0, np.arange(64) / 64.0)
            hh, ww = np.meshgrid(np.arange(25), np.arange(25), indexing="ij")
            h, w_ = hh.reshape(-1, 1) * om, ww.reshape(-1, 1) * om
            self.pos = torch.from_numpy(np.concatenate(
                [np.sin(h), np.cos(h), np.sin(w_), np.cos(w_)], 1)).to(dtype)

    # ---- building blocks (src/ppdoclayout.cpp:379-594) ----------------------
    @staticmethod
    def act(x, a):
        if a == 1:
            return torch.relu(x)
        if a == 2:
            return x / (1.0 + torch.exp(-x))   # ggml_silu, patch:429
        return x

    def conv(self, x, name, s, p, a, pad_hi=None):
        """builder::conv (:388-543): every path computes the same zero-padded
        cross-correlation + bias + activation.  x [C,H,W]."""
        w = self.w[name + ".weight"]
        b = self.w[name + ".bias"]
        groups = x.shape[0] if w.shape[1] == 1 and x.shape[0] != 1 else 1
        y = F.conv2d(x[None], w, b, stride=s, padding=p, groups=groups)[0]
        return self.act(y, a)

    def lin(self, x, name):
        """ggml_mul_mat(W, x) + b (:545-548); x [T, in] -> [T, out]."""
        return x @ self.w[name + ".weight"].T + self.w[name + ".bias"]

    def ln(self, x, name):
        """ggml_norm eps 1e-5, * weight + bias (:550-554)."""
        return F.layer_norm(x, (x.shape[-1],), self.w[name + ".weight"], self.w[name + ".bias"],
                            eps=1e-5)

    def mlp3(self, x, pfx):
        x = torch.relu(self.lin(x, pfx + ".0"))
        x = torch.relu(self.lin(x, pfx + ".1"))
        return self.lin(x, pfx + ".2")

    @staticmethod
    def to_seq(x):
        """CHW -> [H*W, C], token = y*W + x (:566-569)."""
        return x.permute(1, 2, 0).reshape(-1, x.shape[0])

    def mha(self, qk_in, v_in, pfx):
        """8 heads x 32, softmax(q k^T * 1/sqrt(32)) v, then .o (:572-587)."""
        T = qk_in.shape[0]
        q = self.lin(qk_in, pfx + ".q").reshape(T, NH, HD).permute(1, 0, 2)
        k = self.lin(qk_in, pfx + ".k").reshape(T, NH, HD).permute(1, 0, 2)
        v = self.lin(v_in, pfx + ".v").reshape(T, NH, HD).permute(1, 0, 2)
        scale = 1.0 / np.sqrt(HD)
        if self.dtype == torch.float32:
            scale = float(np.float32(scale))  # ggml_scale's float factor
        kq = torch.softmax((q @ k.transpose(1, 2)) * scale, dim=-1)
        o = (kq @ v).permute(1, 0, 2).reshape(T, DM)
        return self.lin(o, pfx + ".o")

    @staticmethod
    def inv_sigmoid(x):
        """(:589-594): log(clamp(x,1e-5,1)) - log(clamp(1-x,1e-5,1)) after clamp [0,1]."""
        x = x.clamp(0.0, 1.0)
        return torch.log(x.clamp(1e-5, 1.0)) - torch.log((1.0 - x).clamp(1e-5, 1.0))

    @staticmethod
    def interp(x, h, w, mode):
        """ggml_interpolate (:670-672).  NEAREST: src = floor(dst / sf);
        BILINEAR without align-corners: src = (dst + 0.5) / sf - 0.5 with the
        edge clamp — the same sampling as torch's align_corners=False."""
        if mode == "nearest":
            return F.interpolate(x[None], size=(h, w), mode="nearest")[0]
        return F.interpolate(x[None], size=(h, w), mode="bilinear", align_corners=False)[0]

    # ---- backbone (:598-652) --------------------------------------------------
    def hg_block(self, x, pfx, light):
        cat = [x]
        cur = x
        for l in range(6):
            lp = f"{pfx}.l{l}"
            if light:
                cur = self.conv(cur, lp + ".c1", 1, 0, 0)
                cur = self.conv(cur, lp + ".c2", 1, 2, 1)
            else:
                cur = self.conv(cur, lp, 1, 1, 1)
            cat.append(cur)
        y = self.conv(torch.cat(cat, 0), pfx + ".agg0", 1, 0, 1)
        return self.conv(y, pfx + ".agg1", 1, 0, 1)

    def backbone(self, img):
        x = self.conv(img, "stem1", 2, 1, 1)                  # 400, 32
        xp = F.pad(x, (0, 1, 0, 1))                            # ggml_pad right/bottom
        a = self.conv(xp, "stem2a", 1, 0, 1)
        a = self.conv(F.pad(a, (0, 1, 0, 1)), "stem2b", 1, 0, 1)
        pl = F.max_pool2d(xp[None], 2, 1)[0]
        x = torch.cat([pl, a], 0)                               # 400, 64
        x = self.conv(x, "stem3", 2, 1, 1)                    # 200, 32
        x = self.conv(x, "stem4", 1, 0, 1)                    # 200, 48
        s0 = self.hg_block(x, "st0.b0", False)
        s1 = self.hg_block(self.conv(s0, "st1.ds", 2, 1, 0), "st1.b0", False)
        s2 = self.hg_block(self.conv(s1, "st2.ds", 2, 1, 0), "st2.b0", True)
        s2 = self.hg_block(s2, "st2.b1", True) + s2
        s2 = self.hg_block(s2, "st2.b2", True) + s2
        s3 = self.hg_block(self.conv(s2, "st3.ds", 2, 1, 0), "st3.b0", True)
        return s0, s1, s2, s3

    # ---- encoder (:656-729) ---------------------------------------------------
    def repvgg(self, x, pfx):
        return self.act(self.conv(x, pfx + ".c1", 1, 1, 0) + self.conv(x, pfx + ".c2", 1, 0, 0), 2)

    def csp(self, x, pfx):
        a = self.conv(x, pfx + ".c1", 1, 0, 2)
        for i in range(3):
            a = self.repvgg(a, f"{pfx}.bn{i}")
        return a + self.conv(x, pfx + ".c2", 1, 0, 2)

    def encoder(self, x4, p8r, p16r, p32r):
        p8 = self.conv(p8r, "enc_in0", 1, 0, 0)
        p16 = self.conv(p16r, "enc_in1", 1, 0, 0)
        p32 = self.conv(p32r, "enc_in2", 1, 0, 0)
        s = self.to_seq(p32)
        at = self.mha(s + self.pos, s, "aifi")
        s = self.ln(s + at, "aifi.ln1")
        ff = self.lin(F.gelu(self.lin(s, "aifi.fc1")), "aifi.fc2")   # gelu_erf
        s = self.ln(s + ff, "aifi.ln2")
        p32 = s.reshape(25, 25, DM).permute(2, 0, 1).contiguous()
        lat0 = self.conv(p32, "lat0", 1, 0, 2)
        f16 = self.csp(torch.cat([self.interp(lat0, 50, 50, "nearest"), p16], 0), "fpn0")
        lat1 = self.conv(f16, "lat1", 1, 0, 2)
        f8 = self.csp(torch.cat([self.interp(lat1, 100, 100, "nearest"), p8], 0), "fpn1")
        n16 = self.csp(torch.cat([self.conv(f8, "pand0", 2, 1, 2), lat1], 0), "pan0")
        n32 = self.csp(torch.cat([self.conv(n16, "pand1", 2, 1, 2), lat0], 0), "pan1")
        h0 = self.conv(f8, "mh0.0", 1, 1, 2)
        h1 = self.interp(self.conv(n16, "mh1.0", 1, 1, 2), 100, 100, "bilinear")
        h2 = self.interp(self.conv(n32, "mh2.0", 1, 1, 2), 50, 50, "bilinear")
        h2 = self.interp(self.conv(h2, "mh2.2", 1, 1, 2), 100, 100, "bilinear")
        mf = self.conv((h0 + h1) + h2, "mh.out", 1, 1, 2)
        mf = self.interp(mf, 200, 200, "bilinear")
        mf = mf + self.conv(x4, "mlat", 1, 1, 2)
        mf = self.conv(mf, "mout.base", 1, 1, 2)
        mf = self.conv(mf, "mout.conv", 1, 0, 0)                       # 32, 200, 200
        return f8, n16, n32, mf

    # ---- full graph (:733-882) + postprocess (:927-993) -----------------------
    @torch.no_grad()
    def forward(self, image: np.ndarray, ori_h: int = 800, ori_w: int = 800, want_masks=True):
        img = torch.from_numpy(np.ascontiguousarray(image, dtype=np.float32)).to(self.dtype)
        f64 = self.dtype == torch.float64
        x4, p8, p16, p32 = self.backbone(img)
        f8, n16, n32, mfeat = self.encoder(x4, p8, p16, p32)
        mflat = mfeat.reshape(32, -1)                                   # [c][p]
        source = torch.cat([self.to_seq(self.conv(f8, "dec_in0", 1, 0, 0)),
                            self.to_seq(self.conv(n16, "dec_in1", 1, 0, 0)),
                            self.to_seq(self.conv(n32, "dec_in2", 1, 0, 0))], 0)
        memory = source * self.valid[:, None]
        om = self.ln(self.lin(memory, "enc_out.l"), "enc_out.ln")
        ecls = self.lin(om, "score_head")                               # [13125][25]
        topk = topk_t(ecls) if f64 else self.o.topk(np.ascontiguousarray(ecls.numpy())[None])[0]
        target = om[torch.from_numpy(topk.astype(np.int64))]
        mq0 = self.mlp3(self.ln(target, "dec_norm"), "mq")              # [300][32]
        encm = (mq0 @ mflat).contiguous()                                # [300][40000]
        refu = mask_box_t(encm) if f64 else torch.from_numpy(self.o.mask_box(encm.numpy()[None])[0])
        ref = torch.sigmoid(refu)
        x = target
        for i in range(6):
            d = f"dec{i}"
            qpos = self.lin(torch.relu(self.lin(ref, "qpos.0")), "qpos.1")
            x = self.ln(x + self.mha(x + qpos, x, d + ".sa"), d + ".ln1")
            z = x + qpos
            value = self.lin(source, d + ".ca.vp")
            offs = self.lin(z, d + ".ca.so")
            aw = self.lin(z, d + ".ca.aw")
            if f64:
                ca = msdeform_t(value, offs, aw, ref)
            else:
                ca = torch.from_numpy(self.o.msdeform(
                    np.ascontiguousarray(value.numpy())[None],
                    np.ascontiguousarray(offs.numpy())[None],
                    np.ascontiguousarray(aw.numpy())[None],
                    np.ascontiguousarray(ref.numpy())[None])[0])
            x = self.ln(x + self.lin(ca, d + ".ca.op"), d + ".ln2")
            ff = self.lin(torch.relu(self.lin(x, d + ".fc1")), d + ".fc2")
            x = self.ln(x + ff, d + ".ln3")
            delta = self.mlp3(x, "bbox_head")
            ref = torch.sigmoid(delta + self.inv_sigmoid(ref))
        outq = self.ln(x, "dec_norm")
        logits = self.lin(outq, "score_head")
        masks = (self.mlp3(outq, "mq") @ mflat).contiguous() if want_masks else None
        gp = self.lin(self.lin(x, "order5"), "gp")
        qv, kv = gp[:, :64], gp[:, 64:]
        order = (qv @ kv.T) / 8.0   # order[i][j] = q_i . k_j / 8  -> flat [j + 300 i]
        res = {
            "logits": logits.numpy().astype(np.float32),
            "boxes": ref.numpy().astype(np.float32),
            "order": np.ascontiguousarray(order.numpy().astype(np.float32)).reshape(-1),
            "topk": topk,
            "enc_max": ecls.max(1).values.double().numpy(),
            "init_ref_unact": refu.numpy(),
        }
        if want_masks:
            res["mask_logits"] = masks.numpy().astype(np.float32)
            dets, m, sel = self.o.postprocess(res["logits"], res["boxes"], res["order"],
                                              res["mask_logits"], ori_h, ori_w)
            res.update(dets=dets, masks=m, sel=sel)
        return res
