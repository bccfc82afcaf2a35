/*
 * ppdl_oracle.c — CPU restatement of the PP-DocLayoutV3 hot-path operators.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker / the timed CPU arm.
 *
 * Every function restates one operator of caojiachen1/ppdoclayout-ggml in
 * plain C with the same arithmetic order as the reference CPU op (or, where
 * the reference only has a GPU kernel, as that kernel), and cites the
 * reference file:line it follows.  Paths are relative to the reference
 * project root.  The reference's CPU custom ops are additionally compiled
 * from the reference sources into oracle/_ref/ (see oracle/Makefile) and the
 * tests pin this restatement against them and against committed golden
 * vectors made from them.
 *
 * Built with -ffp-contract=off so that a*b+c stays a separate multiply and
 * add wherever the reference writes it that way; fmaf() marks the places
 * where the reference kernel fuses.
 *
 * Layouts follow ggml's ne order read as row-major C arrays: a ggml tensor
 * ne(a, b, c) is the C array [c][b][a].  An optional leading batch dimension
 * (pages) is added by this restatement; the reference runs batch 1.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define NQ 300
#define NC 25
#define DM 256
#define NH 8
#define HD 32
#define NLVL 3
#define NPTS 4
#define MASK_HW 200
#define MASK_PIX (MASK_HW * MASK_HW)
#define NTOK 13125

static const int LVL_W[3] = {100, 50, 25};
static const int LVL_H[3] = {100, 50, 25};
static const int LVL_START[3] = {0, 10000, 12500};

#ifdef _OPENMP
#define OMP_FOR _Pragma("omp parallel for schedule(static)")
#else
#define OMP_FOR
#endif

/* ------------------------------------------------------------------ MSDA --
 * In-model form, src/ppdoclayout.cpp:142-198 (op_msdeform):
 *   value  [b][13125][256]  (t*256 + h*32 + c)
 *   off    [b][nq][192]     ((h*3+l)*4+p)*2 + xy
 *   awr    [b][nq][96]      pre-softmax, h*12 + l*4 + p
 *   ref    [b][nq][4]       cxcywh in sigmoid space
 *   out    [b][nq][256]
 * Softmax max/exp/sum/divide as :163-167; location as :174-175; bilinear
 * grid_sample (zeros padding, align_corners=false) as :177-192 with the
 * corner skip rule "out of bounds or corner weight == 0".  Accumulation per
 * channel in l -> p -> corner order with a separate multiply and add. */
static void msda_one(const float *val, const float w[12], const float *locx,
                     const float *locy, int h, float *oq)
{
    for (int l = 0; l < NLVL; l++) {
        const int W = LVL_W[l], H = LVL_H[l], st = LVL_START[l];
        for (int p = 0; p < NPTS; p++) {
            const float lx = locx[l * 4 + p], ly = locy[l * 4 + p];
            const float fx = lx * W - 0.5f;
            const float fy = ly * H - 0.5f;
            const int x0 = (int)floorf(fx), y0 = (int)floorf(fy);
            const float tx = fx - x0, ty = fy - y0;
            const float wt = w[l * 4 + p];
            const float cw[4] = {(1 - tx) * (1 - ty), tx * (1 - ty), (1 - tx) * ty, tx * ty};
            const int xs[4] = {x0, x0 + 1, x0, x0 + 1};
            const int ys[4] = {y0, y0, y0 + 1, y0 + 1};
            for (int k = 0; k < 4; k++) {
                const int xx = xs[k], yy = ys[k];
                if (xx < 0 || xx >= W || yy < 0 || yy >= H || cw[k] == 0.0f) continue;
                const float *v = val + ((size_t)(st + yy * W + xx) * DM) + h * HD;
                const float ww = wt * cw[k];
                for (int c = 0; c < HD; c++) oq[h * HD + c] += ww * v[c];
            }
        }
    }
}

void oracle_msdeform(const float *val, const float *off, const float *awr,
                     const float *ref, float *out, int nq, int batch)
{
    for (int b = 0; b < batch; b++) {
        const float *vb = val + (size_t)b * NTOK * DM;
        OMP_FOR
        for (int q = 0; q < nq; q++) {
            const float *rq = ref + ((size_t)b * nq + q) * 4;
            const float *oo = off + ((size_t)b * nq + q) * 192;
            float *oq = out + ((size_t)b * nq + q) * DM;
            memset(oq, 0, DM * sizeof(float));
            for (int h = 0; h < NH; h++) {
                const float *a = awr + ((size_t)b * nq + q) * 96 + h * 12;
                float amax = a[0];
                for (int i = 1; i < 12; i++) amax = fmaxf(amax, a[i]);
                float w[12], wsum = 0.0f;
                for (int i = 0; i < 12; i++) { w[i] = expf(a[i] - amax); wsum += w[i]; }
                for (int i = 0; i < 12; i++) w[i] /= wsum;
                float locx[12], locy[12];
                for (int l = 0; l < NLVL; l++)
                    for (int p = 0; p < NPTS; p++) {
                        const float ox = oo[((h * 3 + l) * 4 + p) * 2 + 0];
                        const float oy = oo[((h * 3 + l) * 4 + p) * 2 + 1];
                        locx[l * 4 + p] = rq[0] + ox / NPTS * rq[2] * 0.5f;
                        locy[l * 4 + p] = rq[1] + oy / NPTS * rq[3] * 0.5f;
                    }
                msda_one(vb, w, locx, locy, h, oq);
            }
        }
    }
}

/* Canonical (PyTorch MSDeformAttn) form of the same sampling core: sampling
 * locations are given directly in [0,1] and the weights are already
 * softmax-normalised.  Identical bilinear rule and accumulation order as the
 * in-model form above (src/ppdoclayout.cpp:169-194).
 *   loc [b][nq][8][3][4][2], w [b][nq][8][12]. */
void oracle_msdeform_canon(const float *val, const float *loc, const float *wts,
                           float *out, int nq, int batch)
{
    for (int b = 0; b < batch; b++) {
        const float *vb = val + (size_t)b * NTOK * DM;
        OMP_FOR
        for (int q = 0; q < nq; q++) {
            float *oq = out + ((size_t)b * nq + q) * DM;
            memset(oq, 0, DM * sizeof(float));
            for (int h = 0; h < NH; h++) {
                const float *lq = loc + (((size_t)b * nq + q) * NH + h) * 24;
                const float *wq = wts + (((size_t)b * nq + q) * NH + h) * 12;
                float locx[12], locy[12], w[12];
                for (int i = 0; i < 12; i++) {
                    locx[i] = lq[2 * i];
                    locy[i] = lq[2 * i + 1];
                    w[i] = wq[i];
                }
                msda_one(vb, w, locx, locy, h, oq);
            }
        }
    }
}

/* ------------------------------------------------------------- mask->box --
 * src/ppdoclayout.cpp:98-140 (op_mask_box): bbox of logit>0 pixels of each
 * 200x200 mask, [xmin, ymin, xmax+1, ymax+1]/200 -> cxcywh -> inverse
 * sigmoid with the clamp/1e-5 guards of :105-110.  Empty mask -> box 0. */
static float invsig(float x)
{
    x = fminf(fmaxf(x, 0.0f), 1.0f);
    const float x1 = fmaxf(x, 1e-5f);
    const float x2 = fmaxf(1.0f - x, 1e-5f);
    return logf(x1 / x2);
}

void oracle_mask_box(const float *ml, float *out, int nq, int batch)
{
    const int n = nq * batch;
    OMP_FOR
    for (int q = 0; q < n; q++) {
        const float *m = ml + (size_t)q * MASK_PIX;
        float xmin = FLT_MAX, ymin = FLT_MAX, xmax = -FLT_MAX, ymax = -FLT_MAX;
        int any = 0;
        for (int y = 0; y < MASK_HW; y++) {
            const float *row = m + (size_t)y * MASK_HW;
            for (int x = 0; x < MASK_HW; x++) {
                if (row[x] > 0.0f) {
                    any = 1;
                    xmin = fminf(xmin, (float)x);
                    xmax = fmaxf(xmax, (float)x);
                    ymin = fminf(ymin, (float)y);
                    ymax = fmaxf(ymax, (float)y);
                }
            }
        }
        float bx0, by0, bx1, by1;
        if (!any) {
            bx0 = by0 = bx1 = by1 = 0.0f;
        } else {
            bx0 = xmin; by0 = ymin; bx1 = xmax + 1.0f; by1 = ymax + 1.0f;
        }
        bx0 /= MASK_HW; bx1 /= MASK_HW; by0 /= MASK_HW; by1 /= MASK_HW;
        const float cx = (bx0 + bx1) * 0.5f, cy = (by0 + by1) * 0.5f;
        const float bw = bx1 - bx0, bh = by1 - by0;
        float *o = out + (size_t)q * 4;
        o[0] = invsig(cx); o[1] = invsig(cy); o[2] = invsig(bw); o[3] = invsig(bh);
    }
}

/* ---------------------------------------------------------------- top-300 --
 * src/ppdoclayout.cpp:73-96 (op_topk300): per token the max class logit,
 * then the nq tokens with the largest maxima, descending, ties to the lower
 * token index.  Keys are unique under that order, so a full sort gives the
 * same prefix as the reference's partial_sort. */
static const float *g_topk_mx;
static int topk_cmp(const void *pa, const void *pb)
{
    const int a = *(const int *)pa, b = *(const int *)pb;
    const float ma = g_topk_mx[a], mb = g_topk_mx[b];
    if (ma != mb) return ma > mb ? -1 : 1;
    return a < b ? -1 : (a > b ? 1 : 0);
}

void oracle_topk(const float *lg, int32_t *out, int ntok, int nc, int nq, int batch)
{
    float *mx = (float *)malloc(sizeof(float) * ntok);
    int *idx = (int *)malloc(sizeof(int) * ntok);
    for (int b = 0; b < batch; b++) {
        const float *lb = lg + (size_t)b * ntok * nc;
        for (int q = 0; q < ntok; q++) {
            const float *p = lb + (size_t)q * nc;
            float m = p[0];
            for (int c = 1; c < nc; c++) m = (m < p[c]) ? p[c] : m; /* std::max */
            mx[q] = m;
            idx[q] = q;
        }
        g_topk_mx = mx;
        qsort(idx, ntok, sizeof(int), topk_cmp);
        for (int i = 0; i < nq; i++) out[(size_t)b * nq + i] = idx[i];
    }
    free(mx);
    free(idx);
}

/* ------------------------------------------------------ Winograd F(4,3) --
 * Transform matrices of the reference's F(4,3) (numerically solved,
 * row-balanced): B4 is 6x6 (patches/ggml-ppdl.patch:165-172), G4 is 6x3
 * (src/ppdoclayout.cpp:313-320, patch:173-180), A4 is 6x4 (patch:181-188).
 * They are part of the data format of the reference's op 10/11/12 planes and
 * of the ".wg4" repacked weights, so the values are the same here. */
static const float WG_B4[36] = {
     0.156081140f, -0.005399639f, -0.912340343f, -0.209068865f,  0.695356965f,  0.124203928f,
    -0.153710172f, -0.110961877f,  0.797504783f,  0.794400156f,  0.002377054f, -0.019845223f,
     0.423170745f, -0.936912060f, -0.566737831f,  0.947692990f,  0.041719031f, -0.024267767f,
    -0.338096678f,  0.120876059f,  1.953236461f, -0.181245893f, -1.540627480f,  0.223424435f,
     0.295037359f,  0.647394836f, -0.185275897f, -0.582640827f, -0.011674470f,  0.014480385f,
     0.198828861f, -0.241681889f, -0.911203325f,  0.846514463f,  0.049163014f, -0.022408651f,
};
static const float WG_G4[18] = {
    -0.019582119f, -0.133662105f, -0.912340343f,
     0.650278211f,  0.720138848f,  0.797504783f,
    -0.947692990f,  0.466171294f, -0.229310215f,
     0.060792211f, -0.344588995f,  1.953236461f,
     0.647394836f,  0.272543609f,  0.114736818f,
    -0.911203325f,  0.880876958f, -0.851559937f,
};
static const float WG_A4[24] = {
    -0.015757650f, -0.107557341f, -0.734156489f, -5.011147976f,
     0.878285885f,  0.972641826f,  1.077134609f,  1.192853332f,
    -1.655853987f,  0.814516485f, -0.400661618f,  0.197085932f,
    -0.005868433f,  0.033264086f, -0.188551068f,  1.068765521f,
     3.145301104f,  1.324125051f,  0.557437003f,  0.234672695f,
     0.978109479f, -0.945556402f,  0.914086699f, -0.883664429f,
};

const float *oracle_wg4_matrix(int which)
{
    return which == 0 ? WG_B4 : (which == 1 ? WG_G4 : WG_A4);
}

/* Filter transform (src/ppdoclayout.cpp:312-337):
 *   w   [oc][ic][3][3]  (ggml ne(3,3,IC,OC))
 *   wg4 [36][ic][oc],   plane u*6+v = sum_ab G[u][a] G[v][b] w[oc][ic][a][b]
 * with the product evaluated as (G[u][a] * G[v][b]) * w, accumulated in
 * a -> b order in float. */
void oracle_wg4_filter(const float *w, float *wg4, int IC, int OC)
{
    OMP_FOR
    for (int uv = 0; uv < 36; uv++) {
        const int u = uv / 6, v = uv % 6;
        for (int ic = 0; ic < IC; ic++)
            for (int oc = 0; oc < OC; oc++) {
                float s = 0.0f;
                for (int a = 0; a < 3; a++)
                    for (int b = 0; b < 3; b++) {
                        const size_t sidx = (((size_t)oc * IC + ic) * 3 + a) * 3 + b;
                        s += WG_G4[u * 3 + a] * WG_G4[v * 3 + b] * w[sidx];
                    }
                wg4[((size_t)uv * IC + ic) * OC + oc] = s;
            }
    }
}

/* Input transform (patch:496-547 ppdl_wg_input_kernel<6,4>): x is the
 * padded input [IC][IH][IW] (left/top pad 1, right/bottom completing the
 * 4x4 output-tile grid, src/ppdoclayout.cpp:432-439); per (ic, tile) the 6x6
 * patch d at (4*ty, 4*tx) becomes B d B^T with fmaf in the kernel's order;
 * dt [36][IC][T], T = TW*TH, tile = ty*TW + tx. */
void oracle_wg4_input(const float *x, float *dt, int IW, int IH, int IC, int TW, int TH)
{
    const int T = TW * TH;
    OMP_FOR
    for (int ic = 0; ic < IC; ic++) {
        for (int tile = 0; tile < T; tile++) {
            const int ty = tile / TW, tx = tile - ty * TW;
            float d[6][6], t1[6][6];
            for (int a = 0; a < 6; a++)
                for (int b = 0; b < 6; b++)
                    d[a][b] = x[((size_t)ic * IH + 4 * ty + a) * IW + 4 * tx + b];
            for (int u = 0; u < 6; u++)
                for (int v = 0; v < 6; v++) {
                    float s = 0.0f;
                    for (int a = 0; a < 6; a++) s = fmaf(WG_B4[u * 6 + a], d[a][v], s);
                    t1[u][v] = s;
                }
            for (int u = 0; u < 6; u++)
                for (int w = 0; w < 6; w++) {
                    float s = 0.0f;
                    for (int b = 0; b < 6; b++) s = fmaf(t1[u][b], WG_B4[w * 6 + b], s);
                    dt[((size_t)(u * 6 + w) * IC + ic) * T + tile] = s;
                }
        }
    }
}

/* 36-plane madd (patch:787-802, cuBLAS strided-batched SGEMM there):
 *   yt[p][oc][t] = sum_ic dt[p][ic][t] * wg4[p][ic][oc], accumulated in
 *   double and rounded once (the reference's cuBLAS order is not known). */
void oracle_wg4_madd(const float *dt, const float *wg4, float *yt, int T, int IC, int OC)
{
    OMP_FOR
    for (int poc = 0; poc < 36 * OC; poc++) {
        const int p = poc / OC, oc = poc % OC;
        double *acc = (double *)calloc((size_t)T, sizeof(double));
        for (int ic = 0; ic < IC; ic++) {
            const double wv = wg4[((size_t)p * IC + ic) * OC + oc];
            const float *dr = dt + ((size_t)p * IC + ic) * T;
            for (int t = 0; t < T; t++) acc[t] += wv * (double)dr[t];
        }
        float *yr = yt + ((size_t)p * OC + oc) * T;
        for (int t = 0; t < T; t++) yr[t] = (float)acc[t];
        free(acc);
    }
}

static float apply_act(float v, int act)
{
    if (act == 1) return fmaxf(v, 0.0f);
    if (act == 2) return v / (1.0f + expf(-v));
    return v;
}

/* Output transform + bias + activation (patch:549-610
 * ppdl_wg_output_kernel<6,4>): Y = A^T m A + bias[oc], act 0/1/2 =
 * none/ReLU/SiLU, stored CHW [OC][OH][OW] with the tile tail clipped. */
void oracle_wg4_output(const float *yt, const float *bias, float *out, int T, int TW,
                       int OC, int OW, int OH, int act)
{
    OMP_FOR
    for (int oc = 0; oc < OC; oc++) {
        for (int tile = 0; tile < T; tile++) {
            const int ty = tile / TW, tx = tile - ty * TW;
            float m[36], t1[4][6], Y[4][4];
            for (int p = 0; p < 36; p++) m[p] = yt[((size_t)p * OC + oc) * T + tile];
            for (int i = 0; i < 4; i++)
                for (int v = 0; v < 6; v++) {
                    float s = 0.0f;
                    for (int u = 0; u < 6; u++) s = fmaf(WG_A4[u * 4 + i], m[u * 6 + v], s);
                    t1[i][v] = s;
                }
            for (int i = 0; i < 4; i++)
                for (int j = 0; j < 4; j++) {
                    float s = 0.0f;
                    for (int v = 0; v < 6; v++) s = fmaf(t1[i][v], WG_A4[v * 4 + j], s);
                    Y[i][j] = apply_act(s + bias[oc], act);
                }
            for (int i = 0; i < 4; i++) {
                const int py = 4 * ty + i;
                if (py >= OH) break;
                for (int j = 0; j < 4; j++) {
                    const int px = 4 * tx + j;
                    if (px < OW) out[(size_t)oc * OW * OH + (size_t)py * OW + px] = Y[i][j];
                }
            }
        }
    }
}

/* ------------------------------------------------------------- direct conv --
 * The convolution every conv path of builder::conv (src/ppdoclayout.cpp:
 * 388-543) computes: y[oc][oy][ox] = act(b[oc] + sum x[ic][oy*S+kh-P]
 * [ox*S+kw-P] * w[oc][ic][kh][kw]) with zero padding.  groups == IC == OC
 * gives the depthwise conv of :400-404 (w [C][1][K][K]).  Accumulated in
 * double, rounded once before bias and activation, so it is an
 * order-independent oracle for every conv algorithm (im2col+GEMM,
 * Winograd, implicit GEMM). */
void oracle_conv2d(const float *x, const float *w, const float *bias, float *y,
                   int IC, int IH, int IW, int OC, int K, int S, int P, int groups, int act)
{
    const int OH = (IH + 2 * P - K) / S + 1;
    const int OW = (IW + 2 * P - K) / S + 1;
    const int icg = IC / groups, ocg = OC / groups;
    OMP_FOR
    for (int oc = 0; oc < OC; oc++) {
        const int g = oc / ocg;
        for (int oy = 0; oy < OH; oy++)
            for (int ox = 0; ox < OW; ox++) {
                double s = 0.0;
                for (int ci = 0; ci < icg; ci++) {
                    const int ic = g * icg + ci;
                    for (int kh = 0; kh < K; kh++) {
                        const int iy = oy * S + kh - P;
                        if (iy < 0 || iy >= IH) continue;
                        for (int kw = 0; kw < K; kw++) {
                            const int ix = ox * S + kw - P;
                            if (ix < 0 || ix >= IW) continue;
                            s += (double)x[((size_t)ic * IH + iy) * IW + ix] *
                                 (double)w[(((size_t)oc * icg + ci) * K + kh) * K + kw];
                        }
                    }
                }
                y[((size_t)oc * OH + oy) * OW + ox] = apply_act((float)s + bias[oc], act);
            }
    }
}

/* --------------------------------------------------------- host constants --
 * Sine position embedding of the AIFI tokens (src/ppdoclayout.cpp:887-903):
 * 625 x 256, [sin_h | cos_h | sin_w | cos_w], H-outer, float64 math. */
void oracle_pos_embed(float *pos)
{
    double omega[64];
    for (int i = 0; i < 64; i++) omega[i] = 1.0 / pow(10000.0, (double)i / 64.0);
    for (int h = 0; h < 25; h++)
        for (int w = 0; w < 25; w++) {
            float *p = pos + (size_t)(h * 25 + w) * DM;
            for (int i = 0; i < 64; i++) {
                p[i] = (float)sin(h * omega[i]);
                p[64 + i] = (float)cos(h * omega[i]);
                p[128 + i] = (float)sin(w * omega[i]);
                p[192 + i] = (float)cos(w * omega[i]);
            }
        }
}

/* Valid-token mask of the two-stage selection (src/ppdoclayout.cpp:905-923). */
void oracle_valid_mask(float *vm)
{
    const float eps = 1e-2f;
    int t = 0;
    for (int l = 0; l < NLVL; l++) {
        const int W = LVL_W[l], H = LVL_H[l];
        const float wh = 0.05f * (float)pow(2.0f, (float)l);
        for (int y = 0; y < H; y++)
            for (int x = 0; x < W; x++) {
                const float cx = ((float)x + 0.5f) / (float)W;
                const float cy = ((float)y + 0.5f) / (float)H;
                const int ok = cx > eps && cx < 1.0f - eps && cy > eps && cy < 1.0f - eps &&
                               wh > eps && wh < 1.0f - eps;
                vm[t++] = ok ? 1.0f : 0.0f;
            }
    }
}

/* ------------------------------------------------------------ postprocess --
 * src/ppdoclayout.cpp:927-993, one page:
 *   votes[j] = sum_{i != j} sigmoid(order[j + 300 i] - order[i + 300 j]),
 *   stable ascending sort of votes -> rank per query;
 *   scores = sigmoid(logits) over 300 x 25, the 300 largest (ties to the
 *   lower flat index); boxes restored to the original size, ONNX style;
 *   masks thresholded at > 0 and reordered to the selection.
 * dets [300][7] = label, score, x1, y1, x2, y2, order; masks [300][40000]
 * int32; sel [300] flat q*25+c. */
static const float *g_votes;
static int votes_cmp(const void *pa, const void *pb)
{
    const int a = *(const int *)pa, b = *(const int *)pb;
    if (g_votes[a] < g_votes[b]) return -1;
    if (g_votes[b] < g_votes[a]) return 1;
    return a < b ? -1 : (a > b ? 1 : 0); /* stable: original index order */
}
static const float *g_scores;
static int scores_cmp(const void *pa, const void *pb)
{
    const int a = *(const int *)pa, b = *(const int *)pb;
    if (g_scores[a] != g_scores[b]) return g_scores[a] > g_scores[b] ? -1 : 1;
    return a < b ? -1 : (a > b ? 1 : 0);
}

void oracle_postprocess(const float *logits, const float *boxes, const float *order,
                        const float *maskl, int ori_h, int ori_w,
                        float *dets, int32_t *masks, int32_t *sel)
{
    float votes[NQ];
    for (int j = 0; j < NQ; j++) {
        float acc = 0.0f;
        for (int i = 0; i < NQ; i++) {
            if (i == j) continue;
            const float diff = order[(size_t)j + (size_t)NQ * i] - order[(size_t)i + (size_t)NQ * j];
            acc += 1.0f / (1.0f + expf(-diff));
        }
        votes[j] = acc;
    }
    int ptr[NQ], order_seq[NQ];
    for (int i = 0; i < NQ; i++) ptr[i] = i;
    g_votes = votes;
    qsort(ptr, NQ, sizeof(int), votes_cmp);
    for (int r = 0; r < NQ; r++) order_seq[ptr[r]] = r;

    static float scores[NQ * NC];
    static int fi[NQ * NC];
    for (int i = 0; i < NQ * NC; i++) {
        scores[i] = 1.0f / (1.0f + expf(-logits[i]));
        fi[i] = i;
    }
    g_scores = scores;
    qsort(fi, NQ * NC, sizeof(int), scores_cmp);

    const float sf_h = (float)800 / (float)ori_h;
    const float sf_w = (float)800 / (float)ori_w;
    const float oh = floorf((float)800 / sf_h + 0.5f);
    const float ow = floorf((float)800 / sf_w + 0.5f);
    for (int r = 0; r < NQ; r++) {
        const int flat = fi[r];
        const int q = flat / NC, c = flat % NC;
        const float *b = boxes + (size_t)q * 4;
        float *o = dets + (size_t)r * 7;
        o[0] = (float)c;
        o[1] = scores[flat];
        o[2] = (b[0] - b[2] * 0.5f) * ow;
        o[3] = (b[1] - b[3] * 0.5f) * oh;
        o[4] = (b[0] + b[2] * 0.5f) * ow;
        o[5] = (b[1] + b[3] * 0.5f) * oh;
        o[6] = (float)order_seq[q];
        if (sel) sel[r] = flat;
        if (masks) {
            const float *ml = maskl + (size_t)q * MASK_PIX;
            int32_t *mo = masks + (size_t)r * MASK_PIX;
            for (int p = 0; p < MASK_PIX; p++) mo[p] = ml[p] > 0.0f ? 1 : 0;
        }
    }
}
