// conv.cu — Winograd F(4,3) transforms, depthwise conv and the memory-bound
// glue of the conv stack (pool, interpolation, layout changes).
//
// Winograd F(4,3) for k3-s1-p1 convs follows the reference's pipeline
// (src/ppdoclayout.cpp:430-464, patches/ggml-ppdl.patch:488-610): input
// transform d~ = B^T d B per 6x6 tile (stride 4) -> 36 independent
// (T x IC)(IC x OC) products -> output transform Y = A^T m A + bias,
// activation.  Differences of this build:
//   * the zero padding (left/top 1, right/bottom up to the 4x4 tile grid)
//     is applied inside the input transform from the unpadded CHW tensor,
//     so the reference's separate ggml_pad_ext pass disappears;
//   * pages are batched: the planes of page b are z = b*36 + plane;
//   * the output transform can add a residual before or after the
//     activation and writes into a channel slice of a wider buffer, so the
//     RepVGG sum and the HG-block concat cost no extra pass.
// The transform matrices are the reference's (a data format shared with its
// op 10/11/12 planes and ".wg4" weights).
#include "common.cuh"
#include "conv.h"

namespace ppdl {

__constant__ float c_wgB[36] = {
     0.156081140f, -0.005399639f, -0.912340343f, -0.209068865f,  0.695356965f,  0.124203928f,
    -0.153710172f, -0.110961877f,  0.797504783f,  0.794400156f,  0.002377054f, -0.019845223f,
     0.423170745f, -0.936912060f, -0.566737831f,  0.947692990f,  0.041719031f, -0.024267767f,
    -0.338096678f,  0.120876059f,  1.953236461f, -0.181245893f, -1.540627480f,  0.223424435f,
     0.295037359f,  0.647394836f, -0.185275897f, -0.582640827f, -0.011674470f,  0.014480385f,
     0.198828861f, -0.241681889f, -0.911203325f,  0.846514463f,  0.049163014f, -0.022408651f,
};
__constant__ float c_wgG[18] = {
    -0.019582119f, -0.133662105f, -0.912340343f,
     0.650278211f,  0.720138848f,  0.797504783f,
    -0.947692990f,  0.466171294f, -0.229310215f,
     0.060792211f, -0.344588995f,  1.953236461f,
     0.647394836f,  0.272543609f,  0.114736818f,
    -0.911203325f,  0.880876958f, -0.851559937f,
};
__constant__ float c_wgA[24] = {
    -0.015757650f, -0.107557341f, -0.734156489f, -5.011147976f,
     0.878285885f,  0.972641826f,  1.077134609f,  1.192853332f,
    -1.655853987f,  0.814516485f, -0.400661618f,  0.197085932f,
    -0.005868433f,  0.033264086f, -0.188551068f,  1.068765521f,
     3.145301104f,  1.324125051f,  0.557437003f,  0.234672695f,
     0.978109479f, -0.945556402f,  0.914086699f, -0.883664429f,
};

namespace {

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// ---- Winograd input transform -----------------------------------------------
// thread per (page, ic, tile); dt[(b*36 + p)*IC + ic][T] (the reference's
// (T, IC, 36) plane layout per page)
__global__ void __launch_bounds__(256)
wg4_input_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ dt, int IC,
                 int H, int W, int TW, int TH, int pad, int B, int ldt) {
    // grid (IC*T / 256, B): one 32-bit division per thread
    const int T = TW * TH;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= IC * T) return;
    const int ic = i / T, tile = i - ic * T, b = blockIdx.y;
    const int ty = tile / TW, tx = tile - ty * TW;
    const float *xp = x + (long long)b * xbs + (long long)ic * H * W;
    float d[6][6];
#pragma unroll
    for (int a = 0; a < 6; a++) {
        const int iy = 4 * ty + a - pad;
#pragma unroll
        for (int c = 0; c < 6; c++) {
            const int ix = 4 * tx + c - pad;
            d[a][c] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? __ldg(xp + (long long)iy * W + ix)
                                                              : 0.0f;
        }
    }
    float t1[6][6];
#pragma unroll
    for (int u = 0; u < 6; u++)
#pragma unroll
        for (int v = 0; v < 6; v++) {
            float s = 0.0f;
#pragma unroll
            for (int a = 0; a < 6; a++) s = fmaf(c_wgB[u * 6 + a], d[a][v], s);
            t1[u][v] = s;
        }
    float *o = dt + ((long long)b * 36 * IC + ic) * ldt + tile;
#pragma unroll
    for (int u = 0; u < 6; u++)
#pragma unroll
        for (int w = 0; w < 6; w++) {
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < 6; c++) s = fmaf(t1[u][c], c_wgB[w * 6 + c], s);
            o[(long long)(u * 6 + w) * IC * ldt] = s;
        }
}

// ---- Winograd output transform ----------------------------------------------
__global__ void __launch_bounds__(256)
wg4_output_kernel(const float *__restrict__ yt, const float *__restrict__ bias,
                  float *__restrict__ y, long long ybs, const float *__restrict__ res,
                  long long rbs, int res_mode, int OC, int OH, int OW, int TW, int TH, int act,
                  int B, int ldt) {
    // grid (OC*T / 256, B)
    const int T = TW * TH;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= OC * T) return;
    const int oc = i / T, tile = i - oc * T, b = blockIdx.y;
    const int ty = tile / TW, tx = tile - ty * TW;
    const float *m = yt + ((long long)b * 36 * OC + oc) * ldt + tile;
    float mm[36];
#pragma unroll
    for (int p = 0; p < 36; p++) mm[p] = __ldg(m + (long long)p * OC * ldt);
    float t1[4][6];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int v = 0; v < 6; v++) {
            float s = 0.0f;
#pragma unroll
            for (int u = 0; u < 6; u++) s = fmaf(c_wgA[u * 4 + a], mm[u * 6 + v], s);
            t1[a][v] = s;
        }
    const float bv = bias ? bias[oc] : 0.0f;
    float *yp = y + (long long)b * ybs + (long long)oc * OH * OW;
    const float *rp = res_mode ? res + (long long)b * rbs + (long long)oc * OH * OW : nullptr;
#pragma unroll
    for (int a = 0; a < 4; a++) {
        const int py = 4 * ty + a;
        if (py >= OH) break;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int px = 4 * tx + c;
            if (px >= OW) break;
            float s = 0.0f;
#pragma unroll
            for (int v = 0; v < 6; v++) s = fmaf(t1[a][v], c_wgA[v * 4 + c], s);
            float val = __fadd_rn(s, bv);
            const long long off = (long long)py * OW + px;
            if (res_mode == 1) val = __fadd_rn(val, rp[off]);
            val = act_apply(val, act);
            if (res_mode == 2) val = __fadd_rn(val, rp[off]);
            yp[off] = val;
        }
    }
}

// ---- Winograd filter transform ----------------------------------------------
// w [OC][IC][3][3] -> wg4[36][IC][OC], sum_ab (G[u][a] * G[v][b]) * w in the
// order of src/ppdoclayout.cpp:321-333.
__global__ void wg4_filter_kernel(const float *__restrict__ w, float *__restrict__ wg4, int IC,
                                  int OC) {
    const long long n = 36LL * IC * OC;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int oc = (int)(i % OC);
    const long long r = i / OC;
    const int ic = (int)(r % IC);
    const int uv = (int)(r / IC);
    const int u = uv / 6, v = uv % 6;
    float s = 0.0f;
    for (int a = 0; a < 3; a++)
        for (int b = 0; b < 3; b++) {
            const float g = __fmul_rn(c_wgG[u * 3 + a], c_wgG[v * 3 + b]);
            s = __fadd_rn(s, __fmul_rn(g, w[(((long long)oc * IC + ic) * 3 + a) * 3 + b]));
        }
    wg4[i] = s;
}

// wg4 [36][IC][OC] -> hi/lo [36][OC][IC] (K-major B operand of the
// tensor-core madd, split into TF32 halves)
__global__ void wg4_kmajor_split_kernel(const float *__restrict__ wg4, float *__restrict__ hi,
                                        float *__restrict__ lo, int IC, int OC) {
    const long long n = 36LL * IC * OC;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int ic = (int)(i % IC);
    const long long r = i / IC;
    const int oc = (int)(r % OC);
    const int p = (int)(r / OC);
    const float v = wg4[((long long)p * IC + ic) * OC + oc];
    uint32_t hr;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hr) : "f"(v));  // nearest TF32
    const float h = __uint_as_float(hr);
    hi[i] = h;
    lo[i] = v - h;
}

// ---- depthwise conv -----------------------------------------------------------
// ggml_conv_2d_dw_direct + bias + act (src/ppdoclayout.cpp:400-404).
template <int K>
__global__ void __launch_bounds__(256)
dwconv_kernel(const float *__restrict__ x, long long xbs, const float *__restrict__ w,
              const float *__restrict__ bias, float *__restrict__ y, long long ybs, int C, int H,
              int W, int OH, int OW, int S, int P, int act, int B) {
    // grid (C*OH*OW / 256, B)
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= C * OH * OW) return;
    const int c = i / (OH * OW), p = i - c * (OH * OW), b = blockIdx.y;
    const int oy = p / OW, ox = p - oy * OW;
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const float *wp = w + (long long)c * K * K;
    float s = 0.0f;
#pragma unroll
    for (int kh = 0; kh < K; kh++) {
        const int iy = oy * S + kh - P;
        if (iy < 0 || iy >= H) continue;
#pragma unroll
        for (int kw = 0; kw < K; kw++) {
            const int ix = ox * S + kw - P;
            if (ix < 0 || ix >= W) continue;
            s = fmaf(__ldg(xp + (long long)iy * W + ix), __ldg(wp + kh * K + kw), s);
        }
    }
    s = __fadd_rn(s, bias[c]);
    y[(long long)b * ybs + (long long)c * OH * OW + (long long)oy * OW + ox] = act_apply(s, act);
}

// ---- 2x2 stride-1 max pool over the right/bottom zero-padded input ----------
// ggml_pad(x, 1, 1) + ggml_pool_2d(MAX, 2, 2, 1, 1, 0, 0) (src/ppdoclayout.cpp:621-625)
__global__ void maxpool2_pad_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                                    long long ybs, int C, int H, int W, int B) {
    // grid (C*H*W / 256, B)
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= C * H * W) return;
    const int c = i / (H * W), p = i - c * (H * W), b = blockIdx.y;
    const int oy = p / W, ox = p - oy * W;
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const float v00 = xp[(long long)oy * W + ox];
    const float v01 = ox + 1 < W ? xp[(long long)oy * W + ox + 1] : 0.0f;
    const float v10 = oy + 1 < H ? xp[(long long)(oy + 1) * W + ox] : 0.0f;
    const float v11 = (ox + 1 < W && oy + 1 < H) ? xp[(long long)(oy + 1) * W + ox + 1] : 0.0f;
    y[(long long)b * ybs + (long long)c * H * W + (long long)oy * W + ox] =
        fmaxf(fmaxf(v00, v01), fmaxf(v10, v11));
}

// ---- interpolation (ggml_interpolate, src/ppdoclayout.cpp:670-672) -----------
// NEAREST: src = (int)(dst / sf).  BILINEAR (no align-corners): src =
// (dst + 0.5) / sf - 0.5, floor, both taps clamped to the edge, fractional
// weight clamped to [0, 1].  Optionally adds into y (y = base + interp).
__global__ void interp_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                              long long ybs, const float *__restrict__ base, long long bbs, int C,
                              int H, int W, int OH, int OW, int bilinear, int B) {
    // grid (C*OH*OW / 256, B)
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= C * OH * OW) return;
    const int c = i / (OH * OW), p = i - c * (OH * OW), b = blockIdx.y;
    const int oy = p / OW, ox = p - oy * OW;
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const float sfx = (float)OW / (float)W, sfy = (float)OH / (float)H;
    float v;
    if (!bilinear) {
        const int sx = min((int)((float)ox / sfx), W - 1);
        const int sy = min((int)((float)oy / sfy), H - 1);
        v = xp[(long long)sy * W + sx];
    } else {
        const float fx = __fsub_rn(__fdiv_rn(__fadd_rn((float)ox, 0.5f), sfx), 0.5f);
        const float fy = __fsub_rn(__fdiv_rn(__fadd_rn((float)oy, 0.5f), sfy), 0.5f);
        const float flx = floorf(fx), fly = floorf(fy);
        int x0 = (int)flx, y0 = (int)fly;
        int x1 = x0 + 1, y1 = y0 + 1;
        const float dx = fminf(fmaxf(__fsub_rn(fx, flx), 0.0f), 1.0f);
        const float dy = fminf(fmaxf(__fsub_rn(fy, fly), 0.0f), 1.0f);
        x0 = max(0, min(x0, W - 1)); x1 = max(0, min(x1, W - 1));
        y0 = max(0, min(y0, H - 1)); y1 = max(0, min(y1, H - 1));
        const float a = xp[(long long)y0 * W + x0], bq = xp[(long long)y0 * W + x1];
        const float cq = xp[(long long)y1 * W + x0], d = xp[(long long)y1 * W + x1];
        v = a * (1.0f - dx) * (1.0f - dy) + bq * dx * (1.0f - dy) + cq * (1.0f - dx) * dy +
            d * dx * dy;
    }
    const long long off = (long long)c * OH * OW + (long long)oy * OW + ox;
    if (base) v = __fadd_rn(base[(long long)b * bbs + off], v);
    y[(long long)b * ybs + off] = v;
}

// ---- CHW <-> token-major ([H*W][C]) through a shared-memory tile ------------
__global__ void transpose_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                                 long long ybs, int R, int Cc, long long ldx, long long ldy) {
    // y[c][r] = x[r][c] for a R x Cc matrix; x row stride ldx, y row stride ldy
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const float *xp = x + (long long)b * xbs;
    float *yp = y + (long long)b * ybs;
    const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int r = r0 + k, c = c0 + threadIdx.x;
        if (r < R && c < Cc) tile[k][threadIdx.x] = xp[(long long)r * ldx + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int c = c0 + k, r = r0 + threadIdx.x;
        if (r < R && c < Cc) yp[(long long)c * ldy + r] = tile[threadIdx.x][k];
    }
}

// ---- im2col: the M-major GEMM operand of a KS x KS, stride-S conv -----------
// col[b][k][m] = x[b][ic][oy*S + kh - P][ox*S + kw - P] (0 outside H x W and
// for k >= IC*KS*KS), k = (ic*KS + kh)*KS + kw (the raw weight's row order),
// m = oy*OW + ox < M; rows have stride ldm >= M (16-byte multiples for the
// tensor-core GEMM's TMA), the tail m in [M, ldm) is zero.  KS = 1 is a
// channel-plane copy into padded rows.  One block row per k (grid.y).
__global__ void __launch_bounds__(256)
im2col_kernel(const float *__restrict__ x, long long xbs, long long plane, float *__restrict__ col,
              long long cbs, int Kc, int H, int W, int KS, int S, int P, int OW, int M, int ldm) {
    // each thread writes 4 consecutive m with one 16-byte store (ldm % 4 == 0)
    const int k = blockIdx.y, b = blockIdx.z;
    float4 *cr = reinterpret_cast<float4 *>(col + (long long)b * cbs + (long long)k * ldm);
    const int n4 = ldm >> 2;
    if (k >= Kc) {
        for (int m4 = blockIdx.x * 256 + threadIdx.x; m4 < n4; m4 += gridDim.x * 256)
            cr[m4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        return;
    }
    const int kk2 = KS * KS, ic = k / kk2, tap = k - ic * kk2, kh = tap / KS, kw = tap - kh * KS;
    const float *xc = x + (long long)b * xbs + (long long)ic * plane;
    for (int m4 = blockIdx.x * 256 + threadIdx.x; m4 < n4; m4 += gridDim.x * 256) {
        float v[4];
        int m = m4 * 4;
        int oy = m / OW, ox = m - oy * OW;
#pragma unroll
        for (int e = 0; e < 4; e++, m++) {
            v[e] = 0.0f;
            if (m < M) {
                const int iy = oy * S + kh - P, ix = ox * S + kw - P;
                if ((unsigned)iy < (unsigned)H && (unsigned)ix < (unsigned)W)
                    v[e] = __ldg(xc + iy * W + ix);
            }
            if (++ox == OW) {
                ox = 0;
                ++oy;
            }
        }
        cr[m4] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

inline int blocks(long long n, int t = 256) { return (int)((n + t - 1) / t); }

// grid of the per-page kernels: x over the channels x pixels (or tiles) of a
// page as one 32-bit index, y over pages
inline bool grid3_ok(long long pix, int ch, int b) {
    return pix > 0 && ch > 0 && pix * ch < (1LL << 31) && b > 0 && b <= 65535;
}
inline dim3 grid3(long long pix, int ch, int b) { return dim3(blocks(pix * ch), b); }

}  // namespace

Status launch_im2col(const float *x, long long xbs, long long plane, float *col, long long cbs,
                     int Kc, int Kp, int H, int W, int KS, int S, int P, int OW, int M, int ldm,
                     int B, cudaStream_t st) {
    if (Kp < Kc || ldm < M || ldm % 4 || M <= 0 || B <= 0 || Kp > 65535 || B > 65535 ||
        ((uintptr_t)col & 15) || cbs % 4)
        return ERR_SHAPE;
    int gx = blocks(ldm / 4);
    if (gx > 64) gx = 64;
    im2col_kernel<<<dim3(gx, Kp, B), 256, 0, st>>>(x, xbs, plane, col, cbs, Kc, H, W, KS, S, P,
                                                   OW, M, ldm);
    return cuda_status();
}

Status launch_wg4_input(const float *x, long long xbs, float *dt, int IC, int H, int W, int TW,
                        int TH, int pad, int B, cudaStream_t st, int ldt) {
    if (!grid3_ok((long long)TW * TH, IC, B)) return ERR_SHAPE;
    if (ldt <= 0) ldt = TW * TH;
    if (ldt < TW * TH) return ERR_SHAPE;
    wg4_input_kernel<<<grid3((long long)TW * TH, IC, B), 256, 0, st>>>(x, xbs, dt, IC, H, W, TW,
                                                                       TH, pad, B, ldt);
    return cuda_status();
}

Status launch_wg4_output(const float *yt, const float *bias, float *y, long long ybs,
                         const float *res, long long rbs, int res_mode, int OC, int OH, int OW,
                         int TW, int TH, int act, int B, cudaStream_t st, int ldt) {
    if (!grid3_ok((long long)TW * TH, OC, B)) return ERR_SHAPE;
    if (TW < (OW + 3) / 4 || TH < (OH + 3) / 4) return ERR_SHAPE;
    if (ldt <= 0) ldt = TW * TH;
    if (ldt < TW * TH) return ERR_SHAPE;
    wg4_output_kernel<<<grid3((long long)TW * TH, OC, B), 256, 0, st>>>(
        yt, bias, y, ybs, res, rbs, res_mode, OC, OH, OW, TW, TH, act, B, ldt);
    return cuda_status();
}

Status launch_wg4_filter(const float *w, float *wg4, int IC, int OC, cudaStream_t st) {
    const long long n = 36LL * IC * OC;
    wg4_filter_kernel<<<blocks(n), 256, 0, st>>>(w, wg4, IC, OC);
    return cuda_status();
}

Status launch_wg4_kmajor_split(const float *wg4, float *hi, float *lo, int IC, int OC,
                               cudaStream_t st) {
    const long long n = 36LL * IC * OC;
    wg4_kmajor_split_kernel<<<blocks(n), 256, 0, st>>>(wg4, hi, lo, IC, OC);
    return cuda_status();
}

Status launch_dwconv(const float *x, long long xbs, const float *w, const float *bias, float *y,
                     long long ybs, int C, int H, int W, int K, int S, int P, int act, int B,
                     cudaStream_t st) {
    const int OH = (H + 2 * P - K) / S + 1, OW = (W + 2 * P - K) / S + 1;
    if (OH <= 0 || OW <= 0 || !grid3_ok((long long)OH * OW, C, B)) return ERR_SHAPE;
    const dim3 g = grid3((long long)OH * OW, C, B);
    if (K == 3)
        dwconv_kernel<3><<<g, 256, 0, st>>>(x, xbs, w, bias, y, ybs, C, H, W, OH, OW, S, P, act, B);
    else if (K == 5)
        dwconv_kernel<5><<<g, 256, 0, st>>>(x, xbs, w, bias, y, ybs, C, H, W, OH, OW, S, P, act, B);
    else
        return ERR_UNSUPPORTED;
    return cuda_status();
}

Status launch_maxpool2_pad(const float *x, long long xbs, float *y, long long ybs, int C, int H,
                           int W, int B, cudaStream_t st) {
    if (!grid3_ok((long long)H * W, C, B)) return ERR_SHAPE;
    maxpool2_pad_kernel<<<grid3((long long)H * W, C, B), 256, 0, st>>>(x, xbs, y, ybs, C, H, W, B);
    return cuda_status();
}

Status launch_interp(const float *x, long long xbs, float *y, long long ybs, const float *base,
                     long long bbs, int C, int H, int W, int OH, int OW, bool bilinear, int B,
                     cudaStream_t st) {
    if (!grid3_ok((long long)OH * OW, C, B)) return ERR_SHAPE;
    interp_kernel<<<grid3((long long)OH * OW, C, B), 256, 0, st>>>(x, xbs, y, ybs, base, bbs, C, H,
                                                                   W, OH, OW, bilinear ? 1 : 0, B);
    return cuda_status();
}

Status launch_transpose(const float *x, long long xbs, float *y, long long ybs, int R, int Cc,
                        long long ldx, long long ldy, int B, cudaStream_t st) {
    dim3 grid((unsigned)cdiv(Cc, 32), (unsigned)cdiv(R, 32), (unsigned)B);
    transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(x, xbs, y, ybs, R, Cc, ldx, ldy);
    (void)sm_count;
    return cuda_status();
}

}  // namespace ppdl
