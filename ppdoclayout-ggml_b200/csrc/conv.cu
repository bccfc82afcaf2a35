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
#include <cmath>

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
// thread per (page, ic, tile); value (page b, plane p, channel ic, tile t) at
// dt[b*bstride + p*pstride + ic*ldt + t]: the reference's (T, IC, 36) plane
// layout per page (bstride = 36*IC*ldt, pstride = IC*ldt), or the pages side
// by side in each channel row (ldt = B*Tp, pstride = IC*ldt, bstride = Tp),
// which the forward uses so that one plane GEMM's rows run over all pages
__global__ void __launch_bounds__(256, 4)
wg4_input_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ dt, int IC,
                 int H, int W, int TW, int TH, int pad, int B, long long ldt, long long pstride,
                 long long bstride) {
    pdl_begin();
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
    float *o = dt + b * bstride + ic * ldt + tile;
#pragma unroll
    for (int u = 0; u < 6; u++)
#pragma unroll
        for (int w = 0; w < 6; w++) {
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < 6; c++) s = fmaf(t1[u][c], c_wgB[w * 6 + c], s);
            o[(long long)(u * 6 + w) * pstride] = s;
        }
}

// Rows of 4 * TW floats (W % 4 == 0, 16-byte aligned rows) and padding 1, the
// forward's case: the thread of tile (ty, tx) reads the 4 aligned columns
// 4 tx .. 4 tx + 3 of each of its 6 window rows as one float4 (a warp's
// reads are contiguous), and takes column 4 tx - 1 from the previous lane's
// float4 and column 4 tx + 4 from the next lane's by warp shuffles (a scalar
// load at the warp's edges; zeros at the plane's left and right borders).
// 6 vector loads per (tile, channel) instead of 36 scalar ones; the transform
// and the stores are those of wg4_input_kernel.
__global__ void __launch_bounds__(256, 4)
wg4_input_vec_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ dt, int IC,
                     int H, int W, int TW, int TH, int B, long long ldt, long long pstride,
                     long long bstride) {
    pdl_begin();
    const int T = TW * TH;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const bool live = i < IC * T;  // every lane takes part in the shuffles
    const int ii = live ? i : IC * T - 1;
    const int ic = ii / T, tile = ii - ic * T, b = blockIdx.y;
    const int ty = tile / TW, tx = tile - ty * TW;
    const float *xp = x + (long long)b * xbs + (long long)ic * H * W;
    float d[6][6];
#pragma unroll
    for (int a = 0; a < 6; a++) {
        const int iy = 4 * ty + a - 1;
        const bool row_in = (unsigned)iy < (unsigned)H;
        const float *xr = xp + (long long)iy * W + 4 * tx;
        const float4 v = row_in ? __ldg(reinterpret_cast<const float4 *>(xr))
                                : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        const float up = __shfl_up_sync(0xffffffffu, v.w, 1);
        const float dn = __shfl_down_sync(0xffffffffu, v.x, 1);
        float left = 0.0f, right = 0.0f;
        if (tx > 0) left = lane > 0 ? up : (row_in ? __ldg(xr - 1) : 0.0f);
        if (tx < TW - 1) right = lane < 31 ? dn : (row_in ? __ldg(xr + 4) : 0.0f);
        d[a][0] = left; d[a][1] = v.x; d[a][2] = v.y; d[a][3] = v.z; d[a][4] = v.w;
        d[a][5] = right;
    }
    if (!live) return;
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
    float *o = dt + b * bstride + ic * ldt + tile;
#pragma unroll
    for (int u = 0; u < 6; u++)
#pragma unroll
        for (int w = 0; w < 6; w++) {
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < 6; c++) s = fmaf(t1[u][c], c_wgB[w * 6 + c], s);
            o[(long long)(u * 6 + w) * pstride] = s;
        }
}

// ---- RepVGG branch folding ---------------------------------------------------
// The reference's RepVGG block (src/ppdoclayout.cpp:656-661) adds a 3x3 conv
// (w3 [OC][IC][3][3], b3) and a 1x1 conv (w1 [OC][IC], b1) of the same input.
// One 3x3 conv with wm = w3 plus w1 on the centre tap and bm = b3 + b1 is the
// same map in real arithmetic; the forward runs that conv (one Winograd conv
// instead of a 1x1 GEMM, a Winograd conv and a residual read).
__global__ void rep_fold_kernel(const float *__restrict__ w3, const float *__restrict__ b3,
                                const float *__restrict__ w1, const float *__restrict__ b1,
                                float *__restrict__ wm, float *__restrict__ bm, int IC, int OC) {
    pdl_begin();
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i < 9LL * IC * OC) {
        float v = w3[i];
        if (i % 9 == 4) v = __fadd_rn(v, w1[i / 9]);
        wm[i] = v;
    }
    if (i < OC) bm[i] = __fadd_rn(b3[i], b1[i]);
}

// ---- Winograd output transform ----------------------------------------------
// (both transforms are held to 64 registers, four 256-thread blocks per SM:
// their loads are independent and latency-bound, so more warps in flight
// beat the few extra registers)
__global__ void __launch_bounds__(256, 4)
wg4_output_kernel(const float *__restrict__ yt, const float *__restrict__ bias,
                  float *__restrict__ y, long long ybs, const float *__restrict__ res,
                  long long rbs, int res_mode, int OC, int OH, int OW, int TW, int TH, int act,
                  int B, long long ldt, long long pstride, long long bstride) {
    pdl_begin();
    // grid (OC*T / 256, B); yt addressed as dt of the input transform
    const int T = TW * TH;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= OC * T) return;
    const int oc = i / T, tile = i - oc * T, b = blockIdx.y;
    const int ty = tile / TW, tx = tile - ty * TW;
    const float *m = yt + b * bstride + oc * ldt + tile;
    float mm[36];
#pragma unroll
    for (int p = 0; p < 36; p++) mm[p] = __ldg(m + (long long)p * pstride);
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
    // a full 4-pixel row segment goes out as one 16-byte store (and the
    // residual comes in as one 16-byte load) when the rows allow it
    const bool vec = (OW & 3) == 0 && 4 * tx + 3 < OW && ((uintptr_t)yp & 15) == 0 &&
                     (!rp || ((uintptr_t)rp & 15) == 0);
#pragma unroll
    for (int a = 0; a < 4; a++) {
        const int py = 4 * ty + a;
        if (py >= OH) break;
        const long long off0 = (long long)py * OW + 4 * tx;
        float4 r4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (vec && rp) r4 = *reinterpret_cast<const float4 *>(rp + off0);
        float out[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float s = 0.0f;
#pragma unroll
            for (int v = 0; v < 6; v++) s = fmaf(t1[a][v], c_wgA[v * 4 + c], s);
            float val = __fadd_rn(s, bv);
            const float rv = !rp ? 0.0f
                             : vec ? (c == 0 ? r4.x : c == 1 ? r4.y : c == 2 ? r4.z : r4.w)
                             : (4 * tx + c < OW ? rp[off0 + c] : 0.0f);
            if (res_mode == 1) val = __fadd_rn(val, rv);
            val = act_apply(val, act);
            if (res_mode == 2) val = __fadd_rn(val, rv);
            out[c] = val;
        }
        if (vec) {
            *reinterpret_cast<float4 *>(yp + off0) = make_float4(out[0], out[1], out[2], out[3]);
        } else {
#pragma unroll
            for (int c = 0; c < 4; c++)
                if (4 * tx + c < OW) yp[off0 + c] = out[c];
        }
    }
}

// ---- Winograd filter transform ----------------------------------------------
// w [OC][IC][3][3] -> wg4[36][IC][OC], sum_ab (G[u][a] * G[v][b]) * w in the
// order of src/ppdoclayout.cpp:321-333.
__global__ void wg4_filter_kernel(const float *__restrict__ w, float *__restrict__ wg4, int IC,
                                  int OC) {
    pdl_begin();
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
// hi/lo[p][oc][ic] (K-major TF32 halves) from src[p][ic][n0 + oc] (row
// stride ld, plane stride pstride), oc < nc
__global__ void kmajor_split_kernel(const float *__restrict__ src, float *__restrict__ hi,
                                    float *__restrict__ lo, int planes, int IC, int ld,
                                    long long pstride, int nc) {
    pdl_begin();
    const long long n = (long long)planes * IC * nc;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int ic = (int)(i % IC);
    const long long r = i / IC;
    const int oc = (int)(r % nc);
    const int p = (int)(r / nc);
    const float v = src[(long long)p * pstride + (long long)ic * ld + oc];
    uint32_t hr;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hr) : "f"(v));  // nearest TF32
    const float h = __uint_as_float(hr);
    hi[i] = h;
    lo[i] = v - h;
}

// ---- depthwise conv -----------------------------------------------------------
// ggml_conv_2d_dw_direct + bias + act (src/ppdoclayout.cpp:400-404).
// A block computes a 32 x 32 output tile of one (page, channel) plane from a
// shared-memory copy of its input window (halo included, zeros outside the
// image), filled row by row with coalesced loads, so every input is read
// from global memory once per tile.  A thread computes 4 consecutive outputs
// of one row: per kernel row it reads the 3*S + K window values they share
// once into registers (8 threads per output row, 4 rows per warp; the row
// pitch is 1 mod 32, so the 4 rows of a warp fall in different banks).  Per
// output: s = fma over (kh, kw) ascending — the zero taps of the padding
// leave s unchanged — then + bias, activation.
// 4-byte global -> shared copy; valid = false writes a zero without reading
__device__ __forceinline__ void cp_async_zfill4(uint32_t dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}

constexpr int kDwTW = 32, kDwTH = 32;  // 256 threads: 8 x 4-output groups x 32 rows
constexpr size_t kDwPlaneSmemMax = 64 * 1024;  // whole-plane form up to this much input
constexpr size_t kDwBandSmem = 24 * 1024;      // input rows of one band of the band form
constexpr int kDirectTaps = 128;                   // products per output of the direct form
constexpr size_t kDirectWindowBytes = 40 * 1024;   // input window per channel chunk
template <int K, int S>
__global__ void __launch_bounds__(256)
dwconv_kernel(const float *__restrict__ x, long long xbs, const float *__restrict__ w,
              const float *__restrict__ bias, float *__restrict__ y, long long ybs, int H, int W,
              int OH, int OW, int P, int act, int tiles_x) {
    pdl_begin();
    constexpr int IW = (kDwTW - 1) * S + K, IH = (kDwTH - 1) * S + K;
    constexpr int LD = (IW + 30) / 32 * 32 + 1;  // >= IW, 1 mod 32
    constexpr int NV = 3 * S + K;                // window columns of 4 outputs
    __shared__ float tile[IH * LD];
    const int c = blockIdx.y, b = blockIdx.z;
    const int tyi = blockIdx.x / tiles_x;
    const int tx0 = (blockIdx.x - tyi * tiles_x) * kDwTW, ty0 = tyi * kDwTH;
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const int ix0 = tx0 * S - P, iy0 = ty0 * S - P;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // asynchronous 4-byte copies (zero-filled outside the image), all of a
    // thread's in flight at once rather than one load-to-store round trip each
    const uint32_t tile_s = (uint32_t)__cvta_generic_to_shared(tile);
    for (int r = warp; r < IH; r += 8) {
        const int iy = iy0 + r;
        const bool row_in = (unsigned)iy < (unsigned)H;
        const float *xr = xp + (long long)iy * W;
        for (int q = lane; q < IW; q += 32) {
            const int ix = ix0 + q;
            const bool in = row_in && (unsigned)ix < (unsigned)W;
            cp_async_zfill4(tile_s + (uint32_t)(r * LD + q) * 4u, in ? xr + ix : xp, in);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    float wk[K * K];
#pragma unroll
    for (int i = 0; i < K * K; i++) wk[i] = __ldg(w + (long long)c * K * K + i);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int xg = threadIdx.x & 7, ly = threadIdx.x >> 3;
    const int ox0 = tx0 + 4 * xg, oy = ty0 + ly;
    if (ox0 >= OW || oy >= OH) return;
    float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float *tp = tile + (ly * S) * LD + 4 * S * xg;
#pragma unroll
    for (int kh = 0; kh < K; kh++) {
        float v[NV];
#pragma unroll
        for (int i = 0; i < NV; i++) v[i] = tp[kh * LD + i];
#pragma unroll
        for (int o = 0; o < 4; o++)
#pragma unroll
            for (int kw = 0; kw < K; kw++) s[o] = fmaf(v[o * S + kw], wk[kh * K + kw], s[o]);
    }
    const float bv = bias ? __ldg(bias + c) : 0.0f;
    float *yp = y + (long long)b * ybs + (long long)c * OH * OW + (long long)oy * OW + ox0;
#pragma unroll
    for (int o = 0; o < 4; o++)
        if (ox0 + o < OW) yp[o] = act_apply(__fadd_rn(s[o], bv), act);
}

// Whole-plane form for planes whose padded input fits in shared memory (the
// light blocks' 50x50 and 25x25 planes, the 100 -> 50 and 50 -> 25
// downsamples): one block per (page, channel) copies the plane once into a
// zero-bordered copy (border P; 8-byte asynchronous copies when P and W are
// even, 4-byte otherwise), then a thread computes a 4 x 4 block of outputs:
// per input row of its (3 S + K)-square window it reads the row segment as
// float4s (rows of ld floats, ld % 4 == 0, so the reads are 16-byte aligned
// and a quarter warp's are contiguous), and adds it into the outputs whose
// kernel row it is.  Per output the sum runs over kh, then kw, with fmaf,
// then + bias and the activation (ACT: 0 none, 1 ReLU, -1 the runtime act);
// rows of even width leave as float2 stores (when y allows 8-byte stores).
// The form is issue-bound, so its shape keeps the instructions per output
// low: 25 FMAs, about one shared load and a fraction of a copy.
template <int K, int S, int ACT>
__global__ void __launch_bounds__(256)
dwconv_plane_kernel(const float *__restrict__ x, long long xbs, const float *__restrict__ w,
                    const float *__restrict__ bias, float *__restrict__ y, long long ybs, int H,
                    int W, int OH, int OW, int P, int act, int ld, int HPp, int GX, int GY,
                    int pairs, int even) {
    pdl_begin();
    extern __shared__ float4 plane4[];
    float *plane = reinterpret_cast<float *>(plane4);  // HPp rows of ld floats
    constexpr int NX = 3 * S + K;                      // window rows / columns of a 4 x 4 block
    constexpr int N4 = (NX + 3) / 4;
    const int c = blockIdx.x, b = blockIdx.y;
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const uint32_t plane_s = (uint32_t)__cvta_generic_to_shared(plane);
    // one row per warp pass
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int r = warp; r < HPp; r += nwarps) {
        const int iy = r - P;
        const bool row_in = (unsigned)iy < (unsigned)H;
        const float *xr = xp + (long long)iy * W;
        float *prow = plane + r * ld;
        const uint32_t srow = plane_s + (uint32_t)(r * ld) * 4u;
        if (pairs) {
            // P and W even: a column pair is wholly inside or outside the image
            for (int q = 2 * lane; q < ld; q += 64) {
                const int ix = q - P;
                if (row_in && (unsigned)ix < (unsigned)W)
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(srow + 4u * q),
                                 "l"(xr + ix)
                                 : "memory");
                else
                    *reinterpret_cast<float2 *>(prow + q) = make_float2(0.0f, 0.0f);
            }
        } else {
            for (int q = lane; q < ld; q += 32) {
                const int ix = q - P;
                const bool in = row_in && (unsigned)ix < (unsigned)W;
                cp_async_zfill4(srow + 4u * q, in ? xr + ix : xp, in);
            }
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    float wk[K * K];
#pragma unroll
    for (int i = 0; i < K * K; i++) wk[i] = __ldg(w + (long long)c * K * K + i);
    const float bv = bias ? __ldg(bias + c) : 0.0f;
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    float *yp = y + (long long)b * ybs + (long long)c * OH * OW;
    for (int it = threadIdx.x; it < GX * GY; it += blockDim.x) {
        const int ty = it / GX, tx = it - ty * GX;
        const int oy0 = 4 * ty, ox0 = 4 * tx;
        float s[4][4];
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int q = 0; q < 4; q++) s[r][q] = 0.0f;
        const float4 *wp = reinterpret_cast<const float4 *>(plane + (oy0 * S) * ld + ox0 * S);
#pragma unroll
        for (int j = 0; j < NX; j++) {
            float v[4 * N4];
#pragma unroll
            for (int u = 0; u < N4; u++) {
                const float4 t = wp[(j * ld >> 2) + u];
                v[4 * u] = t.x; v[4 * u + 1] = t.y; v[4 * u + 2] = t.z; v[4 * u + 3] = t.w;
            }
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int kh = j - r * S;
                if (kh >= 0 && kh < K) {
#pragma unroll
                    for (int q = 0; q < 4; q++)
#pragma unroll
                        for (int kw = 0; kw < K; kw++)
                            s[r][q] = fmaf(v[q * S + kw], wk[kh * K + kw], s[r][q]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int oy = oy0 + r;
            if (oy >= OH) break;
            float o[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float v = __fadd_rn(s[r][q], bv);
                o[q] = ACT == 0 ? v : ACT == 1 ? fmaxf(v, 0.0f) : act_apply(v, act);
            }
            float *yr = yp + (long long)oy * OW + ox0;
            if (even && ox0 + 4 <= OW) {
                reinterpret_cast<float2 *>(yr)[0] = make_float2(o[0], o[1]);
                reinterpret_cast<float2 *>(yr)[1] = make_float2(o[2], o[3]);
            } else {
#pragma unroll
                for (int q = 0; q < 4; q++)
                    if (ox0 + q < OW) yr[q] = o[q];
            }
        }
    }
}

// Band form, for planes too large for the whole-plane form (the 200 -> 100
// downsample): one block per (page, channel, band of BR output rows, BR a
// multiple of 4) loads the band's (BR - 1) S + K input rows, zero-bordered
// (border P), into shared memory at a row pitch ld of 1 mod 32 with
// asynchronous 4-byte copies, then computes the band.  Blocks are small
// enough that several stay resident per SM, so one block's copies overlap
// another's arithmetic.  A thread computes 4 vertically adjacent outputs of
// one column, consecutive threads on consecutive columns: a warp's
// shared-memory reads fall on consecutive words (conflict-free at stride 1,
// two-way at stride 2; four consecutive outputs of a row per thread would
// be four-way) and its stores on consecutive addresses.  Input rows stream
// through K registers; each output sums over kh, then kw, as the tiled form.
template <int K, int S>
__global__ void __launch_bounds__(256)
dwconv_band_kernel(const float *__restrict__ x, long long xbs, const float *__restrict__ w,
                   const float *__restrict__ bias, float *__restrict__ y, long long ybs, int C,
                   int H, int W, int OH, int OW, int P, int act, int ld, int cols, int BR,
                   int nbands) {
    pdl_begin();
    extern __shared__ float band_rows[];  // ((BR - 1) S + K) rows of ld floats
    constexpr int NV = 3 * S + K;         // input rows of a 4-row output group
    const long long plane = blockIdx.x / nbands;
    const int band = (int)(blockIdx.x - plane * nbands);
    const int b = (int)(plane / C), c = (int)(plane - (long long)b * C);
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const int oy0 = band * BR;
    const int br = OH - oy0 < BR ? OH - oy0 : BR;
    const int rows = (br - 1) * S + K, iy0 = oy0 * S - P;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const uint32_t dst = (uint32_t)__cvta_generic_to_shared(band_rows);
    for (int r = warp; r < rows; r += nwarps) {
        const int iy = iy0 + r;
        const bool row_in = (unsigned)iy < (unsigned)H;
        const float *xr = xp + (long long)iy * W;
        for (int q = lane; q < cols; q += 32) {
            const int ix = q - P;
            const bool in = row_in && (unsigned)ix < (unsigned)W;
            cp_async_zfill4(dst + (uint32_t)(r * ld + q) * 4u, in ? xr + ix : xp, in);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    float wk[K * K];
#pragma unroll
    for (int i = 0; i < K * K; i++) wk[i] = __ldg(w + (long long)c * K * K + i);
    const float bv = bias ? __ldg(bias + c) : 0.0f;
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    float *yp = y + (long long)b * ybs + (long long)c * OH * OW;
    const int groups = (br + 3) >> 2;
    for (int it = threadIdx.x; it < groups * OW; it += blockDim.x) {
        const int rg = it / OW, ox = it - rg * OW;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        // input rows 4 rg S + j, j < NV, columns ox S .. ox S + K - 1; rows
        // past the band's last are read from the buffer's unwritten tail, and
        // their sums are not stored
        const float *tp = band_rows + (4 * rg * S) * ld + ox * S;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            float r[K];
#pragma unroll
            for (int kw = 0; kw < K; kw++) r[kw] = tp[j * ld + kw];
#pragma unroll
            for (int o = 0; o < 4; o++) {
                const int kh = j - o * S;
                if (kh >= 0 && kh < K) {
#pragma unroll
                    for (int kw = 0; kw < K; kw++) s[o] = fmaf(r[kw], wk[kh * K + kw], s[o]);
                }
            }
        }
        float *yc = yp + (long long)(oy0 + 4 * rg) * OW + ox;
#pragma unroll
        for (int o = 0; o < 4; o++)
            if (4 * rg + o < br) yc[(long long)o * OW] = act_apply(__fadd_rn(s[o], bv), act);
    }
}

// ---- direct convolution of narrow convs (the stem) -------------------------
// For convs whose outputs each sum at most kDirectTaps products (IC K K) into
// at most 32 channels (the stem's 3 -> 32 k3-s2 and its 32 -> 16 / 16 -> 32
// k2 convs), a tensor-core tile of 128 pixels x N <= 32 channels carries more
// operand bytes than arithmetic; these run on the CUDA cores in FP32.
// Register tiling: a thread computes 4 consecutive output pixels of a row for
// 16 channels (64 accumulators); per (input channel, kernel row) it reads the
// 3 S + K window values its pixels share as float4s from shared memory, per
// tap the 16 weights as 4 broadcast float4s, and issues 64 FMAs.  Block:
// 256 threads = 16 output rows x 64 columns (16 lanes per row).  Shared
// memory: the weights of the block's 16 channels [ic][kh][kw][16] and the
// input window, ICB channels at a time, filled with asynchronous 4-byte
// copies (zeros outside the input: padding P at the top/left, the bottom /
// right padding follows from OH, OW).  Window rows have a pitch of a
// multiple of 4 floats and start at the block's first input column, so a
// thread's reads are 16-byte aligned.  Each output sums over ic, kh, kw in
// that order with fmaf, then adds the bias.
constexpr int kDirectRows = 16, kDirectCols = 64, kDirectOCB = 16;
template <int K, int S>
__global__ void __launch_bounds__(256)
conv_direct_kernel(const float *__restrict__ x, long long xbs, const float *__restrict__ w,
                   const float *__restrict__ bias, float *__restrict__ y, long long ybs, int IC,
                   int H, int W, int OC, int OH, int OW, int P, int act, int tiles_x, int ICB) {
    pdl_begin();
    constexpr int NX = 3 * S + K;        // window values of a thread's 4 pixels per row
    constexpr int N4 = (NX + 3) / 4;     // float4 reads covering them
    constexpr int IH = (kDirectRows - 1) * S + K;
    constexpr int IWP = ((kDirectCols / 4 - 1) * 4 * S + 4 * N4 + 3) / 4 * 4;  // row pitch
    constexpr int IW = (kDirectCols - 1) * S + K;  // columns copied
    extern __shared__ float4 dsm4[];
    float *ws = reinterpret_cast<float *>(dsm4);           // [IC * K * K][16]
    float *xs = ws + (size_t)IC * K * K * kDirectOCB;      // [ICB][IH][IWP]
    const int tyi = blockIdx.x / tiles_x;
    const int tx0 = (blockIdx.x - tyi * tiles_x) * kDirectCols, ty0 = tyi * kDirectRows;
    const int oc0 = blockIdx.y * kDirectOCB, b = blockIdx.z;
    const int t = threadIdx.x, ly = t >> 4, lx = t & 15;  // output row, 4-pixel group
    for (int i = t; i < IC * K * K * kDirectOCB; i += blockDim.x) {
        const int j = i & (kDirectOCB - 1), tap = i >> 4;  // tap = (ic * K + kh) * K + kw
        ws[i] = oc0 + j < OC ? __ldg(w + (long long)(oc0 + j) * IC * K * K + tap) : 0.0f;
    }
    const float *xb = x + (long long)b * xbs;
    const int iy0 = ty0 * S - P, ix0 = tx0 * S - P;
    const uint32_t xs_s = (uint32_t)__cvta_generic_to_shared(xs);
    float acc[4][kDirectOCB];
#pragma unroll
    for (int p = 0; p < 4; p++)
#pragma unroll
        for (int j = 0; j < kDirectOCB; j++) acc[p][j] = 0.0f;
    for (int ic0 = 0; ic0 < IC; ic0 += ICB) {
        const int nc = IC - ic0 < ICB ? IC - ic0 : ICB;
        __syncthreads();  // the previous chunk is consumed (and the weights written)
        // one window row per warp pass: 16-byte copies of 4 columns where the
        // row and the 4 columns allow, 4-byte copies (zero-filled outside the
        // input) elsewhere
        const int warp = t >> 5, lane = t & 31;
        for (int rr = warp; rr < nc * IH; rr += 8) {  // rr = c * IH + r
            const int c = rr / IH, r = rr - c * IH;
            const int iy = iy0 + r;
            const uint32_t drow = xs_s + (uint32_t)(rr * IWP) * 4u;
            if ((unsigned)iy >= (unsigned)H) {
                for (int q = lane; q < IW; q += 32) cp_async_zfill4(drow + 4u * q, xb, false);
                continue;
            }
            const float *srow = xb + (long long)(ic0 + c) * H * W + (long long)iy * W;
            const bool vec = ((uintptr_t)(srow + ix0) & 15) == 0;
            for (int q4 = 4 * lane; q4 < IW; q4 += 128) {
                const int ix = ix0 + q4;
                if (vec && ix >= 0 && ix + 3 < W && q4 + 3 < IWP) {
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(drow + 4u * q4),
                                 "l"(srow + ix)
                                 : "memory");
                } else {
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const bool in = ix + u >= 0 && ix + u < W && q4 + u < IW;
                        if (q4 + u < IW) cp_async_zfill4(drow + 4u * (q4 + u), in ? srow + ix + u : xb, in);
                    }
                }
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        for (int c = 0; c < nc; c++) {
            const float4 *wc = reinterpret_cast<const float4 *>(ws) +
                               (size_t)(ic0 + c) * K * K * (kDirectOCB / 4);
#pragma unroll
            for (int kh = 0; kh < K; kh++) {
                const float4 *xr = reinterpret_cast<const float4 *>(
                    xs + ((size_t)c * IH + ly * S + kh) * IWP + lx * 4 * S);
                float xv[4 * N4];
#pragma unroll
                for (int u = 0; u < N4; u++) {
                    const float4 v = xr[u];
                    xv[4 * u] = v.x; xv[4 * u + 1] = v.y; xv[4 * u + 2] = v.z; xv[4 * u + 3] = v.w;
                }
#pragma unroll
                for (int kw = 0; kw < K; kw++) {
                    float wv[kDirectOCB];
#pragma unroll
                    for (int q = 0; q < kDirectOCB / 4; q++) {
                        const float4 v = wc[(kh * K + kw) * (kDirectOCB / 4) + q];
                        wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
                    }
#pragma unroll
                    for (int p = 0; p < 4; p++)
#pragma unroll
                        for (int j = 0; j < kDirectOCB; j++)
                            acc[p][j] = fmaf(xv[p * S + kw], wv[j], acc[p][j]);
                }
            }
        }
    }
    const int oy = ty0 + ly, ox0 = tx0 + 4 * lx;
    if (oy >= OH) return;
    float *yp = y + (long long)b * ybs + (long long)oy * OW;
#pragma unroll
    for (int j = 0; j < kDirectOCB; j++) {
        if (oc0 + j >= OC) break;
        const float bv = bias ? __ldg(bias + oc0 + j) : 0.0f;
        float *yc = yp + (long long)(oc0 + j) * OH * OW;
#pragma unroll
        for (int p = 0; p < 4; p++)
            if (ox0 + p < OW) yc[ox0 + p] = act_apply(__fadd_rn(acc[p][j], bv), act);
    }
}

// ---- 2x2 stride-1 max pool over the right/bottom zero-padded input ----------
// ggml_pad(x, 1, 1) + ggml_pool_2d(MAX, 2, 2, 1, 1, 0, 0) (src/ppdoclayout.cpp:621-625)
// 4 consecutive outputs of a row per thread (W a multiple of 4): two 16-byte
// row loads plus the next column, one 16-byte store
__global__ void maxpool2_pad_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                                    long long ybs, int C, int H, int W, int B) {
    pdl_begin();
    // grid (C*H*W / 1024, B)
    const int w4 = W >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= C * H * w4) return;
    const int c = i / (H * w4), p = i - c * (H * w4), b = blockIdx.y;
    const int oy = p / w4, ox = (p - oy * w4) * 4;
    const float *r0 = x + (long long)b * xbs + (long long)c * H * W + (long long)oy * W + ox;
    const bool has_down = oy + 1 < H, has_right = ox + 4 < W;
    const float4 a = *reinterpret_cast<const float4 *>(r0);
    const float4 d = has_down ? *reinterpret_cast<const float4 *>(r0 + W)
                              : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float a4 = has_right ? r0[4] : 0.0f;
    const float d4 = (has_right && has_down) ? r0[W + 4] : 0.0f;
    float4 o;
    o.x = fmaxf(fmaxf(a.x, a.y), fmaxf(d.x, d.y));
    o.y = fmaxf(fmaxf(a.y, a.z), fmaxf(d.y, d.z));
    o.z = fmaxf(fmaxf(a.z, a.w), fmaxf(d.z, d.w));
    o.w = fmaxf(fmaxf(a.w, a4), fmaxf(d.w, d4));
    *reinterpret_cast<float4 *>(y + (long long)b * ybs + (long long)c * H * W + (long long)oy * W +
                                ox) = o;
}

// ---- interpolation (ggml_interpolate, src/ppdoclayout.cpp:670-672) -----------
// NEAREST: src = (int)(dst / sf).  BILINEAR (no align-corners): src =
// (dst + 0.5) / sf - 0.5, floor, both taps clamped to the edge, fractional
// weight clamped to [0, 1].  Optionally adds into y (y = base + interp).
// rx / ry: 1 / sf when sf is a power of two (the quotient is then exact, so
// the product is the same number as the division), else 0: divide.
__device__ __forceinline__ float interp_div(float a, float sf, float r) {
    return r != 0.0f ? __fmul_rn(a, r) : __fdiv_rn(a, sf);
}
__device__ __forceinline__ float interp_one(const float *__restrict__ xp, int ox, int oy, int H,
                                            int W, float sfx, float sfy, float rx, float ry,
                                            int bilinear) {
    if (!bilinear) {
        const int sx = min((int)interp_div((float)ox, sfx, rx), W - 1);
        const int sy = min((int)interp_div((float)oy, sfy, ry), H - 1);
        return xp[(long long)sy * W + sx];
    }
    const float fx = __fsub_rn(interp_div(__fadd_rn((float)ox, 0.5f), sfx, rx), 0.5f);
    const float fy = __fsub_rn(interp_div(__fadd_rn((float)oy, 0.5f), sfy, ry), 0.5f);
    const float flx = floorf(fx), fly = floorf(fy);
    int x0 = (int)flx, y0 = (int)fly;
    int x1 = x0 + 1, y1 = y0 + 1;
    const float dx = fminf(fmaxf(__fsub_rn(fx, flx), 0.0f), 1.0f);
    const float dy = fminf(fmaxf(__fsub_rn(fy, fly), 0.0f), 1.0f);
    x0 = max(0, min(x0, W - 1)); x1 = max(0, min(x1, W - 1));
    y0 = max(0, min(y0, H - 1)); y1 = max(0, min(y1, H - 1));
    const float a = xp[(long long)y0 * W + x0], bq = xp[(long long)y0 * W + x1];
    const float cq = xp[(long long)y1 * W + x0], d = xp[(long long)y1 * W + x1];
    return a * (1.0f - dx) * (1.0f - dy) + bq * dx * (1.0f - dy) + cq * (1.0f - dx) * dy +
           d * dx * dy;
}

// V consecutive output pixels of a row per thread (V = 4: one 16-byte store,
// used when OW is a multiple of 4 and the planes are 16-byte aligned)
template <int V>
__global__ void interp_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                              long long ybs, const float *__restrict__ base, long long bbs, int C,
                              int H, int W, int OH, int OW, int bilinear, int B, float rx,
                              float ry) {
    pdl_begin();
    // grid (C*OH*OW / (256 V), B)
    const int ow = OW / V;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= C * OH * ow) return;
    const int c = i / (OH * ow), p = i - c * (OH * ow), b = blockIdx.y;
    const int oy = p / ow, ox0 = (p - oy * ow) * V;
    const float *xp = x + (long long)b * xbs + (long long)c * H * W;
    const float sfx = (float)OW / (float)W, sfy = (float)OH / (float)H;
    const long long off = (long long)c * OH * OW + (long long)oy * OW + ox0;
    float v[V];
#pragma unroll
    for (int e = 0; e < V; e++)
        v[e] = interp_one(xp, ox0 + e, oy, H, W, sfx, sfy, rx, ry, bilinear);
    if (V == 4) {
        if (base) {
            const float4 b4 = *reinterpret_cast<const float4 *>(base + (long long)b * bbs + off);
            v[0] = __fadd_rn(b4.x, v[0]);
            v[1] = __fadd_rn(b4.y, v[1]);
            v[2] = __fadd_rn(b4.z, v[2]);
            v[3] = __fadd_rn(b4.w, v[3]);
        }
        *reinterpret_cast<float4 *>(y + (long long)b * ybs + off) =
            make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
        for (int e = 0; e < V; e++) {
            if (base) v[e] = __fadd_rn(base[(long long)b * bbs + off + e], v[e]);
            y[(long long)b * ybs + off + e] = v[e];
        }
    }
}

// ---- CHW <-> token-major ([H*W][C]) through a shared-memory tile ------------
__global__ void transpose_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                                 long long ybs, int R, int Cc, long long ldx, long long ldy) {
    pdl_begin();
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

// ---- rows padded to 16-byte multiples ---------------------------------------
// y[b][c][h][w] = x[b][c][h][w] for w < W, 0 for W <= w < Wp (Wp % 4 == 0):
// the input of a tensor-core conv whose rows TMA cannot address otherwise.
// Each thread writes four floats with one 16-byte store.
__global__ void pad_rows_kernel(const float *__restrict__ x, long long xbs, float *__restrict__ y,
                                long long ybs, int C, int H, int W, int Wp) {
    pdl_begin();
    const int q = Wp >> 2;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long n = (long long)C * H * q;
    if (i >= n) return;
    const int b = blockIdx.y;
    const long long row = i / q;  // c * H + h
    const int w0 = (int)(i - row * q) * 4;
    const float *xr = x + (long long)b * xbs + row * W;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = w0 + e < W ? __ldg(xr + w0 + e) : 0.0f;
    reinterpret_cast<float4 *>(y + (long long)b * ybs + row * Wp)[w0 >> 2] =
        make_float4(v[0], v[1], v[2], v[3]);
}

inline int blocks(long long n, int t = 256) { return (int)((n + t - 1) / t); }

// grid of the per-page kernels: x over the channels x pixels (or tiles) of a
// page as one 32-bit index, y over pages
inline bool grid3_ok(long long pix, int ch, int b) {
    return pix > 0 && ch > 0 && pix * ch < (1LL << 31) && b > 0 && b <= 65535;
}
inline dim3 grid3(long long pix, int ch, int b) { return dim3(blocks(pix * ch), b); }

}  // namespace

Status launch_pad_rows(const float *x, long long xbs, float *y, long long ybs, int C, int H,
                       int W, int Wp, int B, cudaStream_t st) {
    if (C <= 0 || H <= 0 || W <= 0 || Wp < W || Wp % 4 || B <= 0 || B > 65535 ||
        ((uintptr_t)y & 15) || ybs % 4)
        return ERR_SHAPE;
    const long long n = (long long)C * H * (Wp / 4);
    pdl_launch(pad_rows_kernel, dim3(blocks(n), B), 256, 0, st, x, xbs, y, ybs, C, H, W, Wp);
    return cuda_status();
}

Status launch_wg4_input(const float *x, long long xbs, float *dt, int IC, int H, int W, int TW,
                        int TH, int pad, int B, cudaStream_t st, long long ldt, long long pstride,
                        long long bstride) {
    if (!grid3_ok((long long)TW * TH, IC, B)) return ERR_SHAPE;
    if (ldt <= 0) ldt = TW * TH;
    if (ldt < TW * TH) return ERR_SHAPE;
    if (pstride <= 0) pstride = IC * ldt;
    if (bstride <= 0) bstride = 36 * pstride;
    if (pad == 1 && W == 4 * TW && ((uintptr_t)x & 15) == 0 && xbs % 4 == 0)
        pdl_launch(wg4_input_vec_kernel, grid3((long long)TW * TH, IC, B), 256, 0, st, x, xbs, dt,
                   IC, H, W, TW, TH, B, ldt, pstride, bstride);
    else
        pdl_launch(wg4_input_kernel, grid3((long long)TW * TH, IC, B), 256, 0, st, x, xbs, dt, IC,
                   H, W, TW, TH, pad, B, ldt, pstride, bstride);
    return cuda_status();
}

Status launch_wg4_output(const float *yt, const float *bias, float *y, long long ybs,
                         const float *res, long long rbs, int res_mode, int OC, int OH, int OW,
                         int TW, int TH, int act, int B, cudaStream_t st, long long ldt,
                         long long pstride, long long bstride) {
    if (!grid3_ok((long long)TW * TH, OC, B)) return ERR_SHAPE;
    if (TW < (OW + 3) / 4 || TH < (OH + 3) / 4) return ERR_SHAPE;
    if (ldt <= 0) ldt = TW * TH;
    if (ldt < TW * TH) return ERR_SHAPE;
    if (pstride <= 0) pstride = OC * ldt;
    if (bstride <= 0) bstride = 36 * pstride;
    pdl_launch(wg4_output_kernel, grid3((long long)TW * TH, OC, B), 256, 0, st, yt, bias, y, ybs,
               res, rbs, res_mode, OC, OH, OW, TW, TH, act, B, ldt, pstride, bstride);
    return cuda_status();
}

Status launch_wg4_filter(const float *w, float *wg4, int IC, int OC, cudaStream_t st) {
    const long long n = 36LL * IC * OC;
    pdl_launch(wg4_filter_kernel, blocks(n), 256, 0, st, w, wg4, IC, OC);
    return cuda_status();
}

Status launch_rep_fold(const float *w3, const float *b3, const float *w1, const float *b1,
                       float *wm, float *bm, int IC, int OC, cudaStream_t st) {
    if (IC <= 0 || OC <= 0) return ERR_SHAPE;
    const long long n = 9LL * IC * OC;
    pdl_launch(rep_fold_kernel, blocks(n), 256, 0, st, w3, b3, w1, b1, wm, bm, IC, OC);
    return cuda_status();
}

Status launch_kmajor_split(const float *src, float *hi, float *lo, int planes, int IC, int ld,
                           long long pstride, int nc, cudaStream_t st) {
    if (planes <= 0 || IC <= 0 || nc <= 0 || ld < nc) return ERR_SHAPE;
    const long long n = (long long)planes * IC * nc;
    pdl_launch(kmajor_split_kernel, blocks(n), 256, 0, st, src, hi, lo, planes, IC, ld, pstride,
               nc);
    return cuda_status();
}

Status launch_wg4_kmajor_split(const float *wg4, float *hi, float *lo, int IC, int OC,
                               cudaStream_t st) {
    return launch_kmajor_split(wg4, hi, lo, 36, IC, OC, (long long)IC * OC, OC, st);
}

Status launch_dwconv(const float *x, long long xbs, const float *w, const float *bias, float *y,
                     long long ybs, int C, int H, int W, int K, int S, int P, int act, int B,
                     cudaStream_t st) {
    const int OH = (H + 2 * P - K) / S + 1, OW = (W + 2 * P - K) / S + 1;
    if (OH <= 0 || OW <= 0 || C <= 0 || C > 65535 || B <= 0 || B > 65535 || P < 0 || P >= K)
        return ERR_SHAPE;
    // whole-plane form: the zero-bordered plane with the rows and columns the
    // 4 x 4 output blocks read (their float4 row segments included), row
    // pitch a multiple of 4 floats
    {
        const int GX = (OW + 3) / 4, GY = (OH + 3) / 4;
        const int n4 = (3 * S + K + 3) / 4;
        int cols = (4 * GX - 1) * S + K;
        if (cols < 4 * (GX - 1) * S + 4 * n4) cols = 4 * (GX - 1) * S + 4 * n4;
        if (cols < W + 2 * P) cols = W + 2 * P;
        const int ld = (cols + 3) / 4 * 4;
        const int HPp = (4 * GY - 1) * S + K;
        const size_t plane_bytes = (size_t)HPp * ld * 4;
        // 8-byte copies: even P and W keep every pair wholly inside or outside
        // the image, and x, the page stride and the plane 8-byte aligned
        const int pairs = (P % 2 == 0 && W % 2 == 0 && ((uintptr_t)x & 7) == 0 && xbs % 2 == 0)
                              ? 1 : 0;
        // float2 stores: even rows, y and its page stride 8-byte aligned
        const int even = (OW % 2 == 0 && ((uintptr_t)y & 7) == 0 && ybs % 2 == 0) ? 1 : 0;
        if (plane_bytes <= kDwPlaneSmemMax && (long long)HPp * ld < (1LL << 31)) {
            const dim3 g(C, B);
            const int sm = (int)plane_bytes;
            // threads: the 4 x 4 blocks of the plane in as few passes of at most
            // 256 threads as possible, in whole warps (a 50 x 50 plane: 169
            // blocks, 192 threads), and at least 128 for the copy
            const int items = GX * GY;
            const int passes = (items + 255) / 256;
            int nthr = ((items + passes - 1) / passes + 31) / 32 * 32;
            if (nthr < 128) nthr = 128;
            const int af = act == ACT_NONE ? 0 : act == ACT_RELU ? 1 : 2;
#define PPDL_DW_PLANE(KK, SS, AA)                                                                 \
    do {                                                                                         \
        if (!smem_attr_once((const void *)dwconv_plane_kernel<KK, SS, AA>,                    \
                            (int)kDwPlaneSmemMax))                                       \
            return ERR_CUDA;                                                                 \
        pdl_launch(dwconv_plane_kernel<KK, SS, AA>, g, nthr, sm, st, x, xbs, w, bias, y, ybs,\
                   H, W, OH, OW, P, act, ld, HPp, GX, GY, pairs, even);                      \
    } while (0)
#define PPDL_DW_PLANE_ACT(KK, SS)                                                                 \
    do {                                                                                         \
        if (af == 0)                                                                             \
            PPDL_DW_PLANE(KK, SS, 0);                                                            \
        else if (af == 1)                                                                        \
            PPDL_DW_PLANE(KK, SS, 1);                                                            \
        else                                                                                     \
            PPDL_DW_PLANE(KK, SS, -1);                                                           \
    } while (0)
            if (K == 3 && S == 1)
                PPDL_DW_PLANE_ACT(3, 1);
            else if (K == 3 && S == 2)
                PPDL_DW_PLANE_ACT(3, 2);
            else if (K == 5 && S == 1)
                PPDL_DW_PLANE_ACT(5, 1);
            else if (K == 5 && S == 2)
                PPDL_DW_PLANE_ACT(5, 2);
            else
                return ERR_UNSUPPORTED;
#undef PPDL_DW_PLANE_ACT
#undef PPDL_DW_PLANE
            return cuda_status();
        }
    }
    // band form for larger planes: bands of BR output rows (a multiple of 4)
    // whose input rows fit kDwBandSmem bytes, unless not even four output rows do
    const int bcols = W + 2 * P;  // >= (OW - 1) S + K
    const int bld = (bcols + 30) / 32 * 32 + 1;
    const int rows_fit = (int)(kDwBandSmem / 4 / bld);
    if (rows_fit >= 3 * S + K) {
        int BR = ((rows_fit - K) / S + 1) / 4 * 4;
        const int OH4 = (OH + 3) / 4 * 4;
        if (BR > OH4) BR = OH4;
        const int nbands = (OH + BR - 1) / BR;
        // equal bands (the last one no shorter than needed)
        BR = ((OH + nbands - 1) / nbands + 3) / 4 * 4;
        const long long nblk = (long long)B * C * nbands;
        if (nblk > 0x7fffffffLL) return ERR_SHAPE;
        const int smem = ((BR - 1) * S + K) * bld * 4;
        // threads: the band's output groups in as few passes of at most 256
        // threads as possible, in whole warps
        const int items = ((BR + 3) / 4) * OW;
        const int passes = (items + 255) / 256;
        const int nthr = ((items + passes - 1) / passes + 31) / 32 * 32;
#define PPDL_DW_BAND(KK, SS)                                                                      \
    do {                                                                                         \
        if (!smem_attr_once((const void *)dwconv_band_kernel<KK, SS>, (int)kDwBandSmem))     \
            return ERR_CUDA;                                                                 \
        pdl_launch(dwconv_band_kernel<KK, SS>, (unsigned)nblk, nthr, smem, st, x, xbs, w,    \
                   bias, y, ybs, C, H, W, OH, OW, P, act, bld, bcols, BR, nbands);           \
    } while (0)
        if (K == 3 && S == 1)
            PPDL_DW_BAND(3, 1);
        else if (K == 3 && S == 2)
            PPDL_DW_BAND(3, 2);
        else if (K == 5 && S == 1)
            PPDL_DW_BAND(5, 1);
        else if (K == 5 && S == 2)
            PPDL_DW_BAND(5, 2);
        else
            return ERR_UNSUPPORTED;
#undef PPDL_DW_BAND
        return cuda_status();
    }
    const int tiles_x = (OW + kDwTW - 1) / kDwTW, tiles_y = (OH + kDwTH - 1) / kDwTH;
    const dim3 g(tiles_x * tiles_y, C, B);
    if (K == 3 && S == 1)
        pdl_launch(dwconv_kernel<3, 1>, g, 256, 0, st, x, xbs, w, bias, y, ybs, H, W, OH, OW, P,
                   act, tiles_x);
    else if (K == 3 && S == 2)
        pdl_launch(dwconv_kernel<3, 2>, g, 256, 0, st, x, xbs, w, bias, y, ybs, H, W, OH, OW, P,
                   act, tiles_x);
    else if (K == 5 && S == 1)
        pdl_launch(dwconv_kernel<5, 1>, g, 256, 0, st, x, xbs, w, bias, y, ybs, H, W, OH, OW, P,
                   act, tiles_x);
    else if (K == 5 && S == 2)
        pdl_launch(dwconv_kernel<5, 2>, g, 256, 0, st, x, xbs, w, bias, y, ybs, H, W, OH, OW, P,
                   act, tiles_x);
    else
        return ERR_UNSUPPORTED;
    return cuda_status();
}

bool conv_direct_ok(int IC, int OC, int K, int S) {
    return IC > 0 && OC > 0 && OC <= 32 && IC * K * K <= kDirectTaps && (K == 2 || K == 3) &&
           (S == 1 || S == 2);
}

Status launch_conv_direct(const float *x, long long xbs, const float *w, const float *bias,
                          float *y, long long ybs, int IC, int H, int W, int OC, int K, int S,
                          int P, int OH, int OW, int act, int B, cudaStream_t st) {
    if (!conv_direct_ok(IC, OC, K, S) || H <= 0 || W <= 0 || OH <= 0 || OW <= 0 || P < 0 ||
        P >= K || B <= 0 || B > 65535 || act < 0 || act > 3)
        return ERR_SHAPE;
    const int tiles_x = (OW + kDirectCols - 1) / kDirectCols;
    const int tiles_y = (OH + kDirectRows - 1) / kDirectRows;
    if ((long long)tiles_x * tiles_y > 0x7fffffffLL) return ERR_SHAPE;
    const int N4 = (3 * S + K + 3) / 4;
    const int IH = (kDirectRows - 1) * S + K;
    const int IWP = ((kDirectCols / 4 - 1) * 4 * S + 4 * N4 + 3) / 4 * 4;
    // input channels per chunk: a window of up to kDirectWindowBytes
    int ICB = (int)(kDirectWindowBytes / (4 * IH * IWP));
    if (ICB > IC) ICB = IC;
    if (ICB < 1) ICB = 1;
    const int smem = 4 * (IC * K * K * kDirectOCB + ICB * IH * IWP);
    const dim3 g((unsigned)(tiles_x * tiles_y), (unsigned)((OC + kDirectOCB - 1) / kDirectOCB),
                 (unsigned)B);
#define PPDL_DIRECT(KK, SS)                                                                       \
    do {                                                                                         \
        if (!smem_attr_once((const void *)conv_direct_kernel<KK, SS>, 64 * 1024))            \
            return ERR_CUDA;                                                                 \
        pdl_launch(conv_direct_kernel<KK, SS>, g, 256, smem, st, x, xbs, w, bias, y, ybs,    \
                   IC, H, W, OC, OH, OW, P, act, tiles_x, ICB);                              \
    } while (0)
    if (K == 2 && S == 1)
        PPDL_DIRECT(2, 1);
    else if (K == 2 && S == 2)
        PPDL_DIRECT(2, 2);
    else if (K == 3 && S == 1)
        PPDL_DIRECT(3, 1);
    else
        PPDL_DIRECT(3, 2);
#undef PPDL_DIRECT
    return cuda_status();
}

Status launch_maxpool2_pad(const float *x, long long xbs, float *y, long long ybs, int C, int H,
                           int W, int B, cudaStream_t st) {
    if (!grid3_ok((long long)H * W, C, B) || W % 4 || ((uintptr_t)x & 15) || xbs % 4 ||
        ((uintptr_t)y & 15) || ybs % 4)
        return ERR_SHAPE;
    pdl_launch(maxpool2_pad_kernel, grid3((long long)H * W / 4, C, B), 256, 0, st, x, xbs, y, ybs,
               C, H, W, B);
    return cuda_status();
}

Status launch_interp(const float *x, long long xbs, float *y, long long ybs, const float *base,
                     long long bbs, int C, int H, int W, int OH, int OW, bool bilinear, int B,
                     cudaStream_t st) {
    if (!grid3_ok((long long)OH * OW, C, B)) return ERR_SHAPE;
    const bool vec = OW % 4 == 0 && ((uintptr_t)y & 15) == 0 && ybs % 4 == 0 &&
                     (!base || (((uintptr_t)base & 15) == 0 && bbs % 4 == 0));
    // 1 / sf when the kernel's sf = out / in is a power of two (the forward's
    // 2x upsamples), so that it multiplies instead of dividing
    auto exact_recip = [](int out, int in) -> float {
        const float sf = (float)out / (float)in;
        int e = 0;
        return std::frexp(sf, &e) == 0.5f ? 1.0f / sf : 0.0f;
    };
    const float rx = exact_recip(OW, W), ry = exact_recip(OH, H);
    if (vec)
        pdl_launch(interp_kernel<4>, grid3((long long)OH * OW / 4, C, B), 256, 0, st, x, xbs, y,
                   ybs, base, bbs, C, H, W, OH, OW, bilinear ? 1 : 0, B, rx, ry);
    else
        pdl_launch(interp_kernel<1>, grid3((long long)OH * OW, C, B), 256, 0, st, x, xbs, y, ybs,
                   base, bbs, C, H, W, OH, OW, bilinear ? 1 : 0, B, rx, ry);
    return cuda_status();
}

Status launch_transpose(const float *x, long long xbs, float *y, long long ybs, int R, int Cc,
                        long long ldx, long long ldy, int B, cudaStream_t st) {
    dim3 grid((unsigned)cdiv(Cc, 32), (unsigned)cdiv(R, 32), (unsigned)B);
    pdl_launch(transpose_kernel, grid, dim3(32, 8), 0, st, x, xbs, y, ybs, R, Cc, ldx, ldy);
    (void)sm_count;
    return cuda_status();
}

}  // namespace ppdl
