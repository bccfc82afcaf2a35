// conv.h — launchers of conv.cu (Winograd transforms, depthwise, glue).
//
// Tensors are CHW per page; "xbs"/"ybs" are the page strides in floats, so a
// view may be a channel slice of a wider (concatenated) buffer.
#pragma once

#include "common.cuh"

namespace ppdl {

// x [B][IC][H][W] -> dt, tiles TW x TH of 4x4 outputs; `pad` is the
// left/top zero padding (1 for a k3-s1-p1 conv on the unpadded tensor, 0 for
// the reference's op 10 on an already padded tensor).  Value (page b, plane
// p, channel ic, tile t) at dt[b*bstride + p*pstride + ic*ldt + t]; the
// defaults (0) give [B*36][IC][ldt] with ldt = T.
Status launch_wg4_input(const float *x, long long xbs, float *dt, int IC, int H, int W, int TW,
                        int TH, int pad, int B, cudaStream_t st, long long ldt = 0,
                        long long pstride = 0, long long bstride = 0);

// yt (addressed as dt above, OC channels) -> y = act(A^T m A + bias (+res if
// res_mode==1)) (+res if res_mode==2), y/res [B][OC][OH][OW] views.
Status launch_wg4_output(const float *yt, const float *bias, float *y, long long ybs,
                         const float *res, long long rbs, int res_mode, int OC, int OH, int OW,
                         int TW, int TH, int act, int B, cudaStream_t st, long long ldt = 0,
                         long long pstride = 0, long long bstride = 0);

// wg4 [36][IC][OC] -> K-major TF32 halves hi/lo [36][OC][IC]
Status launch_wg4_kmajor_split(const float *wg4, float *hi, float *lo, int IC, int OC,
                               cudaStream_t st);

// The general form: src[p][ic][n0 + oc] (row stride ld, plane stride pstride,
// src already offset by n0) -> hi/lo [planes][nc][IC]
Status launch_kmajor_split(const float *src, float *hi, float *lo, int planes, int IC, int ld,
                           long long pstride, int nc, cudaStream_t st);

// RepVGG fold: wm = w3 [OC][IC][3][3] with w1 [OC][IC] added to the centre
// tap, bm = b3 + b1 (wm: 9 IC OC floats, bm: OC floats)
Status launch_rep_fold(const float *w3, const float *b3, const float *w1, const float *b1,
                       float *wm, float *bm, int IC, int OC, cudaStream_t st);

// w [OC][IC][3][3] -> wg4 [36][IC][OC] (G g G^T with the reference's G)
Status launch_wg4_filter(const float *w, float *wg4, int IC, int OC, cudaStream_t st);

// depthwise KxK (K in {3,5}) conv + bias + act, symmetric padding P
Status launch_dwconv(const float *x, long long xbs, const float *w, const float *bias, float *y,
                     long long ybs, int C, int H, int W, int K, int S, int P, int act, int B,
                     cudaStream_t st);

// 2x2 stride-1 max pool of the input zero-padded by one row/column at the
// end: out is H x W like the input (W a multiple of 4, 16-byte aligned planes)
// Direct FP32 conv for narrow convs: OC <= 32, IC*K*K <= 128, K 2..3, S 1..2.
// y[b][oc] = act(bias + sum_{ic,kh,kw} w[oc][ic][kh][kw] x[b][ic][oy S + kh - P][ox S + kw - P]),
// zero outside H x W (bottom/right padding from OH, OW); bias may be null.
bool conv_direct_ok(int IC, int OC, int K, int S);
Status launch_conv_direct(const float *x, long long xbs, const float *w, const float *bias,
                          float *y, long long ybs, int IC, int H, int W, int OC, int K, int S,
                          int P, int OH, int OW, int act, int B, cudaStream_t st);

Status launch_maxpool2_pad(const float *x, long long xbs, float *y, long long ybs, int C, int H,
                           int W, int B, cudaStream_t st);

// ggml_interpolate nearest / bilinear (no align-corners); y = base + interp
// when base is non-null
Status launch_interp(const float *x, long long xbs, float *y, long long ybs, const float *base,
                     long long bbs, int C, int H, int W, int OH, int OW, bool bilinear, int B,
                     cudaStream_t st);

// rows of the C x H x W pages copied into rows of Wp floats (Wp % 4 == 0,
// zero past W): the input of a tensor-core conv whose rows are not 16-byte
// multiples
Status launch_pad_rows(const float *x, long long xbs, float *y, long long ybs, int C, int H,
                       int W, int Wp, int B, cudaStream_t st);

// y[c][r] = x[r][c] for an R x Cc matrix per page (row strides ldx, ldy)
Status launch_transpose(const float *x, long long xbs, float *y, long long ybs, int R, int Cc,
                        long long ldx, long long ldy, int B, cudaStream_t st);

}  // namespace ppdl
