// gemm_tc.h — FP32-faithful tensor-core GEMM for sm_100a (tcgen05 + TMEM +
// TMA), 3xTF32 split.
//
//   C[z](m, n) = post(act(alpha * sum_k A[z](m, k) B[z % planes](n, k) + bias[n] + pre))
//
// A is an FP32 activation, either M-major (CHW conv input: A(m = pixel,
// k = channel) with pixels contiguous) or K-major (token-major rows); it is
// loaded by TMA and split into hi/lo TF32 halves in shared memory.  B is a
// weight pre-split at init into hi/lo arrays, K-major [planes][N][K].
// Each MMA step accumulates hi*hi + hi*lo + lo*hi in FP32 in TMEM.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ppdl {

struct TcEpilogue {
    float *C = nullptr;
    long long ldc_m = 0, ldc_n = 0, c_bs = 0;  // batch stride per z
    const float *bias = nullptr;               // per n, may be null
    const float *res = nullptr;                // residual, C-like addressing
    long long res_ldm = 0, res_ldn = 0, res_bs = 0;
    int res_mode = 0;                          // 1 before, 2 after the activation
    int act = ACT_NONE;
    float alpha = 1.0f;
};

// Convolution read directly from a CHW input (implicit GEMM, no im2col):
// A(m, k) = x[z][ic][oy*S + kh - P][ox*S + kw - P], zero outside H x W,
// with m = oy*OW + ox and k = (ic*KS + kh)*KS + kw — the row order of the
// raw conv weight [OC][IC][KS][KS], so B is that weight as [OC][IC*KS*KS].
// Any plane size and channel stride works (no TMA on A): the converter
// warps gather the A tile from global memory into the K-major swizzled
// layout.  Bottom/right-only padding is expressed by OH/OW alone.
struct TcGather {
    const float *x = nullptr;
    long long x_bs = 0;      // page stride (elements)
    long long plane = 0;     // channel stride (elements), H*W for a dense CHW tensor
    int KS = 1, S = 1, P = 0, H = 0, W = 0, OW = 0;
};

// Implicit convolution fed by TMA boxes of the CHW input (no im2col, no
// per-element gather).  The output is tiled in 4 rows x 32 columns; for
// each kernel row kh and block of CB input channels one TMA box brings the
// input window of the tile (32*S + KS + alignment columns, 4 rows at the
// conv stride, CB channels; zero outside the image) into shared memory, and
// the converter warps read the A rows of all KS kernel columns from it.
// K order of the repacked weight (launch_tf32_split_box): box
// bx = cb*KS + kh, inside a box k = kw*CB + c, each box padded to
// kbpb k-blocks of 32.  Needs W % 4 == 0 (16-byte input rows), S in {1, 2}
// and, for S = 2, an even H (rows are addressed as (H/2, parity) pairs).
struct TcConvBox {
    const float *x = nullptr;
    long long x_bs = 0;   // page stride (elements)
    int IC = 0, H = 0, W = 0, KS = 1, S = 1, P = 0, OH = 0, OW = 0;
    // derived by the planner
    int CB = 32, lcb = 5, kbpb = 1, nbx = 1, Wb = 0, o = 0, tiles_x = 0, tiles_y = 0, nbox = 2;
    uint32_t box_bytes = 0;  // window slot in shared memory (1024-byte multiple)
    uint32_t box_tx = 0;     // bytes one window load transfers (Wb * 4 * 32 * 4)
};

// Channels per window and k-blocks per window.  CB = the power of two >= IC
// (at least 4) when all KS kernel columns of CB channels fit one k-block of
// 32 (then k = kw * CB + c inside the window's single k-block), else 32
// (one k-block per kernel column); channels past IC are zero-filled by TMA.
// The repacked weight has nbx * kbpb * 32 columns, nbx = ceil(IC / CB) * KS.
inline void tc_conv_box_blocks(int IC, int KS, int *CB, int *kbpb, int *nbx) {
    int cb = 4;
    while (cb < IC && cb < 32) cb *= 2;
    if (KS * cb > 32) cb = 32;
    *CB = cb;
    *kbpb = cb == 32 ? KS : 1;
    *nbx = (IC + cb - 1) / cb * KS;
}
inline int tc_conv_box_kdim(int IC, int KS) {
    int cb, kbpb, nbx;
    tc_conv_box_blocks(IC, KS, &cb, &kbpb, &nbx);
    return nbx * kbpb * 32;
}

struct TcGemm {
    CUtensorMap tmA, tmBhi, tmBlo;
    CUtensorMap tmC;     // output stored by TMA: tma_c 1 = CHW, 2 = token-major rows
    int tma_c = 0;
    int M = 0, N = 0, K = 0, batch = 1, planes = 1;
    int a_mn = 1;        // 1: A is M-major (128B-base-32B swizzle), 0: K-major
    int gather = 0;      // 1: A gathered by the converter warps (conv geometry gg)
    TcGather gg;
    int box = 0;         // 1: implicit conv from TMA boxes of the input (geometry cb)
    TcConvBox cb;
    int bits = 0;        // 1: output packed 1 bit per element (tc_gemm_set_bits_output)
    int rows = 0;        // 1: M-major A loaded as 32 channel rows per k-block (rows_plane)
    long long rows_plane = 0;
    int rows_delta = 0;
    int bn = 128;        // N tile
    int stages = 2;
    size_t smem = 0;
    int m_tiles = 0, n_tiles = 0, tiles = 0;
    int max_ctas = 0;    // > 0: at most this many CTAs (SMs left to concurrent launches)
    int kps = 0;         // > 0: split K, this many k-blocks per split (tc_gemm_set_split_k)
    TcEpilogue epi;      // with split K: the reduction's ops (the GEMM writes raw totals)
    float *ws = nullptr;  // split K: the splits' totals [splits][M][N]
    long long ws_bs = 0;  // split K: floats between two splits' totals
    bool ok = false;
};

// Plan a GEMM as tc_gemm_plan (batch 1, one B plane) with K split into
// `splits` ranges of k-blocks: the tiles of all ranges run as one launch and
// write their raw FP32 totals to ws [splits][M][N] (token-major, 16-byte
// aligned, splits * M * N floats); launch_tc_gemm then sums them in split
// order and applies epi (alpha, bias, residual, activation) in a second
// kernel.  For GEMMs with few output tiles and a long K (the decoder's
// 2048 -> 256 linear).  False when the form does not apply.
bool tc_gemm_plan_split_k(TcGemm *g, int M, int N, int K, const float *A, int a_mn, long long lda,
                          const float *Bhi, const float *Blo, const TcEpilogue &epi, int splits,
                          float *ws);

// The tile shape tc_gemm_plan_split_k would choose (no tensor maps encoded):
// splits after rounding, k-blocks per split, tiles of the launch, N tile.
bool tc_gemm_split_k_shape(int M, int N, int K, int splits, int *splits_out, int *kps, int *tiles,
                           int *bn);

// Pre-split a K-major weight [rows][K] into hi (low 13 mantissa bits
// cleared) and lo = w - hi.
Status launch_tf32_split(const float *w, float *hi, float *lo, long long n, cudaStream_t st);

// The same for a [rows][K] weight stored into [rows][Kp] halves (Kp >= K,
// columns K..Kp-1 zero), so that the halves' rows are 16-byte multiples.
Status launch_tf32_split_pad(const float *w, float *hi, float *lo, int rows, int K, int Kp,
                             cudaStream_t st);

// Plan a convolution GEMM with a gathered A (see TcGather): M = OH*OW per
// page, N = OC, K = IC*KS*KS, batch = pages, B hi/lo: [N][Kp] with
// Kp = round_up(K, 4).  The epilogue addresses C(m = pixel, n = channel).
bool tc_gemm_plan_gather(TcGemm *g, int M, int N, int K, int batch, const TcGather &gg,
                         const float *Bhi, const float *Blo, const TcEpilogue &epi);

// Plan a GEMM.  A: base pointer of page 0, a_mn ? (ld = stride of k) :
// (ld = stride of m); batch stride a_bs (elements).  B hi/lo: [planes][N][K].
// Returns false when the shape cannot use the tensor-core path (strides not
// 16-byte multiples, misaligned pointers) — the caller then uses the SIMT GEMM.
bool tc_gemm_plan(TcGemm *g, int M, int N, int K, int batch, const float *A, int a_mn,
                  long long lda, long long a_bs, const float *Bhi, const float *Blo, int planes,
                  const TcEpilogue &epi);

// Plan a conv in box mode (see TcConvBox): M = OH*OW per page, N = OC,
// batch = pages, B hi/lo: the weight repacked by launch_tf32_split_box.  The
// epilogue addresses C(m = oy*OW + ox, n = channel).  False when the
// geometry is outside the mode (the caller then keeps another path).
bool tc_gemm_plan_box(TcGemm *g, int N, int batch, const TcConvBox &cb, const float *Bhi,
                      const float *Blo, const TcEpilogue &epi);

// Plan a GEMM whose M-major A (a CHW activation, A(m, k) = x[z][k][m]) has
// channel rows that TMA cannot describe as one tensor (plane stride or base
// not 16-byte aligned, e.g. 25 x 25 planes): every k-block is loaded as 32
// per-channel TMA rows of 132 floats starting at the 16-byte boundary below
// the row (each in a 160-float slot, 128-byte aligned), and the converter
// indexes past the alignment remainder.
bool tc_gemm_plan_rows(TcGemm *g, int M, int N, int K, int batch, const float *x, long long plane,
                       long long x_bs, const float *Bhi, const float *Blo, const TcEpilogue &epi,
                       int planes = 1);

// Repack and split a conv weight [OC][IC][KS][KS] into the box-mode K order
// (hi/lo rows of tc_conv_box_kdim(IC, KS) floats, zero where no tap/channel).
Status launch_tf32_split_box(const float *w, float *hi, float *lo, int OC, int IC, int KS,
                             cudaStream_t st);

// Turn a planned tile-mode GEMM with no epilogue ops and M % 32 == 0 into
// one that writes C packed: bit (m & 31) of word bits[z * bits_bs +
// n * words_per_n + (m >> 5)] = (total(m, n) > 0).  False when the plan
// does not qualify.
bool tc_gemm_set_bits_output(TcGemm *g, uint32_t *bits, long long words_per_n, long long bits_bs);

Status launch_tc_gemm(const TcGemm &g, cudaStream_t st);

// Device error flag of the tensor-core kernels (set when a bounded wait gave
// up); reads and clears it.
int tc_error_fetch_and_clear();

}  // namespace ppdl
