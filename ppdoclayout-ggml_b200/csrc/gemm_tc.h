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

struct TcGemm {
    CUtensorMap tmA, tmBhi, tmBlo;
    CUtensorMap tmC;     // output stored by TMA: tma_c 1 = CHW, 2 = token-major rows
    int tma_c = 0;
    int M = 0, N = 0, K = 0, batch = 1, planes = 1;
    int a_mn = 1;        // 1: A is M-major (128B-base-32B swizzle), 0: K-major
    int gather = 0;      // 1: A gathered by the converter warps (conv geometry gg)
    TcGather gg;
    int bn = 128;        // N tile
    int stages = 2;
    size_t smem = 0;
    int m_tiles = 0, n_tiles = 0, tiles = 0;
    int max_ctas = 0;    // > 0: at most this many CTAs (SMs left to concurrent launches)
    TcEpilogue epi;
    bool ok = false;
};

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

Status launch_tc_gemm(const TcGemm &g, cudaStream_t st);

// Device error flag of the tensor-core kernels (set when a bounded wait gave
// up); reads and clears it.
int tc_error_fetch_and_clear();

}  // namespace ppdl
