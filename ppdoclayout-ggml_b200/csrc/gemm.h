// gemm.h — strided, batched FP32 GEMM with a fused epilogue.
//
//   C[z](m,n) = post( act( alpha * sum_k A[z](m,k) B[z](k,n) + bias + pre ) )
//
// Every operand is addressed by two strides and a two-level batch offset
// off(z) = (z / div) * bs_hi + (z % div) * bs_lo, which covers the CHW conv
// GEMMs (pages x channel slices of a concat buffer), the 36-plane Winograd
// madd (weights indexed by plane = z % 36) and the per-head attention
// products.  One of (lda_m, lda_k) and one of (ldb_k, ldb_n) must be 1.
#pragma once

#include "common.cuh"

namespace ppdl {

struct Operand {
    const float *p = nullptr;
    long long s0 = 0, s1 = 0;         // strides of the two logical dims
    long long div = 1, bs_hi = 0, bs_lo = 0;
};

// Implicit-GEMM convolution: when K > 0 the B operand is not a matrix but
// the CHW input of page z (B.p + off(z)) read through the conv geometry,
// B(k, n) = x[ic][oy*S + kh - P][ox*S + kw - P] (zero outside H x W) with
// k = (ic*K + kh)*K + kw and n = oy*OW + ox — no im2col is materialised.
// tap_major = 1 orders k as (kh*K + kw)*IC + ic instead, the row order of
// the reference's repacked ".wr" weights (src/ppdoclayout.cpp:273-280).
struct ConvGeom {
    int K = 0, S = 1, P = 0, H = 0, W = 0, OW = 0, IC = 0, tap_major = 0;
};

struct GemmArgs {
    int M = 0, N = 0, K = 0, batch = 1;
    ConvGeom conv;
    Operand A;        // (m, k): s0 = stride of m, s1 = stride of k
    Operand B;        // (k, n): s0 = stride of k, s1 = stride of n
    float *C = nullptr;
    long long ldc_m = 0, ldc_n = 1, c_div = 1, c_bs_hi = 0, c_bs_lo = 0;
    float alpha = 1.0f;
    const float *bias = nullptr;
    int bias_mode = 0;  // 0 none, 1 per row m, 2 per column n
    Operand res;        // residual (m, n) with C-like strides, s0 = m, s1 = n
    int res_mode = 0;   // 0 none, 1 added before the activation, 2 after it
    int act = ACT_NONE;
};

__host__ __device__ inline long long batch_off(long long z, long long div, long long hi,
                                                long long lo) {
    return (z / div) * hi + (z % div) * lo;
}

// FFMA (SIMT) GEMM: the exact-FP32 path, used for every contraction whose
// shape does not go to the tensor-core kernel.
Status launch_gemm_simt(const GemmArgs &g, cudaStream_t stream);

}  // namespace ppdl
