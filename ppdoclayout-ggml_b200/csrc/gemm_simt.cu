// gemm_simt.cu — exact-FP32 FFMA GEMM (the SIMT path of every contraction).
//
// The reference runs its FP32 contractions as cuBLAS SGEMM with TF32 off
// (patches/ggml-ppdl.patch:14-16, 650-665, 787-802) or as SIMT FFMA kernels
// (patch:332-415).  This kernel is the same arithmetic class — one FFMA per
// multiply-add, FP32 accumulation — written as a register-tiled SIMT GEMM:
// a block computes a BM x BN tile with 256 threads (each a (BM/16) x (BN/16)
// micro-tile), K advances in BK slices staged through double-buffered
// shared memory with the next slice prefetched into registers.  Operands
// may be K-contiguous or M/N-contiguous (template), so CHW activations feed
// it without a transpose.  The fused epilogue applies alpha, bias, an
// optional residual (before or after the activation) and the activation,
// and stores through arbitrary strides (CHW or token-major).
#include "gemm.h"
#include "kernels.h"

namespace ppdl {

namespace {

constexpr int kThreads = 256;

template <int BM, int BN, int BK, bool kAK, bool kBN, bool kConv>
__global__ void __launch_bounds__(kThreads)
gemm_simt_kernel(const GemmArgs g) {
    pdl_begin();
    constexpr int TM = BM / 16, TN = BN / 16;
    constexpr int LA = BM * BK / kThreads, LB = BK * BN / kThreads;
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Bs[2][BK][BN + 4];

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const long long z = blockIdx.z;
    const float *A = g.A.p + batch_off(z, g.A.div, g.A.bs_hi, g.A.bs_lo);
    const float *B = g.B.p + batch_off(z, g.B.div, g.B.bs_hi, g.B.bs_lo);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int M = g.M, N = g.N, K = g.K;

    float ra[LA], rb[LB];
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < LA; i++) {
            const int e = tid + i * kThreads;
            int mm, kk;
            if (kAK) { mm = e / BK; kk = e % BK; } else { kk = e / BM; mm = e % BM; }
            const int m = m0 + mm, k = k0 + kk;
            ra[i] = (m < M && k < K) ? __ldg(A + (long long)m * g.A.s0 + (long long)k * g.A.s1) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < LB; i++) {
            const int e = tid + i * kThreads;
            int kk, nn;
            if (kBN) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
            const int n = n0 + nn, k = k0 + kk;
            if (kConv) {
                float v = 0.0f;
                if (n < N && k < K) {
                    const int KK = g.conv.K * g.conv.K;
                    int ic, r;
                    if (g.conv.tap_major) { r = k / g.conv.IC; ic = k - r * g.conv.IC; }
                    else { ic = k / KK; r = k - ic * KK; }
                    const int kh = r / g.conv.K, kw = r - kh * g.conv.K;
                    const int oy = n / g.conv.OW, ox = n - oy * g.conv.OW;
                    const int iy = oy * g.conv.S + kh - g.conv.P;
                    const int ix = ox * g.conv.S + kw - g.conv.P;
                    if (iy >= 0 && iy < g.conv.H && ix >= 0 && ix < g.conv.W)
                        v = __ldg(B + ((long long)ic * g.conv.H + iy) * g.conv.W + ix);
                }
                rb[i] = v;
            } else {
                rb[i] = (n < N && k < K) ? __ldg(B + (long long)k * g.B.s0 + (long long)n * g.B.s1)
                                         : 0.0f;
            }
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < LA; i++) {
            const int e = tid + i * kThreads;
            int mm, kk;
            if (kAK) { mm = e / BK; kk = e % BK; } else { kk = e / BM; mm = e % BM; }
            As[buf][kk][mm] = ra[i];
        }
#pragma unroll
        for (int i = 0; i < LB; i++) {
            const int e = tid + i * kThreads;
            int kk, nn;
            if (kBN) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
            Bs[buf][kk][nn] = rb[i];
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0.0f;

    const int nk = (K + BK - 1) / BK;
    load(0);
    store(0);
    __syncthreads();
    for (int t = 0; t < nk; t++) {
        const int buf = t & 1;
        if (t + 1 < nk) load((t + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[TM], b[TN];
            // rows ty*TM/2 + {0..TM/2-1} and 64/..: split halves keep the
            // float4 shared loads conflict-free
#pragma unroll
            for (int i = 0; i < TM; i += 4) {
                const int mi = (i < TM / 2 ? ty * (TM / 2) + i : BM / 2 + ty * (TM / 2) + i - TM / 2);
                if (TM / 2 >= 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(&As[buf][kk][mi]);
                    a[i] = v.x; a[i + 1] = v.y; a[i + 2] = v.z; a[i + 3] = v.w;
                } else {
#pragma unroll
                    for (int u = 0; u < 4 && i + u < TM; u++) {
                        const int iu = i + u;
                        const int mu = (iu < TM / 2 ? ty * (TM / 2) + iu
                                                    : BM / 2 + ty * (TM / 2) + iu - TM / 2);
                        a[iu] = As[buf][kk][mu];
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < TN; j += 4) {
                const int nj = (j < TN / 2 ? tx * (TN / 2) + j : BN / 2 + tx * (TN / 2) + j - TN / 2);
                const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][kk][nj]);
                b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (t + 1 < nk) {
            store(buf ^ 1);
            __syncthreads();
        }
    }

    // epilogue
    float *C = g.C + batch_off(z, g.c_div, g.c_bs_hi, g.c_bs_lo);
    const float *R = g.res_mode ? g.res.p + batch_off(z, g.res.div, g.res.bs_hi, g.res.bs_lo)
                                : nullptr;
#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = m0 + (i < TM / 2 ? ty * (TM / 2) + i : BM / 2 + ty * (TM / 2) + i - TM / 2);
        if (m >= M) continue;
        const float bm = g.bias_mode == 1 ? g.bias[m] : 0.0f;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = n0 + (j < TN / 2 ? tx * (TN / 2) + j : BN / 2 + tx * (TN / 2) + j - TN / 2);
            if (n >= N) continue;
            float v = acc[i][j];
            if (g.alpha != 1.0f) v = v * g.alpha;
            if (g.bias_mode == 1) v = v + bm;
            else if (g.bias_mode == 2) v = v + g.bias[n];
            if (g.res_mode == 1) v = v + R[(long long)m * g.res.s0 + (long long)n * g.res.s1];
            v = act_apply(v, g.act);
            if (g.res_mode == 2) v = v + R[(long long)m * g.res.s0 + (long long)n * g.res.s1];
            C[(long long)m * g.ldc_m + (long long)n * g.ldc_n] = v;
        }
    }
}

template <int BM, int BN, int BK>
Status dispatch(const GemmArgs &g, cudaStream_t stream) {
    const bool ak = g.A.s1 == 1;  // k contiguous
    const bool bn = g.B.s1 == 1;  // n contiguous
    dim3 grid((unsigned)cdiv(g.N, BN), (unsigned)cdiv(g.M, BM), (unsigned)g.batch);
    if (g.conv.K > 0) {
        if (ak) pdl_launch(gemm_simt_kernel<BM, BN, BK, true, true, true>, grid, kThreads, 0,
                           stream, g);
        else pdl_launch(gemm_simt_kernel<BM, BN, BK, false, true, true>, grid, kThreads, 0, stream,
                        g);
    } else if (ak && bn) {
        pdl_launch(gemm_simt_kernel<BM, BN, BK, true, true, false>, grid, kThreads, 0, stream, g);
    } else if (ak) {
        pdl_launch(gemm_simt_kernel<BM, BN, BK, true, false, false>, grid, kThreads, 0, stream, g);
    } else if (bn) {
        pdl_launch(gemm_simt_kernel<BM, BN, BK, false, true, false>, grid, kThreads, 0, stream, g);
    } else {
        pdl_launch(gemm_simt_kernel<BM, BN, BK, false, false, false>, grid, kThreads, 0, stream, g);
    }
    return cuda_status();
}

}  // namespace

Status launch_gemm_simt(const GemmArgs &g, cudaStream_t stream) {
    if (g.M < 0 || g.N < 0 || g.K < 0 || g.batch < 0) return ERR_SHAPE;
    if (g.M == 0 || g.N == 0 || g.batch == 0) return OK;
    if (g.batch > 65535) return ERR_SHAPE;
    if (g.A.s0 != 1 && g.A.s1 != 1) return ERR_SHAPE;
    if (g.conv.K == 0 && g.B.s0 != 1 && g.B.s1 != 1) return ERR_SHAPE;
    if (g.conv.K > 0 && (g.conv.OW <= 0 || (long long)g.N % g.conv.OW != 0)) return ERR_SHAPE;
    if (g.bias_mode && !g.bias) return ERR_SHAPE;
    if (g.res_mode && !g.res.p) return ERR_SHAPE;
    if (g.M <= 32) return dispatch<32, 128, 8>(g, stream);
    if (g.M <= 64) return dispatch<64, 128, 8>(g, stream);
    return dispatch<128, 128, 8>(g, stream);
}

}  // namespace ppdl
