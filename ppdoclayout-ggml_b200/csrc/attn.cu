// attn.cu — fused multi-head self-attention core, softmax(q k^T * s) v, for
// the encoder's AIFI layer and the decoder's self-attention
// (src/ppdoclayout.cpp:572-587: ggml_mul_mat(k, q) -> ggml_scale(1/sqrt(32))
// -> ggml_soft_max -> ggml_mul_mat with v, 8 heads x 32 dims).
//
// One block computes 32 queries of one (page, head): the score rows of the
// block stay in shared memory (32 x T floats), so the three ggml ops become
// one launch with no [heads][T][T] round trip through HBM.  The arithmetic
// keeps the reference's order of operations: each score is the FP32 dot
// product q . k (ascending dims) multiplied by the FP32 scale; the row softmax
// is max -> exp(x - max) -> sum -> x * (1 / sum) (the softmax_rows kernel's
// reduction); the output sums p_ij v_j over ascending keys.
#include "common.cuh"
#include "dec.h"

namespace ppdl {
namespace {

constexpr int kHeadDim = 32;  // head dim
constexpr int kBQ = 32;       // queries per block
constexpr int kKT = 64;       // keys per shared-memory tile
constexpr int kThreads = 256;

__device__ __forceinline__ float warp_max32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// q, k, v, o: token-major [B][T][ld] with head h at columns h*32 .. h*32+31.
// Shared memory: Q [32][33] | K or V tile [64][33] | scores [32][ldS].
__global__ void __launch_bounds__(kThreads)
attn_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
            float *__restrict__ o, int T, int ld, long long bs, float scale, int ldS) {
    extern __shared__ float sm[];
    float *Qs = sm;                 // [kBQ][33]
    float *Ts = Qs + kBQ * 33;      // [kKT][33]
    float *Ss = Ts + kKT * 33;      // [kBQ][ldS]
    const int q0 = blockIdx.x * kBQ, h = blockIdx.y, b = blockIdx.z;
    const int t = threadIdx.x, lane = t & 31, wq = t >> 5;  // wq: query group of 4
    const long long base = (long long)b * bs + h * kHeadDim;

    for (int i = t; i < kBQ * kHeadDim; i += kThreads) {
        const int r = i >> 5, d = i & 31;
        Qs[r * 33 + d] = q0 + r < T ? q[base + (long long)(q0 + r) * ld + d] : 0.0f;
    }
    // ---- scores: thread -> queries 4wq..4wq+3, keys lane and lane+32 of a tile
    for (int j0 = 0; j0 < T; j0 += kKT) {
        __syncthreads();
        for (int i = t; i < kKT * kHeadDim; i += kThreads) {
            const int r = i >> 5, d = i & 31;
            Ts[r * 33 + d] = j0 + r < T ? k[base + (long long)(j0 + r) * ld + d] : 0.0f;
        }
        __syncthreads();
        float acc[4][2];
#pragma unroll
        for (int r = 0; r < 4; r++) acc[r][0] = acc[r][1] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < kHeadDim; d++) {
            const float k0 = Ts[lane * 33 + d], k1 = Ts[(lane + 32) * 33 + d];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const float qv = Qs[(wq * 4 + r) * 33 + d];
                acc[r][0] = fmaf(qv, k0, acc[r][0]);
                acc[r][1] = fmaf(qv, k1, acc[r][1]);
            }
        }
#pragma unroll
        for (int r = 0; r < 4; r++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int j = j0 + lane + 32 * c;
                if (j < T) Ss[(wq * 4 + r) * ldS + j] = __fmul_rn(acc[r][c], scale);
            }
    }
    __syncthreads();
    // ---- row softmax: warp wq owns rows 4wq..4wq+3
#pragma unroll 1
    for (int r = 0; r < 4; r++) {
        float *p = Ss + (wq * 4 + r) * ldS;
        float m = -INFINITY;
        for (int j = lane; j < T; j += 32) m = fmaxf(m, p[j]);
        m = warp_max32(m);
        float s = 0.0f;
        for (int j = lane; j < T; j += 32) {
            const float e = expf(p[j] - m);
            p[j] = e;
            s += e;
        }
        s = warp_sum32(s);
        const float inv = 1.0f / s;
        for (int j = lane; j < T; j += 32) p[j] *= inv;
    }
    // ---- o = p v: thread -> queries 4wq..4wq+3, dim lane
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j0 = 0; j0 < T; j0 += kKT) {
        __syncthreads();
        for (int i = t; i < kKT * kHeadDim; i += kThreads) {
            const int r = i >> 5, d = i & 31;
            Ts[r * 33 + d] = j0 + r < T ? v[base + (long long)(j0 + r) * ld + d] : 0.0f;
        }
        __syncthreads();
        const int jn = T - j0 < kKT ? T - j0 : kKT;
#pragma unroll 4
        for (int jj = 0; jj < jn; jj++) {
            const float vv = Ts[jj * 33 + lane];
#pragma unroll
            for (int r = 0; r < 4; r++) acc[r] = fmaf(Ss[(wq * 4 + r) * ldS + j0 + jj], vv, acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int i = q0 + wq * 4 + r;
        if (i < T) o[base + (long long)i * ld + lane] = acc[r];
    }
}

size_t attention_smem_bytes(int T) {
    const int ldS = (T + 3) / 4 * 4 + 1;
    return sizeof(float) * ((size_t)kBQ * 33 + (size_t)kKT * 33 + (size_t)kBQ * ldS);
}

}  // namespace

Status launch_attention(const float *q, const float *k, const float *v, float *o, int T, int heads,
                        int ld, long long bs, float scale, int B, cudaStream_t st) {
    if (T <= 0 || heads <= 0 || heads > 65535 || B <= 0 || B > 65535 || ld < heads * kHeadDim)
        return ERR_SHAPE;
    const size_t smem = attention_smem_bytes(T);
    if (smem > 227 * 1024) return ERR_SHAPE;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        if (cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 227 * 1024) != cudaSuccess)
            return ERR_CUDA;
        attr[dev] = true;
    }
    const int ldS = (T + 3) / 4 * 4 + 1;
    attn_kernel<<<dim3((T + kBQ - 1) / kBQ, heads, B), kThreads, smem, st>>>(q, k, v, o, T, ld,
                                                                          bs, scale, ldS);
    return cuda_status();
}

}  // namespace ppdl
