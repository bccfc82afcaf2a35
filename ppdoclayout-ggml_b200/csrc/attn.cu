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
// queries per block: a warp per 4 queries.  Single-tile sequences take 40
// (10 warps): the decoder's 300 queries x 8 heads x 8 pages are then 512
// blocks, two waves of two blocks per SM, where 32 made 640 (a third wave
// one-sixth full); the streamed form keeps 32 (two blocks per SM fit).
constexpr int kBQAll = 40, kBQStream = 32;
constexpr int kLD = 36;       // row stride of the Q and K/V tiles
// Key tiles: sequences of up to kKTAll keys (the decoder's 300 queries) keep
// all keys in one tile, so K and then V each arrive with one wait (V's
// during the softmax) in a single buffer; longer ones (AIFI's 625 tokens)
// stream tiles of 64 keys through two buffers.
constexpr int kKTAll = 320;

__device__ __forceinline__ void cp_async16(float *dst, const float *src, bool valid) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

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

// q, k: token-major [B][T][ldqk] (page stride bsqk), v, o: [B][T][ldvo]
// (page stride bsvo), head h at columns h*32 .. h*32+31 of each.
// Shared memory: Q [32][36] | kBufs K/V tiles [kKT][36] | scores [32][ldS],
// ldS a multiple of 4.  Rows of 36 floats keep the 16-byte loads of a quarter
// warp on distinct banks.  K and V tiles arrive by cp.async: with two buffers
// the next tile lands while the current one is used; with one (all keys in
// one tile) V lands while the softmax runs.
template <int kKT, int kBufs, int kBQ>
__global__ void __launch_bounds__(kBQ / 4 * 32, 2)
attn_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
            float *__restrict__ o, int T, int ldqk, long long bsqk, int ldvo, long long bsvo,
            float scale, int ldS) {
    pdl_begin();
    constexpr int kThreads = kBQ / 4 * 32;
    static_assert(kKT % 64 == 0, "the score loop walks 64-key slices of a tile");
    extern __shared__ float sm[];
    float *Qs = sm;                      // [kBQ][kLD]
    float *Tb = Qs + kBQ * kLD;          // [kBufs][kKT][kLD]
    float *Ss = Tb + kBufs * kKT * kLD;  // [kBQ][ldS]
    const int q0 = blockIdx.x * kBQ, h = blockIdx.y, b = blockIdx.z;
    const int t = threadIdx.x, lane = t & 31, wq = t >> 5;  // wq: query group of 4
    const long long base_qk = (long long)b * bsqk + h * kHeadDim;
    const long long base_vo = (long long)b * bsvo + h * kHeadDim;

    for (int i = t; i < kBQ * kHeadDim; i += kThreads) {
        const int r = i >> 5, d = i & 31;
        Qs[r * kLD + d] = q0 + r < T ? q[base_qk + (long long)(q0 + r) * ldqk + d] : 0.0f;
    }
    // tile j of K or V into buffer j % kBufs; rows past T are zero-filled
    auto load_tile = [&](const float *src, int j, int ld, long long base) {
        float *dst = Tb + (j % kBufs) * kKT * kLD;
        for (int i = t; i < kKT * kHeadDim / 4; i += kThreads) {
            const int r = i >> 3, c4 = i & 7, row = j * kKT + r;
            const bool ok = row < T;
            cp_async16(dst + r * kLD + 4 * c4, ok ? src + base + (long long)row * ld + 4 * c4 : src,
                       ok);
        }
        cp_async_commit();
    };
    const int nt = (T + kKT - 1) / kKT;
    // ---- scores: thread -> queries 4wq..4wq+3
    load_tile(k, 0, ldqk, base_qk);
    for (int jt = 0; jt < nt; jt++) {
        const int j0 = jt * kKT;
        if (kBufs > 1 && jt + 1 < nt) {
            load_tile(k, jt + 1, ldqk, base_qk);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        // 64-key slices of the tile: keys lane and lane + 32 of each
        for (int s0 = 0; s0 < kKT && j0 + s0 < T; s0 += 64) {
            const float *Ts = Tb + (jt % kBufs) * kKT * kLD + s0 * kLD;
            float acc[4][2];
#pragma unroll
            for (int r = 0; r < 4; r++) acc[r][0] = acc[r][1] = 0.0f;
#pragma unroll 2
            for (int d4 = 0; d4 < kHeadDim / 4; d4++) {
                const float4 k0 = *reinterpret_cast<const float4 *>(Ts + lane * kLD + 4 * d4);
                const float4 k1 = *reinterpret_cast<const float4 *>(Ts + (lane + 32) * kLD + 4 * d4);
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    const float4 qv =
                        *reinterpret_cast<const float4 *>(Qs + (wq * 4 + r) * kLD + 4 * d4);
                    acc[r][0] = fmaf(qv.x, k0.x, acc[r][0]);
                    acc[r][0] = fmaf(qv.y, k0.y, acc[r][0]);
                    acc[r][0] = fmaf(qv.z, k0.z, acc[r][0]);
                    acc[r][0] = fmaf(qv.w, k0.w, acc[r][0]);
                    acc[r][1] = fmaf(qv.x, k1.x, acc[r][1]);
                    acc[r][1] = fmaf(qv.y, k1.y, acc[r][1]);
                    acc[r][1] = fmaf(qv.z, k1.z, acc[r][1]);
                    acc[r][1] = fmaf(qv.w, k1.w, acc[r][1]);
                }
            }
#pragma unroll
            for (int r = 0; r < 4; r++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int j = j0 + s0 + lane + 32 * c;
                    if (j < T) Ss[(wq * 4 + r) * ldS + j] = __fmul_rn(acc[r][c], scale);
                }
        }
        __syncthreads();  // the buffer is refilled (kBufs tiles later)
        if (kBufs == 1 && jt + 1 < nt) load_tile(k, jt + 1, ldqk, base_qk);
    }
    load_tile(v, 0, ldvo, base_vo);  // lands during the softmax
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
    for (int jt = 0; jt < nt; jt++) {
        const int j0 = jt * kKT;
        if (kBufs > 1 && jt + 1 < nt) {
            load_tile(v, jt + 1, ldvo, base_vo);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *Ts = Tb + (jt % kBufs) * kKT * kLD;
        const int jn = T - j0 < kKT ? T - j0 : kKT;
        int jj = 0;
        for (; jj + 4 <= jn; jj += 4) {
            const float v0 = Ts[jj * kLD + lane], v1 = Ts[(jj + 1) * kLD + lane];
            const float v2 = Ts[(jj + 2) * kLD + lane], v3 = Ts[(jj + 3) * kLD + lane];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const float4 p = *reinterpret_cast<const float4 *>(Ss + (wq * 4 + r) * ldS + j0 + jj);
                acc[r] = fmaf(p.x, v0, acc[r]);
                acc[r] = fmaf(p.y, v1, acc[r]);
                acc[r] = fmaf(p.z, v2, acc[r]);
                acc[r] = fmaf(p.w, v3, acc[r]);
            }
        }
        for (; jj < jn; jj++) {
            const float vv = Ts[jj * kLD + lane];
#pragma unroll
            for (int r = 0; r < 4; r++) acc[r] = fmaf(Ss[(wq * 4 + r) * ldS + j0 + jj], vv, acc[r]);
        }
        __syncthreads();
        if (kBufs == 1 && jt + 1 < nt) load_tile(v, jt + 1, ldvo, base_vo);
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int i = q0 + wq * 4 + r;
        if (i < T) o[base_vo + (long long)i * ldvo + lane] = acc[r];
    }
}

int attention_lds(int T) { return (T + 3) / 4 * 4; }
size_t attention_smem_bytes(int T) {
    const size_t tiles = T <= kKTAll ? (size_t)kKTAll : 2 * 64;
    const size_t bq = T <= kKTAll ? kBQAll : kBQStream;
    return sizeof(float) * (bq * kLD + tiles * kLD + bq * attention_lds(T));
}

}  // namespace

Status launch_attention(const float *q, const float *k, const float *v, float *o, int T, int heads,
                        int ldqk, long long bsqk, int ldvo, long long bsvo, float scale, int B,
                        cudaStream_t st) {
    if (T <= 0 || heads <= 0 || heads > 65535 || B <= 0 || B > 65535 ||
        ldqk < heads * kHeadDim || ldvo < heads * kHeadDim)
        return ERR_SHAPE;
    // 16-byte rows for the cp.async tiles of k and v
    if ((((uintptr_t)k | (uintptr_t)v) & 15) || ldqk % 4 || ldvo % 4 || bsqk % 4 || bsvo % 4)
        return ERR_SHAPE;
    const size_t smem = attention_smem_bytes(T);
    if (smem > 227 * 1024) return ERR_SHAPE;
    if (!smem_attr_once((const void *)attn_kernel<kKTAll, 1, kBQAll>, 227 * 1024) ||
        !smem_attr_once((const void *)attn_kernel<64, 2, kBQStream>, 227 * 1024))
        return ERR_CUDA;
    const int ldS = attention_lds(T);
    if (T <= kKTAll)
        pdl_launch(attn_kernel<kKTAll, 1, kBQAll>, dim3((T + kBQAll - 1) / kBQAll, heads, B),
                   kBQAll / 4 * 32, smem, st, q, k, v, o, T, ldqk, bsqk, ldvo, bsvo, scale, ldS);
    else
        pdl_launch(attn_kernel<64, 2, kBQStream>,
                   dim3((T + kBQStream - 1) / kBQStream, heads, B), kBQStream / 4 * 32, smem, st,
                   q, k, v, o, T, ldqk, bsqk, ldvo, bsvo, scale, ldS);
    return cuda_status();
}

}  // namespace ppdl
