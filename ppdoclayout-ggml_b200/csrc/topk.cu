// topk.cu — top-300 query selection (op 13).
//
// Reference: op_topk300 (src/ppdoclayout.cpp:73-96) and ppdl_topk_kernel
// (patches/ggml-ppdl.patch:440-486): the nq tokens with the largest
// max-over-classes logit, descending, ties to the lower token index.
//
// B200 design: one block per page.  Each token becomes a 64-bit key
// (order-preserving bits of its max logit << 32 | ~index), so "descending
// key" is exactly the reference order including the tie rule; -0.0 is
// folded to +0.0 first because the reference compares values, under which
// the two zeros tie.  The keys are unique; the nq largest come from the
// block radix select of select.cuh (the logits reach the keys through
// shared memory, 512 tokens at a time).  Larger nq fall back to a bitonic
// sort of all keys.
#include "common.cuh"
#include "kernels.h"
#include "select.cuh"

namespace ppdl {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxKeys = 16384;

__global__ void __launch_bounds__(kThreads)
topk_kernel(const float *__restrict__ lg, int32_t *__restrict__ out, int ntok, int nc, int nq,
            int n2) {
    pdl_begin();
    extern __shared__ unsigned long long s_key[];
    const float *lb = lg + (size_t)blockIdx.x * ntok * nc;
    for (int q = threadIdx.x; q < n2; q += kThreads) {
        unsigned long long key = 0ull;
        if (q < ntok) {
            const float *p = lb + (size_t)q * nc;
            float m = p[0];
            for (int c = 1; c < nc; c++) m = (m < p[c]) ? p[c] : m;  // std::max
            if (m == 0.0f) m = 0.0f;                                 // -0 ties +0
            unsigned u = __float_as_uint(m);
            u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            key = ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)q);
        }
        s_key[q] = key;
    }
    __syncthreads();
    // bitonic sort, descending
    for (int k = 2; k <= n2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n2; i += kThreads) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = s_key[i], b = s_key[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        s_key[i] = b;
                        s_key[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int r = threadIdx.x; r < nq; r += kThreads)
        out[(size_t)blockIdx.x * nq + r] =
            (int32_t)(0xFFFFFFFFu - (unsigned)(s_key[r] & 0xFFFFFFFFull));
}

constexpr size_t kSelSmemMax = 200 * 1024;  // its dynamic shared memory: keys + staged logits

// key of token q: its max logit over the classes, in the reference's order
// (the first of equal values kept: std::max), and its index
__device__ __forceinline__ unsigned long long topk_key(const float *p, int nc, int q) {
    float m = p[0];
    for (int c = 1; c < nc; c++) m = (m < p[c]) ? p[c] : m;  // std::max
    return select_key(m, (unsigned)q);
}

constexpr int kChunk = 512;  // tokens whose logits are staged in shared memory at a time

__global__ void __launch_bounds__(kThreads)
topk_select_kernel(const float *__restrict__ lg, int32_t *__restrict__ out, int ntok, int nc,
                   int nq) {
    pdl_begin();
    extern __shared__ unsigned long long s_key[];  // ntok keys, then kChunk x nc logits
    float *s_lg = reinterpret_cast<float *>(s_key + ntok);
    __shared__ unsigned long long s_sel[kSelectMax];
    const float *lb = lg + (size_t)blockIdx.x * ntok * nc;
    // keys: the page's logits pass through shared memory in chunks of tokens
    // (asynchronous coalesced 4-byte copies, all in flight together), then a
    // thread takes the max over its token's classes
    const uint32_t s_lg_addr = (uint32_t)__cvta_generic_to_shared(s_lg);
    for (int t0 = 0; t0 < ntok; t0 += kChunk) {
        const int n = (ntok - t0 < kChunk ? ntok - t0 : kChunk) * nc;
        const float *src = lb + (size_t)t0 * nc;
        for (int i = threadIdx.x; i < n; i += kThreads)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s_lg_addr + 4u * i),
                         "l"(src + i)
                         : "memory");
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
        __syncthreads();
        const int q = t0 + threadIdx.x;
        if (threadIdx.x < kChunk && q < ntok) s_key[q] = topk_key(s_lg + threadIdx.x * nc, nc, q);
        __syncthreads();
    }
    block_select_top(s_key, ntok, nq, s_sel);
    for (int r = threadIdx.x; r < nq; r += kThreads)
        out[(size_t)blockIdx.x * nq + r] = (int32_t)select_index(s_sel[r]);
}

}  // namespace

Status launch_topk(const float *lg, int32_t *out, int ntok, int nc, int nq, int batch,
                   cudaStream_t stream) {
    if (ntok <= 0 || nc <= 0 || nq <= 0 || batch <= 0) return ERR_SHAPE;
    if (ntok > kMaxKeys || nq > ntok) return ERR_SHAPE;
    int n2 = 1;
    while (n2 < ntok) n2 <<= 1;
    if (n2 < 2) n2 = 2;
    const size_t smem = (size_t)n2 * sizeof(unsigned long long);
    if (!smem_attr_once((const void *)topk_kernel, kMaxKeys * (int)sizeof(unsigned long long)) ||
        !smem_attr_once((const void *)topk_select_kernel, (int)kSelSmemMax))
        return ERR_CUDA;
    const size_t sel_smem = (size_t)ntok * sizeof(unsigned long long) + (size_t)kChunk * nc * 4;
    if (nq <= kSelectMax && sel_smem <= kSelSmemMax)
        pdl_launch(topk_select_kernel, batch, kThreads, sel_smem, stream, lg, out, ntok, nc, nq);
    else
        pdl_launch(topk_kernel, batch, kThreads, smem, stream, lg, out, ntok, nc, nq, n2);
    return cuda_status();
}

}  // namespace ppdl
