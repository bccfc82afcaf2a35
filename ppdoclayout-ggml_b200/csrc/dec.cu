// dec.cu — row-wise and small kernels of the encoder/decoder and the GPU
// postprocess.
//
// LayerNorm (ggml_norm eps 1e-5 * w + b, src/ppdoclayout.cpp:550-554),
// softmax rows (ggml_soft_max, :580), the box-refinement update
// sigmoid(delta + inverse_sigmoid(ref)) (:589-594, :849-850), the masked
// memory (:798) and the top-k row gather (:808), plus the reference's host
// postprocess (:927-993) moved to the device so only the final dets and
// masks cross PCIe.
#include "common.cuh"
#include "dec.h"
#include "select.cuh"

namespace ppdl {

namespace {

inline int blocks(long long n, int t = 256) { return (int)((n + t - 1) / t); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// one warp per 256-wide row; y = LN(x (+ r)) * g + b, and y2 = y + q when q
// is given (the decoder's x1 and x1 + query_pos in one pass)
__global__ void layernorm256_kernel(const float *__restrict__ x, const float *__restrict__ r,
                                    const float *__restrict__ g, const float *__restrict__ bta,
                                    float *__restrict__ y, const float *__restrict__ q,
                                    float *__restrict__ y2, long long rows) {
    pdl_begin();
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int lane = threadIdx.x & 31;
    const float4 *xp = reinterpret_cast<const float4 *>(x + row * 256);
    float4 v[2];
    v[0] = xp[lane];
    v[1] = xp[lane + 32];
    if (r) {
        const float4 *rp = reinterpret_cast<const float4 *>(r + row * 256);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const float4 q = rp[lane + 32 * k];
            v[k].x = __fadd_rn(v[k].x, q.x); v[k].y = __fadd_rn(v[k].y, q.y);
            v[k].z = __fadd_rn(v[k].z, q.z); v[k].w = __fadd_rn(v[k].w, q.w);
        }
    }
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 2; k++) s += v[k].x + v[k].y + v[k].z + v[k].w;
    const float mean = warp_sum(s) * (1.0f / 256.0f);
    float s2 = 0.f;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        v[k].x -= mean; v[k].y -= mean; v[k].z -= mean; v[k].w -= mean;
        s2 += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
    }
    const float var = warp_sum(s2) * (1.0f / 256.0f);
    const float sc = 1.0f / sqrtf(var + 1e-5f);
    const float4 *gp = reinterpret_cast<const float4 *>(g);
    const float4 *bp = reinterpret_cast<const float4 *>(bta);
    float4 *yp = reinterpret_cast<float4 *>(y + row * 256);
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const float4 gg = gp[lane + 32 * k], bb = bp[lane + 32 * k];
        float4 o;
        o.x = v[k].x * sc * gg.x + bb.x; o.y = v[k].y * sc * gg.y + bb.y;
        o.z = v[k].z * sc * gg.z + bb.z; o.w = v[k].w * sc * gg.w + bb.w;
        yp[lane + 32 * k] = o;
        if (q) {
            const float4 qq = reinterpret_cast<const float4 *>(q + row * 256)[lane + 32 * k];
            reinterpret_cast<float4 *>(y2 + row * 256)[lane + 32 * k] =
                make_float4(__fadd_rn(o.x, qq.x), __fadd_rn(o.y, qq.y), __fadd_rn(o.z, qq.z),
                            __fadd_rn(o.w, qq.w));
        }
    }
}

// one warp per row of length L, in place
__global__ void softmax_rows_kernel(float *__restrict__ x, long long rows, int L) {
    pdl_begin();
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int lane = threadIdx.x & 31;
    float *p = x + row * L;
    float m = -INFINITY;
    for (int i = lane; i < L; i += 32) m = fmaxf(m, p[i]);
    m = warp_max(m);
    float s = 0.f;
    for (int i = lane; i < L; i += 32) {
        const float e = expf(p[i] - m);
        p[i] = e;
        s += e;
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    for (int i = lane; i < L; i += 32) p[i] *= inv;
}

__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b,
                           float *__restrict__ y, long long n) {
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(a[i], b[i]);
}

// y[i] = a[i] + b[i % nb]: b shared by every page (nb elements per page)
__global__ void add_bcast_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                 float *__restrict__ y, long long n, long long nb) {
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fadd_rn(a[i], b[i % nb]);
}

__global__ void sigmoid_kernel(const float *__restrict__ x, float *__restrict__ y, long long n) {
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x[i])));
}

// The decoder layer's box update and the next layer's query-position input
// in one launch, one warp per query row (src/ppdoclayout.cpp:848-850 and
// :827):
//   delta = h W^T + b            (bbox_head.2: 256 -> 4)
//   ref   = sigmoid(delta + inverse_sigmoid(ref))  (inverse_sigmoid with
//                                 the clamps of src/ppdoclayout.cpp:589-594)
//   qp    = relu(ref Wq^T + bq)  (qpos.0: 4 -> nq of the next layer; qp may
//                                 be null after the last layer)
// Each lane sums eight consecutive k of the four dot products with fmaf,
// then the warp adds the lanes' partials pairwise.
__global__ void box_refine_kernel(const float *__restrict__ h, const float *__restrict__ w,
                                  const float *__restrict__ b, float *__restrict__ ref,
                                  const float *__restrict__ wq, const float *__restrict__ bq,
                                  float *__restrict__ qp, int rows, int nqp) {
    pdl_begin();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int lane = threadIdx.x & 31;
    const float4 *hp = reinterpret_cast<const float4 *>(h + (long long)row * 256 + lane * 8);
    const float4 h0 = hp[0], h1 = hp[1];
    const float hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    float d[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float4 *wp = reinterpret_cast<const float4 *>(w + j * 256 + lane * 8);
        const float4 w0 = wp[0], w1 = wp[1];
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) acc = fmaf(hv[k], wv[k], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        d[j] = __fadd_rn(acc, b[j]);
    }
    float r[4];
    const float4 r4 = *reinterpret_cast<const float4 *>(ref + (long long)row * 4);
    const float rin[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float x = fminf(fmaxf(rin[j], 0.0f), 1.0f);
        const float x1 = fminf(fmaxf(x, 1e-5f), 1.0f);
        const float x2 = fminf(fmaxf(__fsub_rn(1.0f, x), 1e-5f), 1.0f);
        const float z = __fadd_rn(d[j], __fsub_rn(logf(x1), logf(x2)));
        r[j] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
    }
    __syncwarp();
    if (lane == 0)
        *reinterpret_cast<float4 *>(ref + (long long)row * 4) = make_float4(r[0], r[1], r[2], r[3]);
    if (!qp) return;
    float *q = qp + (long long)row * nqp;
    for (int o = lane; o < nqp; o += 32) {
        const float4 wv = *reinterpret_cast<const float4 *>(wq + o * 4);
        float acc = 0.0f;
        acc = fmaf(r[0], wv.x, acc);
        acc = fmaf(r[1], wv.y, acc);
        acc = fmaf(r[2], wv.z, acc);
        acc = fmaf(r[3], wv.w, acc);
        q[o] = fmaxf(__fadd_rn(acc, bq[o]), 0.0f);
    }
}

// y[b][t][:] = x[b][t][:] * v[t]; four elements per thread (D % 4 == 0),
// 32-bit index arithmetic (n / 4 < 2^31)
__global__ void row_scale_kernel(const float4 *__restrict__ x, const float *__restrict__ v,
                                 float4 *__restrict__ y, unsigned rows_per_page, unsigned d4,
                                 unsigned n4) {
    pdl_begin();
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const float s = v[(i / d4) % rows_per_page];
    const float4 a = x[i];
    y[i] = make_float4(__fmul_rn(a.x, s), __fmul_rn(a.y, s), __fmul_rn(a.z, s), __fmul_rn(a.w, s));
}

// y[b][i][:] = x[b][idx[b][i]][:]
__global__ void gather_rows_kernel(const float *__restrict__ x, const int32_t *__restrict__ idx,
                                   float *__restrict__ y, int rows_in, int rows_out, int D, int B) {
    pdl_begin();
    const long long n = (long long)B * rows_out * D;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int d = (int)(i % D);
    const long long r = i / D;
    const int b = (int)(r / rows_out);
    const int src = idx[r];
    y[i] = x[((long long)b * rows_in + src) * D + d];
}

// ---- postprocess ---------------------------------------------------------------
// votes[j] = sum_{i != j} sigmoid(order[j + 300 i] - order[i + 300 j]) in i
// order (src/ppdoclayout.cpp:935-945).  A block takes 16 consecutive j of a
// page: it stages the 16 rows order[j][*] and the 16 columns order[*][j]
// in shared memory with coalesced loads, all 256 threads evaluate the
// sigmoid terms, and one thread per j adds its 300 terms in i order (the
// reference's order: the sums are bit-identical).  The ranks follow in
// pp_select_kernel.
constexpr int kVoteJ = 16;
__global__ void __launch_bounds__(256)
pp_votes_kernel(const float *__restrict__ order, float *__restrict__ votes) {
    pdl_begin();
    __shared__ float s_row[kVoteJ][kNQ + 1];  // order[j0 + jj][i]
    __shared__ float s_col[kNQ][kVoteJ + 1];  // order[i][j0 + jj], then the terms
    const int b = blockIdx.y, j0 = blockIdx.x * kVoteJ;
    const int nj = min(kVoteJ, kNQ - j0);
    const float *o = order + (long long)b * kNQ * kNQ;
    for (int e = threadIdx.x; e < kVoteJ * kNQ; e += blockDim.x) {
        const int jj = e / kNQ, i = e - jj * kNQ;
        s_row[jj][i] = jj < nj ? o[(j0 + jj) * kNQ + i] : 0.0f;
    }
    for (int e = threadIdx.x; e < kNQ * kVoteJ; e += blockDim.x) {
        const int i = e / kVoteJ, jj = e - i * kVoteJ;
        s_col[i][jj] = jj < nj ? o[i * kNQ + j0 + jj] : 0.0f;
    }
    __syncthreads();
    // term(i, j) = sigmoid(order[j + 300 i] - order[i + 300 j]); the
    // diagonal adds an exact +0 (the sum starts at +0 and only grows)
    for (int e = threadIdx.x; e < kNQ * kVoteJ; e += blockDim.x) {
        const int i = e / kVoteJ, jj = e - i * kVoteJ;
        const float diff = __fsub_rn(s_col[i][jj], s_row[jj][i]);
        const float term = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-diff)));
        s_col[i][jj] = (i == j0 + jj) ? 0.0f : term;
    }
    __syncthreads();
    if (threadIdx.x < nj) {
        float acc = 0.0f;
        for (int i = 0; i < kNQ; i++) acc = __fadd_rn(acc, s_col[i][threadIdx.x]);
        votes[b * kNQ + j0 + threadIdx.x] = acc;
    }
}

// top-300 of the 7500 sigmoid scores (ties to the lower flat index) and the
// detections rows; one block per page, block radix select (select.cuh)
__global__ void __launch_bounds__(1024)
pp_select_kernel(const float *__restrict__ logits, const float *__restrict__ boxes,
                 const float *__restrict__ votes, const int32_t *__restrict__ ori_hw,
                 float *__restrict__ dets, int32_t *__restrict__ sel) {
    pdl_begin();
    constexpr int N = kNQ * kNC;
    extern __shared__ unsigned long long s_key[];  // N keys (dynamic)
    __shared__ unsigned long long s_top[kSelectMax];
    __shared__ float s_votes[kNQ];
    __shared__ int s_rank[kNQ];
    const int b = blockIdx.x;
    const float *lg = logits + (long long)b * N;
    for (int i = threadIdx.x; i < N; i += blockDim.x)
        s_key[i] = select_key(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-lg[i]))), (unsigned)i);
    for (int j = threadIdx.x; j < kNQ; j += blockDim.x) s_votes[j] = votes[b * kNQ + j];
    __syncthreads();
    // reading order: rank = position in the stable ascending sort of the votes
    for (int j = threadIdx.x; j < kNQ; j += blockDim.x) {
        const float vj = s_votes[j];
        int r = 0;
        for (int k = 0; k < kNQ; k++) {
            const float vk = s_votes[k];
            r += (vk < vj) || (vk == vj && k < j);
        }
        s_rank[j] = r;
    }
    __syncthreads();
    block_select_top(s_key, N, kNQ, s_top);
    const float sf_h = __fdiv_rn((float)kImg, (float)ori_hw[2 * b]);
    const float sf_w = __fdiv_rn((float)kImg, (float)ori_hw[2 * b + 1]);
    const float oh = floorf(__fadd_rn(__fdiv_rn((float)kImg, sf_h), 0.5f));
    const float ow = floorf(__fadd_rn(__fdiv_rn((float)kImg, sf_w), 0.5f));
    for (int r = threadIdx.x; r < kNQ; r += blockDim.x) {
        const int flat = (int)select_index(s_top[r]);
        const int q = flat / kNC, c = flat - q * kNC;
        const float *bx = boxes + ((long long)b * kNQ + q) * 4;
        float *o = dets + ((long long)b * kNQ + r) * 7;
        o[0] = (float)c;
        o[1] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-lg[flat])));
        o[2] = __fmul_rn(__fsub_rn(bx[0], __fmul_rn(bx[2], 0.5f)), ow);
        o[3] = __fmul_rn(__fsub_rn(bx[1], __fmul_rn(bx[3], 0.5f)), oh);
        o[4] = __fmul_rn(__fadd_rn(bx[0], __fmul_rn(bx[2], 0.5f)), ow);
        o[5] = __fmul_rn(__fadd_rn(bx[1], __fmul_rn(bx[3], 0.5f)), oh);
        o[6] = (float)s_rank[q];
        sel[b * kNQ + r] = flat;
    }
}

// masks[b][r][p] = mask_logits[b][sel/25][p] > 0
__global__ void pp_masks_kernel(const float *__restrict__ ml, const int32_t *__restrict__ sel,
                                int32_t *__restrict__ out) {
    pdl_begin();
    const int r = blockIdx.y, b = blockIdx.z;
    const int q = sel[b * kNQ + r] / kNC;
    const float4 *src = reinterpret_cast<const float4 *>(ml + ((long long)b * kNQ + q) * kMaskPix);
    int4 *dst = reinterpret_cast<int4 *>(out + ((long long)b * kNQ + r) * kMaskPix);
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= kMaskPix / 4) return;
    const float4 v = __ldg(src + i);
    dst[i] = make_int4(v.x > 0.0f, v.y > 0.0f, v.z > 0.0f, v.w > 0.0f);
}

// Packed masks: word w of detection row r holds pixels 32w .. 32w + 31 of
// the thresholded mask of the query selected for that row (bit i = pixel
// 32w + i, logit > 0 — the reference's threshold, src/ppdoclayout.cpp:985-990).
// A warp owns 8 consecutive words: each lane issues its 8 loads (one per
// word, lanes on consecutive pixels: eight 128-byte lines in flight per
// warp) before the 8 ballots.
constexpr int kBitsWordsPerWarp = 8;
__global__ void pp_mask_bits_kernel(const float *__restrict__ ml, const int32_t *__restrict__ sel,
                                    uint32_t *__restrict__ bits) {
    pdl_begin();
    const int r = blockIdx.y, b = blockIdx.z;
    const int q = sel ? sel[b * kNQ + r] / kNC : r;  // no sel: row r is query r
    const float *src = ml + ((long long)b * kNQ + q) * kMaskPix;
    uint32_t *dst = bits + ((long long)b * kNQ + r) * kMaskWords;
    const int lane = threadIdx.x & 31;
    const int w0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kBitsWordsPerWarp;
    float v[kBitsWordsPerWarp];
#pragma unroll
    for (int j = 0; j < kBitsWordsPerWarp; j++)
        v[j] = w0 + j < kMaskWords ? __ldg(src + (w0 + j) * 32 + lane) : 0.0f;
    uint32_t mine = 0;
#pragma unroll
    for (int j = 0; j < kBitsWordsPerWarp; j++) {
        const uint32_t word = __ballot_sync(0xffffffffu, v[j] > 0.0f);
        if (lane == j) mine = word;
    }
    if (lane < kBitsWordsPerWarp && w0 + lane < kMaskWords) dst[w0 + lane] = mine;
}

// Packed masks of the detection rows from the packed masks of the queries:
// row r of page b is query sel[b][r] / 25's 1250 words (16-byte copies).
__global__ void pp_gather_bits_kernel(const uint32_t *__restrict__ qbits,
                                      const int32_t *__restrict__ sel,
                                      uint32_t *__restrict__ bits) {
    pdl_begin();
    const int r = blockIdx.y, b = blockIdx.z;
    const int q = sel[b * kNQ + r] / kNC;
    const uint32_t *src = qbits + ((long long)b * kNQ + q) * kMaskWords;
    uint32_t *dst = bits + ((long long)b * kNQ + r) * kMaskWords;
    for (int i = threadIdx.x; i < kMaskWords / 2; i += blockDim.x) {
        // 1250 words = 625 8-byte pairs; rows start 5000 bytes apart (8-byte aligned)
        reinterpret_cast<uint2 *>(dst)[i] = __ldg(reinterpret_cast<const uint2 *>(src) + i);
    }
}

// int32 masks (the reference's result format) from packed masks: each
// thread expands one word into 32 ints (eight 16-byte stores).
__global__ void unpack_mask_bits_kernel(const uint32_t *__restrict__ bits,
                                        int32_t *__restrict__ masks, long long words) {
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= words) return;
    const uint32_t w = __ldg(bits + i);
    int4 *dst = reinterpret_cast<int4 *>(masks + i * 32);
#pragma unroll
    for (int j = 0; j < 8; j++)
        dst[j] = make_int4((w >> (4 * j)) & 1, (w >> (4 * j + 1)) & 1, (w >> (4 * j + 2)) & 1,
                           (w >> (4 * j + 3)) & 1);
}

}  // namespace

Status launch_pack_mask_bits(const float *ml, uint32_t *bits, int B, cudaStream_t st) {
    if (B <= 0 || B > 65535) return ERR_SHAPE;
    dim3 grid((unsigned)cdiv(kMaskWords, 8 * kBitsWordsPerWarp), kNQ, (unsigned)B);
    pdl_launch(pp_mask_bits_kernel, grid, 256, 0, st, ml, nullptr, bits);
    return cuda_status();
}

Status launch_unpack_mask_bits(const uint32_t *bits, int32_t *masks, long long rows,
                               cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? OK : ERR_SHAPE;
    const long long words = rows * kMaskWords;
    pdl_launch(unpack_mask_bits_kernel, blocks(words), 256, 0, st, bits, masks, words);
    return cuda_status();
}

Status launch_layernorm256(const float *x, const float *r, const float *g, const float *b,
                           float *y, long long rows, cudaStream_t st) {
    return launch_layernorm256_add(x, r, g, b, y, nullptr, nullptr, rows, st);
}

Status launch_layernorm256_add(const float *x, const float *r, const float *g, const float *b,
                               float *y, const float *q, float *y2, long long rows,
                               cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? OK : ERR_SHAPE;
    if (q && !y2) return ERR_SHAPE;
    pdl_launch(layernorm256_kernel, blocks(rows * 32), 256, 0, st, x, r, g, b, y, q, y2, rows);
    return cuda_status();
}

Status launch_softmax_rows(float *x, long long rows, int L, cudaStream_t st) {
    pdl_launch(softmax_rows_kernel, blocks(rows * 32), 256, 0, st, x, rows, L);
    return cuda_status();
}

Status launch_add(const float *a, const float *b, float *y, long long n, cudaStream_t st) {
    pdl_launch(add_kernel, blocks(n), 256, 0, st, a, b, y, n);
    return cuda_status();
}

Status launch_add_bcast(const float *a, const float *b, float *y, long long n_per_page,
                        int pages, cudaStream_t st) {
    if (n_per_page <= 0 || pages <= 0) return ERR_SHAPE;
    const long long n = n_per_page * pages;
    pdl_launch(add_bcast_kernel, blocks(n), 256, 0, st, a, b, y, n, n_per_page);
    return cuda_status();
}

Status launch_sigmoid(const float *x, float *y, long long n, cudaStream_t st) {
    pdl_launch(sigmoid_kernel, blocks(n), 256, 0, st, x, y, n);
    return cuda_status();
}

Status launch_box_refine(const float *h, const float *w, const float *b, float *ref,
                         const float *wq, const float *bq, float *qp, int rows, int nqp,
                         cudaStream_t st) {
    if (rows <= 0 || (qp && nqp <= 0) ||
        (((uintptr_t)h | (uintptr_t)w | (uintptr_t)ref | (uintptr_t)wq) & 15))
        return ERR_SHAPE;
    pdl_launch(box_refine_kernel, cdiv(rows, 8), 256, 0, st, h, w, b, ref, wq, bq, qp, rows, nqp);
    return cuda_status();
}

Status launch_row_scale(const float *x, const float *v, float *y, long long rows_per_page, int D,
                        int B, cudaStream_t st) {
    const long long n = (long long)B * rows_per_page * D;
    if (D % 4 || n / 4 >= (1LL << 31) || ((uintptr_t)x & 15) || ((uintptr_t)y & 15))
        return ERR_SHAPE;
    pdl_launch(row_scale_kernel, blocks(n / 4), 256, 0, st, reinterpret_cast<const float4 *>(x), v,
               reinterpret_cast<float4 *>(y), (unsigned)rows_per_page, (unsigned)(D / 4),
               (unsigned)(n / 4));
    return cuda_status();
}

Status launch_gather_rows(const float *x, const int32_t *idx, float *y, int rows_in, int rows_out,
                          int D, int B, cudaStream_t st) {
    const long long n = (long long)B * rows_out * D;
    pdl_launch(gather_rows_kernel, blocks(n), 256, 0, st, x, idx, y, rows_in, rows_out, D, B);
    return cuda_status();
}

Status launch_postprocess(const float *logits, const float *boxes, const float *order,
                          const float *mask_logits, const uint32_t *mask_bits_q,
                          const int32_t *ori_hw, int32_t *rank, float *dets, int32_t *sel,
                          int32_t *masks, uint32_t *mask_bits, int B, cudaStream_t st) {
    const int smem = kNQ * kNC * (int)sizeof(unsigned long long);
    if (!smem_attr_once((const void *)pp_select_kernel, smem)) return ERR_CUDA;
    float *votes = reinterpret_cast<float *>(rank);  // the 300 votes of each page
    pdl_launch(pp_votes_kernel, dim3(cdiv(kNQ, kVoteJ), B), 256, 0, st, order, votes);
    pdl_launch(pp_select_kernel, B, 1024, smem, st, logits, boxes, votes, ori_hw, dets, sel);
    if (masks) {
        dim3 grid((unsigned)cdiv(kMaskPix / 4, 256), kNQ, (unsigned)B);
        pdl_launch(pp_masks_kernel, grid, 256, 0, st, mask_logits, sel, masks);
    }
    if (mask_bits && mask_bits_q) {
        pdl_launch(pp_gather_bits_kernel, dim3(1, kNQ, (unsigned)B), 128, 0, st, mask_bits_q, sel,
                   mask_bits);
    } else if (mask_bits && mask_logits) {
        // 1250 words per row: blocks of 8 warps x 8 words
        dim3 grid((unsigned)cdiv(kMaskWords, 8 * kBitsWordsPerWarp), kNQ, (unsigned)B);
        pdl_launch(pp_mask_bits_kernel, grid, 256, 0, st, mask_logits, sel, mask_bits);
    }
    return cuda_status();
}

}  // namespace ppdl
