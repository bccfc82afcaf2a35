// maskbox.cu — mask -> box (op 1).
//
// Reference: op_mask_box (src/ppdoclayout.cpp:98-140) and
// ppdl_mask_box_kernel (patches/ggml-ppdl.patch:211-253).  Per query: the
// bounding box of the logit > 0 pixels of its 200x200 mask, as
// [xmin, ymin, xmax+1, ymax+1] / 200 -> cxcywh -> inverse sigmoid with the
// clamp / 1e-5 guards; an empty mask gives the zero box.
//
// B200 design: a streaming reduction over 160 KB per query (48 MB per page),
// so the kernel is HBM-bound: one block per query, 16-byte streaming loads
// (a float4 never straddles a 200-pixel row), per-thread integer extents,
// warp min/max reductions (redux.sync) and one shared-memory combine — no
// per-pixel shared-memory atomics.  The final arithmetic follows the CPU op
// (division by 200, then cxcywh, then logf), so the result is bit-identical
// to the reference CPU op whenever logf agrees.
#include <climits>

#include "common.cuh"
#include "kernels.h"

namespace ppdl {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float invsig(float x) {
    x = fminf(fmaxf(x, 0.0f), 1.0f);
    const float x1 = fmaxf(x, 1e-5f);
    const float x2 = fmaxf(__fsub_rn(1.0f, x), 1e-5f);
    return logf(__fdiv_rn(x1, x2));
}

// [xmin, ymin, xmax+1, ymax+1] / 200 -> cxcywh -> inverse sigmoid, in the
// CPU op's order (xmax < 0: empty mask, zero box)
__device__ __forceinline__ void write_box(int xmin, int ymin, int xmax, int ymax, float *o4) {
    float bx0, by0, bx1, by1;
    if (xmax < 0) {
        bx0 = by0 = bx1 = by1 = 0.0f;
    } else {
        bx0 = (float)xmin; by0 = (float)ymin;
        bx1 = __fadd_rn((float)xmax, 1.0f); by1 = __fadd_rn((float)ymax, 1.0f);
    }
    const float hw = (float)kMaskHW;
    bx0 = __fdiv_rn(bx0, hw); bx1 = __fdiv_rn(bx1, hw);
    by0 = __fdiv_rn(by0, hw); by1 = __fdiv_rn(by1, hw);
    const float cx = __fmul_rn(__fadd_rn(bx0, bx1), 0.5f);
    const float cy = __fmul_rn(__fadd_rn(by0, by1), 0.5f);
    const float bw = __fsub_rn(bx1, bx0), bh = __fsub_rn(by1, by0);
    float4 o;
    o.x = invsig(cx); o.y = invsig(cy); o.z = invsig(bw); o.w = invsig(bh);
    *reinterpret_cast<float4 *>(o4) = o;
}

__global__ void __launch_bounds__(kThreads)
mask_box_kernel(const float *__restrict__ ml, float *__restrict__ out) {
    pdl_begin();
    const int q = blockIdx.x;
    const float4 *m = reinterpret_cast<const float4 *>(ml + (size_t)q * kMaskPix);
    constexpr int kRowVec = kMaskHW / 4;  // 50 float4 per mask row
    int xmin = INT_MAX, ymin = INT_MAX, xmax = -1, ymax = -1;
    for (int i = threadIdx.x; i < kMaskPix / 4; i += kThreads) {
        const float4 v = __ldcs(m + i);
        const bool p0 = v.x > 0.0f, p1 = v.y > 0.0f, p2 = v.z > 0.0f, p3 = v.w > 0.0f;
        if (p0 | p1 | p2 | p3) {
            const int y = i / kRowVec;
            const int x = (i - y * kRowVec) * 4;
            const int xa = p0 ? x : (p1 ? x + 1 : (p2 ? x + 2 : x + 3));
            const int xb = p3 ? x + 3 : (p2 ? x + 2 : (p1 ? x + 1 : x));
            xmin = min(xmin, xa);
            xmax = max(xmax, xb);
            ymin = min(ymin, y);
            ymax = max(ymax, y);
        }
    }
    xmin = __reduce_min_sync(0xffffffffu, xmin);
    ymin = __reduce_min_sync(0xffffffffu, ymin);
    xmax = __reduce_max_sync(0xffffffffu, xmax);
    ymax = __reduce_max_sync(0xffffffffu, ymax);
    __shared__ int s_ext[kThreads / 32][4];
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        s_ext[warp][0] = xmin; s_ext[warp][1] = ymin;
        s_ext[warp][2] = xmax; s_ext[warp][3] = ymax;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < kThreads / 32; w++) {
        xmin = min(xmin, s_ext[w][0]); ymin = min(ymin, s_ext[w][1]);
        xmax = max(xmax, s_ext[w][2]); ymax = max(ymax, s_ext[w][3]);
    }
    write_box(xmin, ymin, xmax, ymax, out + (size_t)q * 4);
}

// The same op on packed masks (bit p & 31 of word p >> 5 = logit of pixel p
// > 0, the forward's own mask output): a word covers 32 consecutive pixels,
// at most two mask rows (200 = 6 x 32 + 8), each part's extent from its
// lowest and highest set bit.  Same pixels, same extents, same result.
__global__ void __launch_bounds__(kThreads)
mask_box_bits_kernel(const uint32_t *__restrict__ bits, float *__restrict__ out) {
    pdl_begin();
    const int q = blockIdx.x;
    const uint32_t *m = bits + (size_t)q * kMaskWords;
    int xmin = INT_MAX, ymin = INT_MAX, xmax = -1, ymax = -1;
    for (int w = threadIdx.x; w < kMaskWords; w += kThreads) {
        const uint32_t v = __ldg(m + w);
        if (!v) continue;
        const int p0 = w * 32, y0 = p0 / kMaskHW, x0 = p0 - y0 * kMaskHW;
        const int s = kMaskHW - x0;  // pixels of the word left in row y0
        const uint32_t a = s >= 32 ? v : v & ((1u << s) - 1u);
        if (a) {
            xmin = min(xmin, x0 + __ffs(a) - 1);
            xmax = max(xmax, x0 + 31 - __clz(a));
            ymin = min(ymin, y0);
            ymax = max(ymax, y0);
        }
        if (s < 32) {
            const uint32_t b = v >> s;  // pixels 0 .. 31 - s of row y0 + 1
            if (b) {
                xmin = min(xmin, __ffs(b) - 1);
                xmax = max(xmax, 31 - __clz(b));
                ymin = min(ymin, y0 + 1);
                ymax = max(ymax, y0 + 1);
            }
        }
    }
    xmin = __reduce_min_sync(0xffffffffu, xmin);
    ymin = __reduce_min_sync(0xffffffffu, ymin);
    xmax = __reduce_max_sync(0xffffffffu, xmax);
    ymax = __reduce_max_sync(0xffffffffu, ymax);
    __shared__ int s_ext[kThreads / 32][4];
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        s_ext[warp][0] = xmin; s_ext[warp][1] = ymin;
        s_ext[warp][2] = xmax; s_ext[warp][3] = ymax;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < kThreads / 32; w++) {
        xmin = min(xmin, s_ext[w][0]); ymin = min(ymin, s_ext[w][1]);
        xmax = max(xmax, s_ext[w][2]); ymax = max(ymax, s_ext[w][3]);
    }
    write_box(xmin, ymin, xmax, ymax, out + (size_t)q * 4);
}

}  // namespace

Status launch_mask_box_bits(const uint32_t *bits, float *out, int rows, cudaStream_t stream) {
    if (rows <= 0) return rows == 0 ? OK : ERR_SHAPE;
    if ((uintptr_t)out & 15) return ERR_SHAPE;
    pdl_launch(mask_box_bits_kernel, rows, kThreads, 0, stream, bits, out);
    return cuda_status();
}

Status launch_mask_box(const float *ml, float *out, int rows, cudaStream_t stream) {
    if (rows <= 0) return rows == 0 ? OK : ERR_SHAPE;
    if (((uintptr_t)ml | (uintptr_t)out) & 15) return ERR_SHAPE;
    pdl_launch(mask_box_kernel, rows, kThreads, 0, stream, ml, out);
    return cuda_status();
}

}  // namespace ppdl
