// msda.cu — multi-scale deformable attention sampling core (MSDeformAttn).
//
// Reference: op_msdeform (src/ppdoclayout.cpp:142-198) and
// ppdl_msdeform_kernel (patches/ggml-ppdl.patch:255-312).  For every page b,
// query q and head h: softmax over the 12 (level, point) logits, sampling
// location ref.xy + off/4 * ref.wh * 0.5, bilinear grid_sample (zeros
// padding, align_corners=false) on level l of the value map, and the
// weighted sum of 32 head channels over the 48 (point, corner) taps.
//
// B200 design: the op is a memory-bound gather of 128-byte value rows
// (32 f32 of one head at one token).  A block takes 16 (query, head) pairs:
//   phase 1  the softmax (one thread per pair) and the 48 taps of every pair
//            (one thread per sampling point) go to shared memory as
//            (token row or -1, tap weight) — the per-tap index math is done
//            once instead of once per channel lane;
//   phase 2  eight lanes own one pair, each lane one float4 of the head's
//            32 channels, so one warp instruction fetches four whole
//            128-byte rows (4 pairs) with 16-byte loads.  Per level a lane
//            issues all 16 tap loads (4 points x 4 corners) before it
//            accumulates them, so 16 rows per lane are in flight; taps
//            outside the map or with zero weight point at the head's row 0
//            with weight 0 (no branch around the loads), and adding
//            0 * (finite value) leaves the sum unchanged.  Each lane
//            accumulates its four channels over the 48 taps in the
//            reference's l -> p -> corner order with separate multiply and
//            add, which keeps the result bit-identical to the reference CPU
//            op whenever expf agrees.
// The value rows may be strided (ldv floats per token: the six decoder
// layers' projections share one [B][13125][6 * 256] buffer).
// The canonical (PyTorch MSDeformAttn) form takes locations and
// post-softmax weights directly and shares phase 2.
#include "common.cuh"
#include "kernels.h"

namespace ppdl {

namespace {

constexpr int kPairs = 16;     // (query, head) pairs per block
constexpr int kThreads = 128;  // 4 warps x 4 pairs
constexpr int kTaps = 48;      // 3 levels x 4 points x 4 corners
constexpr int kTapStride = kTaps + 1;  // bank-conflict padding

__constant__ int c_lvl_w[3] = {100, 50, 25};
__constant__ int c_lvl_h[3] = {100, 50, 25};
__constant__ int c_lvl_start[3] = {0, 10000, 12500};

// (8 blocks per SM, 64 registers a thread: measured fastest of 4..10 blocks;
// with no bound ptxas keeps fewer loads in flight)
template <bool kCanon>
__global__ void __launch_bounds__(kThreads, 8)
msda_kernel(const float *__restrict__ val,  // [B][13125][ldv], 256 used
            const float *__restrict__ p1,   // offsets or locations [B*nq][ld1], 192 used
            const float *__restrict__ p2,   // logits or weights    [B*nq][ld2], 96 used
            const float *__restrict__ ref,  // [B*nq][4] (in-model only)
            float *__restrict__ out,        // [B*nq][256]
            int nq, int npairs, int ld1, int ld2, int ldv) {
    pdl_begin();
    __shared__ float s_w[kPairs][12];
    __shared__ int s_idx[kPairs][kTapStride];
    __shared__ float s_tw[kPairs][kTapStride];

    const int t = threadIdx.x;
    const int pair0 = blockIdx.x * kPairs;

    // phase 1a: attention weights of each pair (src/ppdoclayout.cpp:161-167)
    if (t < kPairs) {
        const int gp = pair0 + t;
        if (gp < npairs) {
            const int bq = gp >> 3, h = gp & 7;
            const float *a = p2 + (size_t)bq * ld2 + h * 12;
            if (kCanon) {
#pragma unroll
                for (int i = 0; i < 12; i++) s_w[t][i] = a[i];
            } else {
                float e[12];
                float amax = a[0];
#pragma unroll
                for (int i = 1; i < 12; i++) amax = fmaxf(amax, a[i]);
                float wsum = 0.0f;
#pragma unroll
                for (int i = 0; i < 12; i++) {
                    e[i] = expf(__fsub_rn(a[i], amax));
                    wsum = __fadd_rn(wsum, e[i]);
                }
#pragma unroll
                for (int i = 0; i < 12; i++) s_w[t][i] = __fdiv_rn(e[i], wsum);
            }
        }
    }
    __syncthreads();

    // phase 1b: taps of each sampling point (src/ppdoclayout.cpp:169-192)
    for (int it = t; it < kPairs * 12; it += kThreads) {
        const int lp = it / 12, pt = it - lp * 12;
        const int gp = pair0 + lp;
        if (gp >= npairs) continue;
        const int bq = gp >> 3, h = gp & 7;
        const int l = pt >> 2, p = pt & 3;
        const float ox = p1[(size_t)bq * ld1 + ((h * 3 + l) * 4 + p) * 2 + 0];
        const float oy = p1[(size_t)bq * ld1 + ((h * 3 + l) * 4 + p) * 2 + 1];
        float lx, ly;
        if (kCanon) {
            lx = ox;
            ly = oy;
        } else {
            const float *rq = ref + (size_t)bq * 4;
            // rq[0] + ox / NPTS * rq[2] * 0.5f, evaluated left to right
            lx = __fadd_rn(rq[0], __fmul_rn(__fmul_rn(__fmul_rn(ox, 0.25f), rq[2]), 0.5f));
            ly = __fadd_rn(rq[1], __fmul_rn(__fmul_rn(__fmul_rn(oy, 0.25f), rq[3]), 0.5f));
        }
        const int W = c_lvl_w[l], H = c_lvl_h[l], st = c_lvl_start[l];
        const float fx = __fsub_rn(__fmul_rn(lx, (float)W), 0.5f);
        const float fy = __fsub_rn(__fmul_rn(ly, (float)H), 0.5f);
        const float flx = floorf(fx), fly = floorf(fy);
        // (int) floor(f): the reference casts the float floor; values far
        // outside the map only need to stay out of bounds, so clamp before
        // the conversion to keep it defined.
        const int x0 = (int)fminf(fmaxf(flx, -4.0f), 4096.0f);
        const int y0 = (int)fminf(fmaxf(fly, -4.0f), 4096.0f);
        const float tx = __fsub_rn(fx, flx), ty = __fsub_rn(fy, fly);
        const float wt = s_w[lp][pt];
        const float cw[4] = {__fmul_rn(__fsub_rn(1.0f, tx), __fsub_rn(1.0f, ty)),
                             __fmul_rn(tx, __fsub_rn(1.0f, ty)),
                             __fmul_rn(__fsub_rn(1.0f, tx), ty), __fmul_rn(tx, ty)};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int xx = x0 + (k & 1), yy = y0 + (k >> 1);
            const bool ok = xx >= 0 && xx < W && yy >= 0 && yy < H && cw[k] != 0.0f;
            // a skipped tap reads row 0 with weight 0
            s_idx[lp][pt * 4 + k] = ok ? st + yy * W + xx : 0;
            s_tw[lp][pt * 4 + k] = ok ? __fmul_rn(wt, cw[k]) : 0.0f;
        }
    }
    __syncthreads();

    // phase 2: gather + weighted sum, 8 lanes x float4 per pair
    const int warp = t >> 5, lane = t & 31;
    const int lp = warp * 4 + (lane >> 3);
    const int c4 = (lane & 7) * 4;
    const int gp = pair0 + lp;
    if (gp >= npairs) return;
    const int bq = gp >> 3, h = gp & 7;
    const int b = bq / nq;
    const float *vb = val + (size_t)b * kNTok * ldv + h * kHD + c4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int l = 0; l < 3; l++) {
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; i++)
            v[i] = __ldg(reinterpret_cast<const float4 *>(vb + (size_t)s_idx[lp][l * 16 + i] * ldv));
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const float ww = s_tw[lp][l * 16 + i];
            acc.x = __fadd_rn(acc.x, __fmul_rn(ww, v[i].x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(ww, v[i].y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(ww, v[i].z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(ww, v[i].w));
        }
    }
    *reinterpret_cast<float4 *>(out + (size_t)bq * kDM + h * kHD + c4) = acc;
}

}  // namespace

Status launch_msda(const float *val, const float *p1, const float *p2, const float *ref,
                   float *out, int nq, int batch, bool canon, int ld1, int ld2,
                   cudaStream_t stream, int ldv) {
    if (nq <= 0 || batch <= 0 || ld1 < 192 || ld2 < 96 || ldv < kDM || ldv % 4) return ERR_SHAPE;
    if (((uintptr_t)val | (uintptr_t)out) & 15) return ERR_SHAPE;
    const int npairs = batch * nq * kNH;
    const int grid = cdiv(npairs, kPairs);
    if (canon)
        pdl_launch(msda_kernel<true>, grid, kThreads, 0, stream, val, p1, p2, ref, out, nq, npairs,
                   ld1, ld2, ldv);
    else
        pdl_launch(msda_kernel<false>, grid, kThreads, 0, stream, val, p1, p2, ref, out, nq, npairs,
                   ld1, ld2, ldv);
    return cuda_status();
}

}  // namespace ppdl
