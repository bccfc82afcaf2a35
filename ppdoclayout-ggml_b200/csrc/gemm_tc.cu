// gemm_tc.cu — FP32-faithful 3xTF32 GEMM on the 5th-generation tensor cores.
//
// Replaces the reference's cuBLAS SGEMM (CUBLAS_DEFAULT_MATH, no TF32:
// patches/ggml-ppdl.patch:14-16, 650-665, 787-802) for the 1x1 convs, the
// Winograd 36-plane madd and the decoder linears.  A plain TF32 product
// loses ~3 decimal digits, so every operand x is split into
// hi = x with the low 13 mantissa bits cleared (exactly TF32) and
// lo = x - hi (exact in FP32), and each K step accumulates
// hi_A*hi_B + hi_A*lo_B + lo_A*hi_B in FP32 — the classic 3xTF32 scheme,
// ~2^-21 relative per product, inside the hot path's 1e-5 gate.
//
// Kernel structure (persistent, one CTA per SM, 320 threads):
//   warp 8      TMA producer: A tile (FP32 activation) + B hi/lo tiles
//               (weights pre-split at init) into a stage of shared memory;
//   warps 4-7   converter: split the A tile in place (hi over the raw
//               values, lo into a twin buffer with the same layout), then
//               fence.proxy.async so the tensor core sees the writes;
//   warp 9      MMA issuer: one thread issues tcgen05.mma kind::tf32
//               (M=128, N=bn, K=8) x3 per K step into a TMEM accumulator,
//               tcgen05.commit frees the stage / publishes the tile;
//   warps 0-3   epilogue: tcgen05.ld 32x32b from the lane quadrant of
//               their warp, bias / residual / activation, global stores.
// Two TMEM accumulators (2 x 256 columns) overlap a tile's epilogue with
// the next tile's main loop.
//
// Layouts: A is either M-major — a CHW activation, pixels contiguous — read
// by TMA boxes of 32 pixels x 32 channels with the 128-byte swizzle on a
// 32-byte atom (the one M-major form UMMA accepts for TF32; descriptor
// layout type 1), or K-major (token-major rows, 128-byte swizzle).  B is
// K-major [N][K] with the 128-byte swizzle.  The element-wise split does not
// depend on the swizzle, so it runs in place on the TMA image.
//
// Every mbarrier wait is bounded (~2 s of clock64); on expiry the kernel
// raises a device error flag, all roles drain out, pending TMA and MMA work
// is waited for (again bounded) and TMEM is released before the CTA exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>

#include "gemm_tc.h"

namespace ppdl {

__device__ int g_tc_error = 0;

namespace {

constexpr int kBM = 128, kBK = 32;
// warps 0-3 and 8-11 epilogue, 4-5 converter, 6 TMA producer, 7 MMA issuer
constexpr int kThreads = 384;
constexpr int kWarpProducer = 6, kWarpMma = 7, kWarpEpi2 = 8;
constexpr int kConvThreads = 64;
constexpr int kEpiThreads = 256;
constexpr int kHalfCols = 64;  // columns of the N tile per epilogue warp
constexpr uint32_t kTmemCols = 512;
constexpr long long kTimeoutCycles = 4000000000LL;
constexpr int kMaxStages = 4;
constexpr int kABytes = kBM * kBK * 4;  // 16 KB
// TMEM (512 columns): hi*hi partials P0 | P1 (chunks of kChunkKB k-blocks,
// 16 MMA adds each) and cross-term accumulators X0 | X1 (hi*lo + lo*hi of a
// whole tile; they are ~2^-11 of the result, so their own accumulation error
// is negligible).  The running total lives in epilogue registers.
constexpr int kChunkKB = 1;
constexpr int kSlots = 2;
constexpr int kSlotCols = 128;
constexpr int kXCol = 256;
constexpr int kMaxBN = 128;

struct Args {
    int M, N, K, batch, planes, a_mn, bn, stages, m_tiles, n_tiles, tiles;
    uint32_t stage_bytes, tx_bytes, idesc;
    TcEpilogue epi;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: false when the phase did not complete within the time limit
// or another role already aborted.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > kTimeoutCycles) {
                *abort_flag = 1;
                atomicExch(&g_tc_error, 1);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *tm, uint32_t bar,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // descriptor version of sm_100
    d |= (uint64_t)(layout & 7u) << 61;
    return d;
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

template <int ACT>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBhi,
               const __grid_constant__ CUtensorMap tmBlo, const Args a) {
    extern __shared__ uint8_t smem_raw[];
    // control block: 16 mbarriers + tmem base + abort flag, then 1024-aligned stages
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ctrl = raw;
    const uint32_t bar_full = ctrl, bar_conv = ctrl + 8 * kMaxStages,
                   bar_empty = ctrl + 16 * kMaxStages, bar_pfull = ctrl + 24 * kMaxStages,
                   bar_pempty = bar_pfull + 8 * kSlots, bar_xfull = bar_pempty + 8 * kSlots,
                   bar_xempty = bar_xfull + 16, bar_done = bar_xempty + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem_raw + 256);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem_raw + 260);
    const uint32_t stage0 = (raw + 512 + 1023) & ~1023u;
    uint8_t *stage0_ptr = smem_raw + (stage0 - raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_conv + 8 * s, kConvThreads);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int i = 0; i < kSlots; i++) {
            mbar_init(bar_pfull + 8 * i, 1);
            mbar_init(bar_pempty + 8 * i, kEpiThreads);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bar_xfull + 8 * i, 1);
            mbar_init(bar_xempty + 8 * i, kEpiThreads);
        }
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int kblocks = (a.K + kBK - 1) / kBK;

    if (warp == kWarpProducer) {
        if (lane == 0) {
            long long it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x) {
                const int z = t / (a.m_tiles * a.n_tiles);
                const int r = t - z * a.m_tiles * a.n_tiles;
                const int m0 = (r / a.n_tiles) * kBM, n0 = (r % a.n_tiles) * a.bn;
                const int pz = z % a.planes;
                for (int kb = 0; kb < kblocks; kb++, it++) {
                    const int s = (int)(it % S);
                    const uint32_t ph = (uint32_t)((it / S) & 1);
                    if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t st = stage0 + s * a.stage_bytes;
                    const uint32_t fb = bar_full + 8 * s;
                    mbar_expect_tx(fb, a.tx_bytes);
                    const int k0 = kb * kBK;
                    if (a.a_mn) {
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            tma_load_3d(st + i * 4096, &tmA, fb, m0 + 32 * i, k0, z);
                    } else {
                        tma_load_3d(st, &tmA, fb, k0, m0, z);
                    }
                    tma_load_3d(st + 2 * kABytes, &tmBhi, fb, k0, n0, pz);
                    tma_load_3d(st + 2 * kABytes + a.bn * 128, &tmBlo, fb, k0, n0, pz);
                }
            }
            // drain: the last issued stages must land before the CTA may exit
            const long long first = it > S ? it - S : 0;
            for (long long j = first; j < it; j++) {
                const int s = (int)(j % S);
                int dummy = 0;
                mbar_wait(bar_full + 8 * s, (uint32_t)((j / S) & 1), (volatile int *)&dummy);
            }
        }
    } else if (warp >= 4 && warp < kWarpProducer) {
        // converter: in-place 3xTF32 split of the A tile
        const int ct = threadIdx.x - 128;
        long long it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < kblocks; kb++, it++) {
                const int s = (int)(it % S);
                const uint32_t ph = (uint32_t)((it / S) & 1);
                if (!mbar_wait(bar_full + 8 * s, ph, abort_flag)) {
                    ok = false;
                    break;
                }
                float4 *hi = reinterpret_cast<float4 *>(stage0_ptr + (size_t)s * a.stage_bytes);
                float4 *lo = hi + kABytes / 16;
#pragma unroll
                for (int i = 0; i < kABytes / 16 / kConvThreads; i++) {
                    const int idx = ct + kConvThreads * i;
                    const float4 v = hi[idx];
                    float4 h, l;
                    h.x = tf32_rna(v.x); h.y = tf32_rna(v.y);
                    h.z = tf32_rna(v.z); h.w = tf32_rna(v.w);
                    l.x = v.x - h.x; l.y = v.y - h.y; l.z = v.z - h.z; l.w = v.w - h.w;
                    hi[idx] = h;
                    lo[idx] = l;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(bar_conv + 8 * s);
            }
        }
    } else if (warp == kWarpMma) {
        // hi*hi products go to a fresh TMEM partial every kChunkKB k-blocks
        // (two slots, alternating), which the epilogue folds into its running
        // total with FP32 adds — the tensor core's own accumulation then sums
        // at most 16 of the large terms; the two small cross products go to
        // the tile's X slot.
        if (lane == 0) {
            long long it = 0, ctr = 0;
            int tcnt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x, tcnt++) {
                const int xs = tcnt & 1;
                if (!mbar_wait(bar_xempty + 8 * xs, (uint32_t)(((tcnt >> 1) & 1) ^ 1), abort_flag))
                    break;
                const uint32_t dx = tmem_base + (uint32_t)(kXCol + xs * kSlotCols);
                for (int kb0 = 0; kb0 < kblocks && ok; kb0 += kChunkKB, ctr++) {
                    const int p = (int)(ctr % kSlots);
                    const uint32_t pph = (uint32_t)((ctr / kSlots) & 1);
                    if (!mbar_wait(bar_pempty + 8 * p, pph ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(p * kSlotCols);
                    const int kb1 = kb0 + kChunkKB < kblocks ? kb0 + kChunkKB : kblocks;
                    for (int kb = kb0; kb < kb1; kb++, it++) {
                        const int s = (int)(it % S);
                        const uint32_t ph = (uint32_t)((it / S) & 1);
                        if (!mbar_wait(bar_conv + 8 * s, ph, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t st = stage0 + s * a.stage_bytes;
                        const uint32_t ahi = st, alo = st + kABytes;
                        const uint32_t bhi = st + 2 * kABytes, blo = bhi + a.bn * 128;
#pragma unroll
                        for (int kk = 0; kk < kBK / 8; kk++) {
                            uint64_t dah, dal;
                            if (a.a_mn) {  // 8 K rows = two 4-row groups of 512 B
                                dah = smem_desc(ahi + kk * 1024, 4096, 512, 1);
                                dal = smem_desc(alo + kk * 1024, 4096, 512, 1);
                            } else {       // 32 bytes of K inside the swizzled 128-byte row
                                dah = smem_desc(ahi + kk * 32, 16, 1024, 2);
                                dal = smem_desc(alo + kk * 32, 16, 1024, 2);
                            }
                            const uint64_t dbh = smem_desc(bhi + kk * 32, 16, 1024, 2);
                            const uint64_t dbl = smem_desc(blo + kk * 32, 16, 1024, 2);
                            umma_tf32(d, dah, dbh, a.idesc, (kb == kb0 && kk == 0) ? 0u : 1u);
                            umma_tf32(dx, dal, dbh, a.idesc, (kb == 0 && kk == 0) ? 0u : 1u);
                            umma_tf32(dx, dah, dbl, a.idesc, 1u);
                        }
                        umma_commit(bar_empty + 8 * s);
                    }
                    if (!ok) break;
                    umma_commit(bar_pfull + 8 * p);
                }
                if (!ok) break;
                umma_commit(bar_xfull + 8 * xs);
            }
            // all issued MMAs must finish before TMEM is released
            umma_commit(bar_done);
            int dummy = 0;
            mbar_wait(bar_done, 0, (volatile int *)&dummy);
        }
    } else if (warp < 4 || warp >= kWarpEpi2) {
        // epilogue, 8 warps: two per TMEM lane quadrant (warp % 4), each
        // owning 64 of the bn <= 128 columns.  Every partial is folded into a
        // running FP32 total held in registers; the tile's cross terms are
        // added last and the total goes back into the X slot, from where a
        // compact 16-column loop applies bias / residual / activation and
        // stores (a small loop body keeps the instruction cache warm for the
        // other roles).
        const TcEpilogue &e = a.epi;
        const int quad = warp & 3;
        const int c_lo = warp >= kWarpEpi2 ? kHalfCols : 0;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const int nchunks = (kblocks + kChunkKB - 1) / kChunkKB;
        float tot[kHalfCols];
        long long ctr = 0;
        int tcnt = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x, tcnt++) {
            const int z = t / (a.m_tiles * a.n_tiles);
            const int r = t - z * a.m_tiles * a.n_tiles;
            const int m0 = (r / a.n_tiles) * kBM, n0 = (r % a.n_tiles) * a.bn;
            const int m = m0 + quad * 32 + lane;
            float *C = e.C + (long long)z * e.c_bs;
            const float *R = e.res_mode ? e.res + (long long)z * e.res_bs : nullptr;
            for (int c = 0; c < nchunks; c++, ctr++) {
                const int p = (int)(ctr % kSlots);
                const uint32_t pph = (uint32_t)((ctr / kSlots) & 1);
                if (!mbar_wait(bar_pfull + 8 * p, pph, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t part = tmem_base + lane_base + (uint32_t)(p * kSlotCols + c_lo);
#pragma unroll
                for (int q = 0; q < kHalfCols / 32; q++) {
                    if (c_lo + q * 32 < a.bn) {
                        uint32_t v[32];
                        tmem_ld32(part + (uint32_t)(q * 32), v);
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            tot[q * 32 + j] = c == 0 ? __uint_as_float(v[j])
                                                     : tot[q * 32 + j] + __uint_as_float(v[j]);
                    }
                }
                tc_fence_before();
                mbar_arrive(bar_pempty + 8 * p);
            }
            if (!ok) break;
            const int xs = tcnt & 1;
            if (!mbar_wait(bar_xfull + 8 * xs, (uint32_t)((tcnt >> 1) & 1), abort_flag)) break;
            tc_fence_after();
            const uint32_t xa = tmem_base + lane_base + (uint32_t)(kXCol + xs * kSlotCols + c_lo);
#pragma unroll
            for (int q = 0; q < kHalfCols / 32; q++) {
                if (c_lo + q * 32 < a.bn) {
                    uint32_t v[32];
                    tmem_ld32(xa + (uint32_t)(q * 32), v);
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        v[j] = __float_as_uint(tot[q * 32 + j] + __uint_as_float(v[j]));
                    tmem_st32(xa + (uint32_t)(q * 32), v);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            const bool row_ok = m < a.M;
            float *Crow = C + (long long)m * e.ldc_m;
            const float *Rrow = R ? R + (long long)m * e.res_ldm : nullptr;
            const int c_hi = a.bn < c_lo + kHalfCols ? a.bn : c_lo + kHalfCols;
            const uint32_t xt = tmem_base + lane_base + (uint32_t)(kXCol + xs * kSlotCols);
#pragma unroll 1
            for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
                const uint32_t xa = xt;
                uint32_t v[16];
                tmem_ld16(xa + (uint32_t)c0, v);
                if (!row_ok) continue;
                // row-major output (token-major linears): each thread owns a
                // row, so 16 consecutive columns go out as four 16-byte stores
                float *cp = Crow + (n0 + c0);
                if (e.ldc_n == 1 && n0 + c0 + 16 <= a.N && ((uintptr_t)cp & 15) == 0 &&
                    (e.res_mode == 0 || e.res_ldn == 1)) {
                    float y[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int n = n0 + c0 + j;
                        float x = __uint_as_float(v[j]);
                        if (e.alpha != 1.0f) x = x * e.alpha;
                        if (e.bias) x = x + __ldg(e.bias + n);
                        if (e.res_mode == 1) x = x + Rrow[n];
                        x = act_apply(x, ACT);
                        if (e.res_mode == 2) x = x + Rrow[n];
                        y[j] = x;
                    }
                    float4 *c4 = reinterpret_cast<float4 *>(cp);
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        c4[j] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
                    continue;
                }
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int n = n0 + c0 + j;
                    if (n < a.N) {
                        float x = __uint_as_float(v[j]);
                        if (e.alpha != 1.0f) x = x * e.alpha;
                        if (e.bias) x = x + __ldg(e.bias + n);
                        if (e.res_mode == 1) x = x + Rrow[(long long)n * e.res_ldn];
                        x = act_apply(x, ACT);
                        if (e.res_mode == 2) x = x + Rrow[(long long)n * e.res_ldn];
                        Crow[(long long)n * e.ldc_n] = x;
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(bar_xempty + 8 * xs);
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kWarpMma) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols)
                     : "memory");
    }
}

__global__ void tf32_split_kernel(const float *__restrict__ w, float *__restrict__ hi,
                                  float *__restrict__ lo, long long n) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = w[i];
    const float h = tf32_rna(v);
    hi[i] = h;
    lo[i] = v - h;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
        else
            cudaGetLastError();
    }
    return fn;
}

bool encode3d(CUtensorMap *tm, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t s1_bytes, uint64_t s2_bytes, uint32_t b0, uint32_t b1,
              CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    if (((uintptr_t)base & 15) || (s1_bytes & 15) || (s2_bytes & 15)) return false;
    const cuuint64_t dims[3] = {d0, d1, d2 ? d2 : 1};
    const cuuint64_t strides[2] = {s1_bytes, s2_bytes ? s2_bytes : s1_bytes * d1};
    const cuuint32_t box[3] = {b0, b1, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(base), dims, strides, box,
              es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

}  // namespace

Status launch_tf32_split(const float *w, float *hi, float *lo, long long n, cudaStream_t st) {
    if (n <= 0) return n == 0 ? OK : ERR_SHAPE;
    tf32_split_kernel<<<(int)((n + 255) / 256), 256, 0, st>>>(w, hi, lo, n);
    return cuda_status();
}

bool tc_gemm_plan(TcGemm *g, int M, int N, int K, int batch, const float *A, int a_mn,
                  long long lda, long long a_bs, const float *Bhi, const float *Blo, int planes,
                  const TcEpilogue &epi) {
    g->ok = false;
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || planes <= 0) return false;
    if (K % 4) return false;  // B rows must be 16-byte multiples
    // N tile (multiple of 16, <= 160 so that two partial slots and the total
    // fit in the 512 TMEM columns): least padded columns, then the widest
    int bn = 16;
    long long best = -1;
    for (int c = 16; c <= kMaxBN; c += 16) {
        const long long cover = (long long)((N + c - 1) / c) * c;
        if (best < 0 || cover < best || (cover == best && c > bn)) {
            best = cover;
            bn = c;
        }
    }
    const uint32_t stage_bytes = 2 * kABytes + 2 * 128 * bn;
    int stages = (int)((220 * 1024 - 2048) / stage_bytes);
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return false;
    g->M = M; g->N = N; g->K = K; g->batch = batch; g->planes = planes;
    g->a_mn = a_mn; g->bn = bn; g->stages = stages;
    g->smem = 2048 + (size_t)stages * stage_bytes;
    if (g->smem < 120 * 1024) g->smem = 120 * 1024;  // one CTA per SM: TMEM is not shared
    g->m_tiles = (M + kBM - 1) / kBM;
    g->n_tiles = (N + bn - 1) / bn;
    g->tiles = g->m_tiles * g->n_tiles * batch;
    g->epi = epi;
    bool ok;
    if (a_mn)
        ok = encode3d(&g->tmA, A, (uint64_t)M, (uint64_t)K, (uint64_t)batch, (uint64_t)lda * 4,
                      (uint64_t)a_bs * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    else
        ok = encode3d(&g->tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)batch, (uint64_t)lda * 4,
                      (uint64_t)a_bs * 4, 32, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    ok = ok && encode3d(&g->tmBhi, Bhi, (uint64_t)K, (uint64_t)N, (uint64_t)planes,
                        (uint64_t)K * 4, (uint64_t)K * N * 4, 32, (uint32_t)bn,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    ok = ok && encode3d(&g->tmBlo, Blo, (uint64_t)K, (uint64_t)N, (uint64_t)planes,
                        (uint64_t)K * 4, (uint64_t)K * N * 4, 32, (uint32_t)bn,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    g->ok = ok;
    return ok;
}

Status launch_tc_gemm(const TcGemm &g, cudaStream_t st) {
    if (!g.ok || g.epi.act < 0 || g.epi.act > 3) return ERR_SHAPE;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        const int smax = 227 * 1024;
        if (cudaFuncSetAttribute(tc_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smax) != cudaSuccess ||
            cudaFuncSetAttribute(tc_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smax) != cudaSuccess ||
            cudaFuncSetAttribute(tc_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smax) != cudaSuccess ||
            cudaFuncSetAttribute(tc_gemm_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smax) != cudaSuccess)
            return ERR_CUDA;
        attr[dev] = true;
    }
    Args a;
    a.M = g.M; a.N = g.N; a.K = g.K; a.batch = g.batch; a.planes = g.planes;
    a.a_mn = g.a_mn; a.bn = g.bn; a.stages = g.stages;
    a.m_tiles = g.m_tiles; a.n_tiles = g.n_tiles; a.tiles = g.tiles;
    a.stage_bytes = 2 * kABytes + 2 * 128 * g.bn;
    a.tx_bytes = kABytes + 2 * 128 * g.bn;
    a.idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(g.a_mn ? 1 : 0) << 15) |
              ((uint32_t)(g.bn >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
    a.epi = g.epi;
    int grid = sm_count();
    if (grid > g.tiles) grid = g.tiles;
    switch (g.epi.act) {
        case ACT_RELU:
            tc_gemm_kernel<ACT_RELU><<<grid, kThreads, g.smem, st>>>(g.tmA, g.tmBhi, g.tmBlo, a);
            break;
        case ACT_SILU:
            tc_gemm_kernel<ACT_SILU><<<grid, kThreads, g.smem, st>>>(g.tmA, g.tmBhi, g.tmBlo, a);
            break;
        case ACT_GELU:
            tc_gemm_kernel<ACT_GELU><<<grid, kThreads, g.smem, st>>>(g.tmA, g.tmBhi, g.tmBlo, a);
            break;
        default:
            tc_gemm_kernel<ACT_NONE><<<grid, kThreads, g.smem, st>>>(g.tmA, g.tmBhi, g.tmBlo, a);
    }
    return cuda_status();
}

int tc_error_fetch_and_clear() {
    int h = 0, zero = 0;
    cudaMemcpyFromSymbol(&h, g_tc_error, sizeof(int));
    if (h) cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    return h;
}

}  // namespace ppdl
