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
// Kernel structure (persistent, one CTA per SM, 512 threads):
//   warp 12      TMA producer: A tile (FP32 activation) + B hi/lo tiles
//                (weights pre-split at init) into a stage of shared memory;
//   warps 4-7    converter, one warp per TMEM lane quadrant: each thread
//                reads one row of the stage's A tile (32 k values), splits
//                it into TF32 hi / lo and writes both into a TMEM A stage
//                with tcgen05.st — or, in gather mode, first builds its row
//                from a CHW conv input (implicit GEMM, any plane stride);
//   warps 13-14  MMA issuers: one thread each, taking alternate k-blocks,
//                issues tcgen05.mma kind::tf32 with A read from TMEM and B
//                from shared memory (M=128, N=bn, K=8), x3 per K step; one
//                tcgen05.commit per k-block frees the stage, the TMEM A
//                stage and publishes the partial;
//   warps 0-3,   epilogue: tcgen05.ld 32x32b from the lane quadrant of
//   8-11         their warp, FP32 folding of the partials, bias / residual /
//                activation; CHW and token-major outputs leave through
//                shared-memory boxes and TMA stores (asynchronous, clipped at
//                the tensor edges), other layouts through direct stores;
//   warp 15      idle (it completes the fourth warpgroup's register split).
// The A operand comes from TMEM because a TF32 MMA that reads both operands
// from shared memory runs at 153 cycles per 128x128x8 step on the B200
// against 64 with A in TMEM (measured back to back on one SM).
// An MMA issue blocks until the tensor pipe accepts it, so a lone issuing
// thread leaves the pipe idle through its waits and bookkeeping between
// k-blocks; with two, one thread's bookkeeping overlaps the other's MMAs
// (each tcgen05.commit tracks only its own thread's MMAs, and alternate
// k-blocks use disjoint TMEM slots and A stages).
// Three TMEM partial slots let the MMAs run ahead of the epilogue's folds and
// overlap a tile's stores with the next tile's main loop.
//
// Layouts: A is either M-major — a CHW activation, pixels contiguous — read
// by one TMA box of 128 pixels x 32 channels without swizzle (a converter
// lane reads its pixel down the 32 channel rows), or K-major (token-major
// rows or the gathered conv tile, 128-byte swizzle: a lane reads the eight
// 16-byte chunks of its row).  B is K-major [N][K] with the 128-byte swizzle.
//
// Every mbarrier wait is bounded (~2 s of clock64); on expiry the kernel
// raises a device error flag, all roles drain out, pending TMA and MMA work
// is waited for (again bounded) and TMEM is released before the CTA exits.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "gemm_tc.h"

namespace ppdl {

__device__ int g_tc_error = 0;

namespace {

constexpr int kBM = 128, kBK = 32;
// warps 0-3 and 8-11 epilogue, 4-7 converter, 12 TMA producer, 13 MMA issuer
constexpr int kThreads = 512;
constexpr int kWarpConv = 4, kWarpEpi2 = 8, kWarpProducer = 12, kWarpMma = 13, kMmaWarps = 2;
constexpr int kConvThreads = 128;
constexpr int kEpiThreads = 256;
constexpr int kHalfCols = 64;  // columns of the N tile per epilogue warp
constexpr uint32_t kTmemCols = 512;
constexpr long long kTimeoutCycles = 4000000000LL;
constexpr int kMaxStages = 6;
constexpr int kABytes = kBM * kBK * 4;  // 16 KB
// TMEM (512 columns): three partial slots of 128 columns, one k-block of all
// three products each (4 large + 8 small MMA adds; the running total lives
// in epilogue registers), then two A stages of 64 columns (hi in the first
// 32, lo in the next 32; lane = row of the A tile, column = k).
constexpr int kSlots = 3;
constexpr int kSlotCols = 128;
constexpr int kAStages = 2;
constexpr int kACol0 = kSlots * kSlotCols;
constexpr int kACols = 2 * kBK;
constexpr int kMaxBN = 128;
static_assert(kACol0 + kAStages * kACols <= (int)kTmemCols, "TMEM columns exceeded");
// Waiters on a stage's empty barrier (the epilogue for a partial, the
// converter for a TMEM A stage) rely on the stage ring being at least as
// long as the slot and A-stage rings, so that a barrier cannot complete a
// second phase before they look; the planner keeps stages >= kMinStages.
constexpr int kMinStages = kSlots > kAStages ? kSlots : kAStages;

// Epilogue staging for TMA stores of CHW outputs: per epilogue warp two
// boxes of 32 pixels x 16 channels (2 KB each).
constexpr int kBoxN = 16;
constexpr int kBoxBytes = 32 * kBoxN * 4;
constexpr int kStagingBytes = 8 * 2 * kBoxBytes;  // 32 KB
constexpr int kCtrlBytes = 2048;                 // control block + 1024-alignment slack
// box mode: input windows in flight (a ring of their own beside the stages)
constexpr int kMaxBoxes = 4;
// Alternate-tile epilogue (the ALT instantiations, for narrow tiles of one or
// two k-blocks, many per CTA): each epilogue warpgroup owns kSlots partial
// slots of kAltSlotCols columns (warpgroup g's slot s at TMEM column
// (g kSlots + s) kAltSlotCols, below the A stages) and the barriers that go
// with them.
constexpr int kAltSlotCols = 64;
static_assert(2 * kSlots * kAltSlotCols <= kACol0, "alternate slots overlap the A stages");
static_assert(16 * kMaxStages + 8 * kAStages + 8 * kSlots + 8 + 16 * kMaxBoxes <= 256 &&
                  16 * kMaxStages + 8 * kAStages + 32 * kSlots + 8 + 16 * kMaxBoxes <= 384,
              "mbarriers overlap the control words");
// rows mode: channel rows c and c + 4 of a CHW tensor lie 4 * plane floats
// apart, a 16-byte multiple for any plane, so the tensor is viewed as
// [pages][C / 4][4 * plane] and a k-block (32 channels) is four TMA boxes,
// one per q = c % 4, each 8 rows (channels q, q + 4, ..., q + 28) of
// kRowsBox floats: 128 pixels plus up to 3 floats of alignment remainder,
// rounded to 16 bytes.  A box is 4224 bytes (128-byte aligned boxes); the A
// region is rounded to 17 KB so that B stays 1024-byte aligned.
constexpr int kRowsBox = 132;
constexpr int kRowsQBytes = 8 * kRowsBox * 4;
constexpr int kRowsBytes = (4 * kRowsQBytes + 1023) / 1024 * 1024;
static_assert(kRowsQBytes % 128 == 0 && kRowsBytes % 1024 == 0, "rows-mode layout");
constexpr int kSmemMax = 227 * 1024;

// Registers per thread: at launch (the __launch_bounds__(512, 1) maximum,
// checked on the host before every launch) and after the setmaxnreg split
// (converter and producer / MMA warpgroups down, the two epilogue
// warpgroups up; each role sets its count in its own branch, because after a
// join the compiler may only assume the smaller one).
constexpr int kLaunchRegs = 128, kRegsConv = 96, kRegsMma = 48, kRegsEpi = 184;
static_assert(128 * kRegsConv + 128 * kRegsMma + 256 * kRegsEpi <= kThreads * kLaunchRegs,
              "register split exceeds the block's register pool");

struct Args {
    int M, N, K, batch, planes, a_mn, bn, stages, m_tiles, n_tiles, tiles;
    int gather, tma_c, box, rows, rows_offmul, rows_delta, kps;
    long long rows_plane;
    uint32_t stage_bytes, tx_bytes, idesc, staging_off;
    TcGather gg;
    TcConvBox cb;
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
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
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

// Position in a ring of n stages or slots: index and mbarrier phase parity,
// advanced by one step at a time (no division on the issue paths).
struct Ring {
    int i = 0, n;
    uint32_t ph = 0;
    __device__ explicit Ring(int n_) : n(n_) {}
    __device__ __forceinline__ void next() {
        if (++i == n) {
            i = 0;
            ph ^= 1u;
        }
    }
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *tm, uint32_t bar,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, uint32_t bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *tm, uint32_t bar,
                                            int x, int y, int z, int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap *tm, uint32_t bar,
                                            int x, int y, int z, int w, int v) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v)
        : "memory");
}

// TMA store of a shared-memory box into the tensor (async proxy; the box
// must be published with fence.proxy.async first).  Coordinates are never
// negative here; parts of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *tm, uint32_t src, int x, int y,
                                             int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(tm)),
        "r"(src), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *tm, uint32_t src, int x, int y,
                                             int z, int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(tm)),
        "r"(src), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// at most one committed store group may still be reading shared memory
__device__ __forceinline__ void bulk_wait_read_1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
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

// D (TMEM) (+)= A (TMEM, 128 lanes x 8 columns) * B (shared-memory descriptor)
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
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
// 64 columns of the warp's lane quadrant, loaded and waited for in one
// statement (the wait and the register outputs cannot be separated)
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
        "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
        "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
        "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63 "
        "}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[64]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {"
        "%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, "
        "%33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, "
        "%49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64 "
        "};"
        ::"r"(taddr),
          "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]),
          "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]),
          "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]),
          "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]),
          "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
        : "memory");
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
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Gather mode: converter thread ct builds row ct of a stage's A tile
// (pixel m0 + ct, k = k0 .. k0 + 31) straight from the CHW input with 4-byte
// cp.async copies (zero-filled outside the image or past K/M), into the
// K-major 128-byte-swizzled layout (16-byte chunk c of row r at chunk
// position c ^ (r & 7)), the layout of a TMA-loaded K-major tile; the same
// thread later reads the row back for the split (split_row_kmajor).  Lanes
// run over consecutive pixels, so every copy instruction reads one
// contiguous (stride S) run of an input row.  oy0/ox0 hold the row's
// top-left input coordinate (oy*S - P, ox*S - P), oy0 = -64 for rows past M
// (below any kernel tap, and small enough that oy0 * W cannot overflow).
__device__ __forceinline__ void cp_async4(uint32_t dst, const float *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}

__device__ __forceinline__ void gather_issue(const TcGather &g, int K, const float *__restrict__ xz,
                                             uint32_t stage, int ct, int oy0, int ox0, int k0) {
    const uint32_t row_dst = stage + (uint32_t)ct * 128u;
    const uint32_t sw = (uint32_t)(ct & 7);
    if (g.KS == 1) {
        // pointwise conv: A(m, k) = x[k][m] (S = 1, P = 0)
        const bool in_m = oy0 >= 0;
        const float *xm = xz + (in_m ? oy0 * g.W + ox0 : 0);
#pragma unroll 8
        for (int j = 0; j < kBK; j++) {
            const bool in = in_m && k0 + j < K;
            const uint32_t off = ((((uint32_t)j >> 2) ^ sw) << 4) + ((uint32_t)j & 3u) * 4u;
            cp_async4(row_dst + off, in ? xm + (long long)(k0 + j) * g.plane : xz, in);
        }
    } else {
        const int kk2 = g.KS * g.KS;
        int ic = k0 / kk2;
        const int tap = k0 - ic * kk2;
        int kh = tap / g.KS;
        int kw = tap - kh * g.KS;
#pragma unroll 8
        for (int j = 0; j < kBK; j++) {
            const bool kv = k0 + j < K;
            const float *xc = xz + (long long)ic * g.plane + kh * g.W + kw;
            const uint32_t off = ((((uint32_t)j >> 2) ^ sw) << 4) + ((uint32_t)j & 3u) * 4u;
            const int iy = oy0 + kh, ix = ox0 + kw;
            const bool in = kv && (unsigned)iy < (unsigned)g.H && (unsigned)ix < (unsigned)g.W;
            cp_async4(row_dst + off, in ? xc + (oy0 * g.W + ox0) : xz, in);
            if (++kw == g.KS) {
                kw = 0;
                if (++kh == g.KS) {
                    kh = 0;
                    ++ic;
                }
            }
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// 3xTF32 split of 8 values into TMEM: hi = x rounded to the nearest TF32,
// ties away from zero, lo = x - hi (exact in FP32, either sign, so the
// tensor core's truncation of lo carries no bias); hi goes to columns
// col .. col + 7 of the warp's lane quadrant, lo 32 columns further.  The
// rounding is done on the bit pattern — add half a TF32 unit (bit 12) to
// the sign-magnitude encoding and clear the 13 low mantissa bits, carries
// running into the exponent — which gives cvt.rna.tf32.f32's result for
// every finite x (measured bitwise-equal GEMM outputs) in two integer ops
// (the split runs at the converter warps' throughput limit).
__device__ __forceinline__ uint32_t tf32_rna_bits(float x) {
    return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}

__device__ __forceinline__ void split_store8(uint32_t col, const float (&x)[8]) {
    uint32_t h[8], l[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
        h[u] = tf32_rna_bits(x[u]);
        l[u] = __float_as_uint(x[u] - __uint_as_float(h[u]));
    }
    tmem_st8(col, h);
    tmem_st8(col + kBK, l);
}

// The thread's row r of a K-major 128-byte-swizzled A tile (TMA-loaded or
// gathered) into the TMEM A stage at column col.
__device__ __forceinline__ void split_row_kmajor(const uint8_t *tile, int r, uint32_t col) {
    const float4 *row = reinterpret_cast<const float4 *>(tile + (size_t)r * 128);
#pragma unroll
    for (int h = 0; h < 4; h++) {
        const float4 v0 = row[(2 * h) ^ (r & 7)], v1 = row[(2 * h + 1) ^ (r & 7)];
        const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        split_store8(col + 8 * h, x);
    }
}

// The thread's row r (a pixel) of an M-major A tile stored as 32 channel
// rows of 128 pixels (no swizzle) into the TMEM A stage at column col.
__device__ __forceinline__ void split_row_mmajor(const uint8_t *tile, int r, uint32_t col) {
    const float *t = reinterpret_cast<const float *>(tile) + r;
#pragma unroll
    for (int h = 0; h < 4; h++) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) x[u] = t[(8 * h + u) * kBM];
        split_store8(col + 8 * h, x);
    }
}

// Box mode: the thread's A row (one output pixel) of k-block j of the
// current input window.  base = the pixel's offset in the window (row
// r * Wb + column cx * S + alignment remainder), chs = the window's channel
// stride (4 * Wb floats).  With 32 channels per window (lcb = 5) k-block j
// is kernel column j; with CB = 4, 8 or 16 channels (lcb = 2..4) the one
// k-block of the window holds all KS kernel columns, k = kw * CB + c, and
// k >= KS * CB (zero weight columns) reads column 0, which holds finite data.
template <int LCB>
__device__ __forceinline__ void split_row_box_small(const float *win, int base, int chs, int KS,
                                                    uint32_t col) {
#pragma unroll
    for (int h = 0; h < 4; h++) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            constexpr int kCB = 1 << LCB;
            const int k = 8 * h + u, kw = k >> LCB, c = k & (kCB - 1);
            x[u] = kw < KS ? win[base + c * chs + kw] : win[base];
        }
        split_store8(col + 8 * h, x);
    }
}

__device__ __forceinline__ void split_row_box(const float *win, int base, int chs, int j, int lcb,
                                              int KS, uint32_t col) {
    if (lcb == 5) {
        const float *t = win + base + j;
#pragma unroll
        for (int h = 0; h < 4; h++) {
            float x[8];
#pragma unroll
            for (int u = 0; u < 8; u++) x[u] = t[(8 * h + u) * chs];
            split_store8(col + 8 * h, x);
        }
    } else if (lcb == 4) {
        split_row_box_small<4>(win, base, chs, KS, col);
    } else if (lcb == 3) {
        split_row_box_small<3>(win, base, chs, KS, col);
    } else {
        split_row_box_small<2>(win, base, chs, KS, col);
    }
}

// Rows mode: the thread's pixel r of a k-block stored as four boxes (q =
// channel % 4) of 8 rows of kRowsBox floats, the rows of box q starting
// (q * offmul + delta) & 3 floats late (the box began at the 16-byte
// boundary below them).
__device__ __forceinline__ void split_row_rows(const uint8_t *tile, int r, int offmul, int delta,
                                               uint32_t col) {
    const float *t = reinterpret_cast<const float *>(tile) + r;
    int off[4];
#pragma unroll
    for (int q = 0; q < 4; q++) off[q] = q * (kRowsQBytes / 4) + ((q * offmul + delta) & 3);
#pragma unroll
    for (int h = 0; h < 4; h++) {
        float x[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int j = 8 * h + u;  // channel k0 + j: box j % 4, row j / 4
            x[u] = t[off[j & 3] + (j >> 2) * kRowsBox];
        }
        split_store8(col + 8 * h, x);
    }
}

// A-operand modes, a template parameter so that each role keeps only the
// state of its mode (the converter runs at its register limit)
constexpr int kModeTile = 0;  // TMA tile of A (M- or K-major), or the gather
constexpr int kModeBox = 1;   // implicit conv from TMA windows of the input
constexpr int kModeRows = 2;  // M-major A as 32 per-channel TMA rows
constexpr int kModeBits = 3;  // A as kModeTile; output packed 1 bit per (m, n): total > 0

template <int ACT, int AMODE, bool ALT = false>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBhi,
               const __grid_constant__ CUtensorMap tmBlo, const __grid_constant__ CUtensorMap tmC,
               const __grid_constant__ Args a) {
    extern __shared__ uint8_t smem_raw[];
    // control block: mbarriers + tmem base + abort flag, then 1024-aligned stages
    //   full[s]   TMA bytes of stage s landed (producer arrive + tx)
    //   empty[s]  the MMAs of the k-block in stage s completed (one
    //             tcgen05.commit): stage s is free, and so are that
    //             k-block's TMEM A stage and its partial slot may be folded
    //   afull[j]  TMEM A stage j written by the 128 converter threads
    //   pempty[p] partial slot p folded by the 256 epilogue threads
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ctrl = raw;
    const uint32_t bar_full = ctrl, bar_empty = ctrl + 8 * kMaxStages,
                   bar_afull = ctrl + 16 * kMaxStages, bar_pempty = bar_afull + 8 * kAStages,
                   bar_done = bar_pempty + 8 * (ALT ? 2 * kSlots : kSlots),
                   bar_bfull = bar_done + 8, bar_bempty = bar_bfull + 8 * kMaxBoxes,
                   bar_pfull = bar_bempty + 8 * kMaxBoxes;  // ALT only
    constexpr int kCtrlWord = ALT ? 384 : 256;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem_raw + kCtrlWord);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem_raw + kCtrlWord + 4);
    const uint32_t stage0 = (raw + 512 + 1023) & ~1023u;
    uint8_t *stage0_ptr = smem_raw + (stage0 - raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int j = 0; j < kAStages; j++) mbar_init(bar_afull + 8 * j, kConvThreads);
        if constexpr (ALT) {
            // pempty[p]: slot p folded by its warpgroup (slots 0..2 by
            // warpgroup 0, 3..5 by warpgroup 1); pfull[p]: its partial is
            // complete
            for (int i = 0; i < 2 * kSlots; i++) {
                mbar_init(bar_pempty + 8 * i, kEpiThreads / 2);
                mbar_init(bar_pfull + 8 * i, 1);
            }
        } else {
            for (int i = 0; i < kSlots; i++) mbar_init(bar_pempty + 8 * i, kEpiThreads);
        }
        mbar_init(bar_done, kMmaWarps);
        // box mode: bfull[b] window b landed (producer arrive + tx),
        // bempty[b] window b read by all 128 converter threads
        for (int b = 0; b < kMaxBoxes; b++) {
            mbar_init(bar_bfull + 8 * b, 1);
            mbar_init(bar_bempty + 8 * b, kConvThreads);
        }
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
    // barriers and TMEM are set up before the wait for the previous grid:
    // every global access of every role follows it
    pdl_begin();
    const int kblocks = (a.K + kBK - 1) / kBK;
    // k-blocks of the tiles of batch entry z: all of them, or with split K
    // (a.kps > 0) the range [z kps, z kps + kps) of the entry's split z
    const int pkps = a.kps;
    auto kb_first = [&](int z) { return pkps ? z * pkps : 0; };
    auto kb_count = [&](int z) {
        return pkps ? (kblocks - z * pkps < pkps ? kblocks - z * pkps : pkps) : kblocks;
    };

    // register split: the converter and producer / MMA warpgroups hand
    // registers to the two epilogue warpgroups, whose 64-float running
    // totals would otherwise spill to local memory.  The host launches only
    // when the kernel holds kLaunchRegs registers per thread, so the block's
    // pool covers both shares.
    if (warp >= kWarpProducer) {
        // producer / MMA warpgroup
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsMma));
        // parameters in registers (the waits below clobber memory)
        const int ptiles = a.tiles, pmt = a.m_tiles, pnt = a.n_tiles, pbn = a.bn,
                  pamn = a.a_mn, pgather = a.gather,
                  pplanes = a.planes;
        const uint32_t pstage = a.stage_bytes, ptx = a.tx_bytes, pidesc = a.idesc;
        if (warp == kWarpProducer) {
            if constexpr (AMODE == kModeRows) {
                // rows mode, the whole warp: lane 0 waits for the stage and
                // arms its barrier, then lanes 0-3 issue the four boxes of
                // the k-block (each from the 16-byte boundary below its rows)
                // and lane 0 the B loads
                long long it = 0;
                Ring rs(S);
                bool ok = true;
                const long long rplane = a.rows_plane;
                const int rdelta = a.rows_delta;
                for (int t = blockIdx.x; t < ptiles && ok; t += gridDim.x) {
                    const int z = t / (pmt * pnt);
                    const int r = t - z * pmt * pnt;
                    const int mt = r / pnt;
                    const int m0 = mt * kBM, n0 = (r - mt * pnt) * pbn;
                    const int pz = z % pplanes;
                    const int nkb = kb_count(z);
                    for (int kb = 0; kb < nkb; kb++, it++, rs.next()) {
                        const int s = rs.i;
                        bool good = true;
                        if (lane == 0) {
                            good = mbar_wait(bar_empty + 8 * s, rs.ph ^ 1, abort_flag);
                            if (good) mbar_expect_tx(bar_full + 8 * s, ptx);
                        }
                        if (!__shfl_sync(0xffffffffu, good ? 1 : 0, 0)) {
                            ok = false;
                            break;
                        }
                        const uint32_t st = stage0 + s * pstage;
                        const uint32_t fb = bar_full + 8 * s;
                        const int k0 = (kb_first(z) + kb) * kBK;
                        if (lane < 4) {
                            const long long xr = (long long)lane * rplane + m0 + rdelta;
                            tma_load_3d(st + (uint32_t)(lane * kRowsQBytes), &tmA, fb,
                                        (int)(xr & ~3LL), k0 >> 2, z);
                        }
                        if (lane == 0) {
                            const uint32_t stb = st + pstage - 2u * 128u * pbn;
                            tma_load_3d(stb, &tmBhi, fb, k0, n0, pz);
                            tma_load_3d(stb + pbn * 128, &tmBlo, fb, k0, n0, pz);
                        }
                    }
                }
                if (lane == 0) {
                    const long long first = it > S ? it - S : 0;
                    for (long long jj = first; jj < it; jj++) {
                        int dummy = 0;
                        mbar_wait(bar_full + 8 * (int)(jj % S), (uint32_t)((jj / S) & 1),
                                  (volatile int *)&dummy);
                    }
                }
            } else if (lane == 0) {
                constexpr bool pbox = AMODE == kModeBox;
                const uint32_t box0 = stage0 + (uint32_t)S * pstage;
                long long it = 0, ib = 0;  // stages and windows issued
                Ring rs(S), rb(a.cb.nbox);
                bool ok = true;
                for (int t = blockIdx.x; t < ptiles && ok; t += gridDim.x) {
                    const int z = t / (pmt * pnt);
                    const int r = t - z * pmt * pnt;
                    const int mt = r / pnt;
                    const int m0 = mt * kBM, n0 = (r - mt * pnt) * pbn;
                    const int pz = z % pplanes;
                    // box mode: output tile origin and the window walk
                    // (k-block j of window (cb, kh))
                    int oy0 = 0, ox0 = 0, j = 0, kh = 0, cbk = 0;
                    if (pbox) {
                        const int ty = mt / a.cb.tiles_x;
                        oy0 = ty * 4;
                        ox0 = (mt - ty * a.cb.tiles_x) * 32;
                    }
                    // split K: every split reads the one A (batch entry 0) and
                    // B plane 0 at its own k range
                    const int nkb = kb_count(z), kbz = kb_first(z), az = pkps ? 0 : z;
                    const int bz = pkps ? 0 : pz;
                    for (int kb = 0; kb < nkb; kb++, it++, rs.next()) {
                        const int k0 = (kbz + kb) * kBK;
                        if (pbox && j == 0) {
                            if (!mbar_wait(bar_bempty + 8 * rb.i, rb.ph ^ 1, abort_flag)) {
                                ok = false;
                                break;
                            }
                            const uint32_t bb = bar_bfull + 8 * rb.i;
                            const uint32_t dst = box0 + (uint32_t)rb.i * a.cb.box_bytes;
                            mbar_expect_tx(bb, a.cb.box_tx);
                            const int x = ox0 * a.cb.S - a.cb.P - a.cb.o;
                            const int d = kh - a.cb.P;
                            if (a.cb.S == 1)
                                tma_load_4d(dst, &tmA, bb, x, oy0 + d, cbk * a.cb.CB, z);
                            else  // rows (H/2, parity): input row 2 * oy + d
                                tma_load_5d(dst, &tmA, bb, x, oy0 + (d >> 1), d & 1,
                                            cbk * a.cb.CB, z);
                            rb.next();
                            ib++;
                        }
                        const int s = rs.i;
                        const uint32_t ph = rs.ph;
                        if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        const uint32_t st = stage0 + s * pstage;
                        const uint32_t fb = bar_full + 8 * s;
                        mbar_expect_tx(fb, ptx);
                        if (pgather || pbox) {
                            // A is written by the converter warps / comes from a window
                        } else if (pamn) {
                            tma_load_3d(st, &tmA, fb, m0, k0, az);
                        } else {
                            tma_load_3d(st, &tmA, fb, k0, m0, az);
                        }
                        const uint32_t stb = st + (uint32_t)a.stage_bytes - 2u * 128u * pbn;
                        tma_load_3d(stb, &tmBhi, fb, k0, n0, bz);
                        tma_load_3d(stb + pbn * 128, &tmBlo, fb, k0, n0, bz);
                        if (pbox && ++j == a.cb.kbpb) {
                            j = 0;
                            if (++kh == a.cb.KS) {
                                kh = 0;
                                ++cbk;
                            }
                        }
                    }
                }
                // drain: the last issued stages and windows must land before
                // the CTA may exit
                const long long first = it > S ? it - S : 0;
                for (long long jj = first; jj < it; jj++) {
                    const int s = (int)(jj % S);
                    int dummy = 0;
                    mbar_wait(bar_full + 8 * s, (uint32_t)((jj / S) & 1), (volatile int *)&dummy);
                }
                const int nb = a.cb.nbox;
                const long long bfirst = ib > nb ? ib - nb : 0;
                for (long long jj = bfirst; jj < ib; jj++) {
                    int dummy = 0;
                    mbar_wait(bar_bfull + 8 * (int)(jj % nb), (uint32_t)((jj / nb) & 1),
                              (volatile int *)&dummy);
                }
            }
        } else if (warp < kWarpMma + kMmaWarps) {
            // Every k-block accumulates into a TMEM partial slot of its own
            // (kSlots slots, round robin), which the epilogue folds into its
            // running FP32 total.  Inside a k-block the two small cross products
            // go in first and the four large hi*hi products last, so the tensor
            // core's truncating accumulation acts on the large values only four
            // times per partial (the rounding of the small ones is ~2^-11 of
            // that).  With several slots the MMAs run ahead of the epilogue's
            // folds instead of waiting for each one.
            if (lane == 0) {
                // this thread issues the k-blocks it with it % kMmaWarps == q
                const int q = warp - kWarpMma;
                int it = 0;
                // rp: slot ring (ALT: of warpgroup 0's tiles; rq of
                // warpgroup 1's, which owns the CTA's odd tiles)
                Ring rs(S), rp(kSlots), rq(kSlots), ra(kAStages);
                bool ok = true;
                for (int t = blockIdx.x; t < ptiles && ok; t += gridDim.x) {
                    const int nkb = pkps ? kb_count(t / (pmt * pnt)) : kblocks;
                    const bool own1 = ALT && (((t - (int)blockIdx.x) / (int)gridDim.x) & 1);
                    for (int kb = 0; kb < nkb;
                         kb++, it++, rs.next(), (own1 ? rq : rp).next(), ra.next()) {
                        if (it % kMmaWarps != q) continue;
                        const Ring &sr = own1 ? rq : rp;
                        const int sp = own1 ? kSlots + sr.i : sr.i;
                        // the A stage is written only after the stage's TMA landed,
                        // so afull also covers the B operand
                        if (!mbar_wait(bar_pempty + 8 * sp, sr.ph ^ 1, abort_flag) ||
                            !mbar_wait(bar_afull + 8 * ra.i, ra.ph, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d =
                            tmem_base + (uint32_t)(sp * (ALT ? kAltSlotCols : kSlotCols));
                        const uint32_t ahi = tmem_base + (uint32_t)(kACol0 + ra.i * kACols);
                        const uint32_t alo = ahi + kBK;
                        const uint32_t bhi = stage0 + rs.i * pstage + pstage - 2u * 128u * pbn;
                        // B K-major: the K=8 step kk is 32 bytes into the swizzled
                        // row, i.e. +2 in the descriptor's start-address field
                        // (which cannot carry: shared addresses stay below 256 KB)
                        const uint64_t dbh = smem_desc(bhi, 16, 1024, 2);
                        const uint64_t dbl = smem_desc(bhi + pbn * 128, 16, 1024, 2);
#pragma unroll
                        for (int kk = 0; kk < kBK / 8; kk++) {
                            umma_tf32_ts(d, alo + 8 * kk, dbh + 2 * kk, pidesc, kk == 0 ? 0u : 1u);
                            umma_tf32_ts(d, ahi + 8 * kk, dbl + 2 * kk, pidesc, 1u);
                        }
#pragma unroll
                        for (int kk = 0; kk < kBK / 8; kk++)
                            umma_tf32_ts(d, ahi + 8 * kk, dbh + 2 * kk, pidesc, 1u);
                        umma_commit(bar_empty + 8 * rs.i);
                        if constexpr (ALT) umma_commit(bar_pfull + 8 * sp);
                    }
                }
                // all issued MMAs must finish before TMEM is released (both
                // issuers commit; the phase completes after the later one)
                umma_commit(bar_done);
                int dummy = 0;
                mbar_wait(bar_done, 0, (volatile int *)&dummy);
            }
        }
    } else if (warp >= kWarpConv && warp < kWarpEpi2) {
        // converter warpgroup
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsConv));
        // parameters in registers (the waits below clobber memory)
        const int ptiles = a.tiles, pmt = a.m_tiles, pnt = a.n_tiles, pbn = a.bn,
                  pamn = a.a_mn, pgather = a.gather,
                  pplanes = a.planes;
        const uint32_t pstage = a.stage_bytes, ptx = a.tx_bytes, pidesc = a.idesc;
        {
            // converter: thread ct owns row ct of every A tile (TMEM lane ct,
            // the lane quadrant of its warp).  For k-block i it writes TMEM A
            // stage i % 2 once the MMAs of k-block i - 2 (the stage's last
            // reader) completed — the empty barrier of that k-block's shared
            // stage, tracked by the lagging ring rw.
            const int ct = threadIdx.x - kWarpConv * 32;
            const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
            // the gather geometry stays in the parameter space (constant
            // cache), which keeps the converter inside its register share
            const TcGather &gg = a.gg;
            // gather mode: copies of up to `depth` k-blocks stay in flight; the
            // oldest is split once a newer one is issued.  A gathered row is
            // read back only by the thread that copied it, so a stage's A
            // region is free again once that k-block was split (depth < S).
            const int depth = S - 1 < 3 ? S - 1 : 3;
            int it = 0, pub = 0;  // k-blocks [pub, it) issued, not yet split (gather)
            Ring rs(S), rp(S), rw(S), ra(kAStages);  // issue, split, TMEM wait, A stage
            bool ok = true;
            // box mode: window ring, the thread's pixel offset in a window
            // and the k-block index inside the current window
            constexpr bool pbox = AMODE == kModeBox, prows = AMODE == kModeRows;
            Ring rbw(a.cb.nbox);
            const float *box0_ptr =
                reinterpret_cast<const float *>(stage0_ptr + (size_t)S * pstage);
            const int chs = 4 * a.cb.Wb;
            int wbase = 0, wj = 0;
            // split the k-block at ring position rp into TMEM A stage ra
            // (lane 0 waits for the warp and the verdict is shared, so the
            // warp-collective TMEM stores always run converged)
            auto publish = [&](int i) -> bool {
                bool good = true;
                if (lane == 0)
                    good = mbar_wait(bar_full + 8 * rp.i, rp.ph, abort_flag) &&
                           (i < kAStages || mbar_wait(bar_empty + 8 * rw.i, rw.ph, abort_flag));
                if (!__shfl_sync(0xffffffffu, good ? 1 : 0, 0)) return false;
                if (i >= kAStages) rw.next();
                tc_fence_after();
                const uint8_t *tile = stage0_ptr + (size_t)rp.i * pstage;
                const uint32_t col = tmem_base + lane_base + (uint32_t)(kACol0 + ra.i * kACols);
                if (pbox)
                    split_row_box(box0_ptr + (size_t)rbw.i * (a.cb.box_bytes / 4), wbase, chs, wj,
                                  a.cb.lcb, a.cb.KS, col);
                else if (prows)
                    split_row_rows(tile, ct, a.rows_offmul, a.rows_delta, col);
                else if (pamn && !pgather)
                    split_row_mmajor(tile, ct, col);
                else
                    split_row_kmajor(tile, ct, col);
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(bar_afull + 8 * ra.i);
                rp.next();
                ra.next();
                return true;
            };
            for (int t = blockIdx.x; t < ptiles && ok; t += gridDim.x) {
                const int z = t / (pmt * pnt);
                const int r = t - z * pmt * pnt;
                const int m0 = (r / pnt) * kBM;
                const float *xz = pgather ? gg.x + (long long)z * gg.x_bs : nullptr;
                if (pbox) {
                    // pixel (row ct / 32, column ct % 32) of the 4 x 32 tile
                    wbase = (ct >> 5) * a.cb.Wb + (ct & 31) * a.cb.S + a.cb.o;
                    wj = 0;
                }
                int oy0 = -64, ox0 = 0;
                if (pgather && m0 + ct < a.M) {
                    const int oy = (m0 + ct) / gg.OW;
                    const int ox = m0 + ct - oy * gg.OW;
                    oy0 = oy * gg.S - gg.P;
                    ox0 = ox * gg.S - gg.P;
                }
                const int nkb = kb_count(z);
                for (int kb = 0; kb < nkb; kb++, it++, rs.next()) {
                    if (pbox) {
                        if (wj == 0) {
                            bool good = true;
                            if (lane == 0) good = mbar_wait(bar_bfull + 8 * rbw.i, rbw.ph, abort_flag);
                            if (!__shfl_sync(0xffffffffu, good ? 1 : 0, 0)) {
                                ok = false;
                                break;
                            }
                        }
                        if (!publish(it)) {
                            ok = false;
                            break;
                        }
                        if (++wj == a.cb.kbpb) {
                            // the thread's reads of this window are done
                            mbar_arrive(bar_bempty + 8 * rbw.i);
                            rbw.next();
                            wj = 0;
                        }
                        continue;
                    }
                    if (!pgather) {
                        if (!publish(it)) {
                            ok = false;
                            break;
                        }
                        continue;
                    }
                    gather_issue(gg, a.K, xz, stage0 + (uint32_t)rs.i * pstage, ct, oy0, ox0,
                                 kb * kBK);
                    if (it + 1 - pub > depth) {
                        // at most `depth` newer groups pending -> k-block pub landed
                        if (depth >= 3)
                            asm volatile("cp.async.wait_group 3;" ::: "memory");
                        else if (depth == 2)
                            asm volatile("cp.async.wait_group 2;" ::: "memory");
                        else
                            asm volatile("cp.async.wait_group 1;" ::: "memory");
                        if (!publish(pub)) {
                            ok = false;
                            break;
                        }
                        pub++;
                    }
                }
            }
            if (pgather) {
                asm volatile("cp.async.wait_all;" ::: "memory");
                for (; ok && pub < it; pub++)
                    if (!publish(pub)) ok = false;
            }
        }
    } else {
        // epilogue warpgroups (warps 0-3, 8-11)
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsEpi));
        // epilogue, 8 warps: two per TMEM lane quadrant (warp % 4), each
        // owning 64 of the bn <= 128 columns.  Every partial is folded into a
        // running FP32 total held in registers and its slot freed at once, so
        // the MMAs of the next tile never wait for this tile's stores.  The
        // totals leave in 16-column chunks through a shared-memory box, where
        // a rolled loop applies bias / residual / activation (a small loop
        // body keeps the instruction cache warm for the other roles): CHW and
        // token-major outputs by TMA stores, other layouts by direct stores.
        // parameters in registers: every TMEM wait carries a memory clobber,
        // after which fields read through the parameter block would be
        // fetched again
        const TcEpilogue e = a.epi;
        const int pM = a.M, pN = a.N, pbn = a.bn, ptiles = a.tiles, pmt = a.m_tiles,
                  pnt = a.n_tiles, ptma = a.tma_c;
        const int quad = warp & 3;
        // the two warpgroups split the N tile in 16-column units: [0, half)
        // and [half, bn), half <= kHalfCols (a narrow tile keeps both busy).
        // ALT (N tiles of at most kHalfCols columns, one or two k-blocks,
        // several tiles per CTA, where the epilogue's per-tile instructions
        // bound the pipeline): each warpgroup instead takes every other tile
        // whole, so that a tile's folds and stores have two tile periods;
        // its slots and barriers are its own, so every waiter sees every
        // phase of its barriers in order, as in the shared form.
        const bool wg = warp >= kWarpEpi2;
        const int half = ((pbn + 31) / 32) * 16;
        const int c_lo = (wg && !ALT) ? half : 0;
        const int c_hi = (wg || ALT) ? pbn : half;
        const int ew = warp < 4 ? warp : warp - 4;  // epilogue warp 0..7
        // ReLU / SiLU / identity outputs apply alpha, bias and a mode-1
        // residual in registers before the box (measured faster); the GELU
        // form keeps the all-in-the-box loop
        constexpr bool kPreOps = ACT != ACT_GELU;
        const uint32_t staging = stage0 + a.staging_off;
        float *staging_ptr = reinterpret_cast<float *>(stage0_ptr + a.staging_off);
        constexpr bool pbox = AMODE == kModeBox;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        float tot[kHalfCols];
        long long ctr = 0;
        // rp: partial slot of the k-block, re: its shared stage, whose empty
        // barrier completes when the k-block's MMAs (and so its partial) did
        Ring rp(kSlots), re(S);
        int nbox = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ptiles && ok; t += gridDim.x) {
            const int z = t / (pmt * pnt);
            if constexpr (ALT) {
                if ((((t - (int)blockIdx.x) / (int)gridDim.x) & 1) != (int)wg)
                    continue;  // the other warpgroup's tile
            }
            const int r = t - z * pmt * pnt;
            const int mt = r / pnt;
            const int m0 = mt * kBM, n0 = (r - mt * pnt) * pbn;
            float *C = e.C + (long long)z * e.c_bs;
            const float *R = e.res_mode ? e.res + (long long)z * e.res_bs : nullptr;
            // (ReLU / SiLU outputs) the bias of the warp's columns c_lo + lane
            // and c_lo + 32 + lane, loaded while the k-blocks are folded and
            // handed to the store phase by warp shuffles
            float bias_lo = 0.0f, bias_hi = 0.0f;
            if (kPreOps && e.bias) {
                const int n_lo = n0 + c_lo + lane, n_hi = n_lo + 32;
                if (c_lo + lane < c_hi && n_lo < pN) bias_lo = __ldg(e.bias + n_lo);
                if (c_lo + 32 + lane < c_hi && n_hi < pN) bias_hi = __ldg(e.bias + n_hi);
            }
            // bias of column c (c_lo <= c < c_hi, warp-uniform half c - c_lo >= 32
            // or per-lane offsets below 32 within one half)
            auto bias_of = [&](int c) {
                const int o = c - c_lo;
                return __shfl_sync(0xffffffffu, o >= 32 ? bias_hi : bias_lo, o & 31);
            };
            const int nkb = kb_count(z);
            for (int c = 0; c < nkb; c++, ctr++, rp.next(), re.next()) {
                const int p = (ALT && wg) ? kSlots + rp.i : rp.i;
                if (!(ALT ? mbar_wait(bar_pfull + 8 * p, rp.ph, abort_flag)
                          : mbar_wait(bar_empty + 8 * re.i, re.ph, abort_flag))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t part = tmem_base + lane_base +
                                      (uint32_t)(p * (ALT ? kAltSlotCols : kSlotCols) + c_lo);
#pragma unroll
                for (int q = 0; q < kHalfCols / 32; q++) {
                    if (c_lo + q * 32 < c_hi) {
                        uint32_t v[32];
                        tmem_ld32(part + (uint32_t)(q * 32), v);
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            tot[q * 32 + j] = c == 0 ? __uint_as_float(v[j])
                                                     : tot[q * 32 + j] + __uint_as_float(v[j]);
                    }
                }
                // the slot is free as soon as it is folded, the tile's last one
                // included: the stores below work from the register totals
                tc_fence_before();
                mbar_arrive(bar_pempty + 8 * p);
            }
            if (!ok) break;
            // the tile's output rows (computed after the folds, which hold
            // the most registers): row m of the GEMM, or in box mode pixel
            // ox0 + lane of output row oy0 + quad (the warp's 32 rows)
            int m = m0 + quad * 32 + lane;
            bool row_ok = m < pM;
            int oy0 = 0, ox0 = 0;
            if (pbox) {
                const int ty = mt / a.cb.tiles_x;
                oy0 = ty * 4;
                ox0 = (mt - ty * a.cb.tiles_x) * 32;
                const int oy = oy0 + quad, ox = ox0 + lane;
                row_ok = oy < a.cb.OH && ox < a.cb.OW;
                m = oy * a.cb.OW + ox;
            }
            float *Crow = C + (long long)m * e.ldc_m;
            const float *Rrow = R ? R + (long long)m * e.res_ldm : nullptr;
            const bool ops = ACT != ACT_NONE || e.alpha != 1.0f || e.bias || e.res_mode;
            // one 16-column chunk of the register totals: staged through a
            // shared-memory box and a TMA store, or stored directly
            auto store_chunk = [&](int c0, const float (&v)[16]) {
                if constexpr (AMODE == kModeBits) {
                    // packed output (no epilogue ops): bit (m & 31) of word
                    // (m >> 5) of column n is total(m, n) > 0; the warp's 32
                    // rows are one word per column, made by one ballot
                    uint32_t mine = 0;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const uint32_t word = __ballot_sync(0xffffffffu, row_ok && v[j] > 0.0f);
                        if (lane == j) mine = word;
                    }
                    const int n = n0 + c0 + lane;
                    if (lane < 16 && n < pN && m0 + quad * 32 < pM)
                        reinterpret_cast<uint32_t *>(C)[(long long)n * e.ldc_n +
                                                        ((m0 + quad * 32) >> 5)] = mine;
                    return;
                }
                if (ptma == 1 || ptma == 3) {
                    // CHW output: the warp's 32 pixels x 16 channels go into a
                    // staging box (lane = pixel, conflict-free rows of 128 B)
                    // and out with one TMA store, which clips rows >= M and
                    // channels >= N (box mode: a 4-D store of 32 pixels of one
                    // output row, clipped at the row end).  Two boxes per warp
                    // alternate.
                    const int b = nbox & 1;
                    if (nbox >= 2) {
                        if (lane == 0) bulk_wait_read_1();
                        __syncwarp();
                    }
                    float *box = staging_ptr + (size_t)(ew * 2 + b) * (kBoxBytes / 4);
                    if constexpr (kPreOps) {
                        // op order per element: alpha, + bias, + residual (mode
                        // 1), activation, + residual (mode 2).  The chunk's 16
                        // residual loads are issued together up front; alpha,
                        // bias and a mode-1 residual are applied in registers on
                        // the way into the box, the activation in a rolled loop
                        // over the box, a mode-2 residual in a last pass.
                        float rres[16];
                        if (e.res_mode && ACT != ACT_NONE) {
#pragma unroll
                            for (int j = 0; j < 16; j++) {
                                const int n = n0 + c0 + j;
                                rres[j] =
                                    (n < pN && row_ok) ? Rrow[(long long)n * e.res_ldn] : 0.0f;
                            }
                        }
                        if constexpr (ACT == ACT_NONE) {
                            // identity: both residual modes add after the bias
#pragma unroll
                            for (int j = 0; j < 16; j++) {
                                float x = v[j];
                                if (e.alpha != 1.0f) x = x * e.alpha;
                                if (e.bias) x = x + bias_of(c0 + j);
                                box[j * 32 + lane] = x;
                            }
                            if (e.res_mode) {
#pragma unroll 4
                                for (int j = 0; j < 16; j++) {
                                    const int n = n0 + c0 + j;
                                    if (n < pN && row_ok)
                                        box[j * 32 + lane] += Rrow[(long long)n * e.res_ldn];
                                }
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; j++) {
                                float x = v[j];
                                if (e.alpha != 1.0f) x = x * e.alpha;
                                if (e.bias) x = x + bias_of(c0 + j);
                                if (e.res_mode == 1) x = x + rres[j];
                                box[j * 32 + lane] = x;
                            }
                            // four independent activations per pass: one at a
                            // time, SiLU's exp -> divide chain is latency-bound
#pragma unroll 4
                            for (int j = 0; j < 16; j++)
                                box[j * 32 + lane] = act_apply(box[j * 32 + lane], ACT);
                        }
                        if (ACT != ACT_NONE && e.res_mode == 2) {
#pragma unroll
                            for (int j = 0; j < 16; j++) box[j * 32 + lane] += rres[j];
                        }
                    } else {
                        // raw values first (16 stores), then alpha / bias /
                        // residual / activation in a rolled loop over the box: a
                        // small loop body, once per tile, keeps instruction
                        // fetch short (and the registers of the identity and
                        // GELU forms below their limit)
#pragma unroll
                        for (int j = 0; j < 16; j++) box[j * 32 + lane] = v[j];
                        if (ops) {
                            // four columns at a time: their bias and residual
                            // loads are issued together
#pragma unroll 1
                            for (int j0 = 0; j0 < 16; j0 += 4) {
                                float bb[4], rr[4];
#pragma unroll
                                for (int u = 0; u < 4; u++) {
                                    const int n = n0 + c0 + j0 + u;
                                    const bool ok_n = n < pN;
                                    bb[u] = (e.bias && ok_n) ? __ldg(e.bias + n) : 0.0f;
                                    rr[u] = (e.res_mode && ok_n && row_ok)
                                                ? Rrow[(long long)n * e.res_ldn] : 0.0f;
                                }
#pragma unroll
                                for (int u = 0; u < 4; u++) {
                                    float x = box[(j0 + u) * 32 + lane];
                                    if (e.alpha != 1.0f) x = x * e.alpha;
                                    if (e.bias) x = x + bb[u];
                                    if (e.res_mode == 1) x = x + rr[u];
                                    x = act_apply(x, ACT);
                                    if (e.res_mode == 2) x = x + rr[u];
                                    box[(j0 + u) * 32 + lane] = x;
                                }
                            }
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        // boxes wholly past the tensor edge are skipped; the
                        // group is committed regardless to keep the count
                        if (ptma == 3) {
                            if (oy0 + quad < a.cb.OH && n0 + c0 < pN)
                                tma_store_4d(&tmC, staging + (uint32_t)((ew * 2 + b) * kBoxBytes),
                                             ox0, oy0 + quad, n0 + c0, z);
                        } else if (m0 + quad * 32 < pM && n0 + c0 < pN) {
                            tma_store_3d(&tmC, staging + (uint32_t)((ew * 2 + b) * kBoxBytes),
                                         m0 + quad * 32, n0 + c0, z);
                        }
                        bulk_commit();
                    }
                    nbox++;
                    return;
                }
                if (!pbox && ptma == 2) {
                    // token-major output: the warp's 32 rows x 16 columns go into
                    // a row-major staging box (lane = row, four 16-byte stores)
                    // and out with one TMA store; the ops pass walks the box
                    // linearly, so consecutive lanes touch consecutive words:
                    // element i of the pass (box word i * 32 + lane) is column
                    // lane % 16 of row 2 i + lane / 16.  Without an activation
                    // (the decoder's residual linears) the 16 residual loads
                    // are issued together before the box is touched; with one,
                    // four at a time in a rolled loop (registers).
                    constexpr bool kResAhead = ACT == ACT_NONE;
                    float rres[kResAhead ? 16 : 1];
                    if (kResAhead && e.res_mode) {
#pragma unroll
                        for (int i = 0; i < (kResAhead ? 16 : 1); i++) {
                            const int n = n0 + c0 + (lane & 15);
                            const int mr = m0 + quad * 32 + 2 * i + (lane >> 4);
                            rres[i] = (n < pN && mr < pM)
                                          ? R[(long long)mr * e.res_ldm + (long long)n * e.res_ldn]
                                          : 0.0f;
                        }
                    }
                    const int b = nbox & 1;
                    if (nbox >= 2) {
                        if (lane == 0) bulk_wait_read_1();
                        __syncwarp();
                    }
                    float *box = staging_ptr + (size_t)(ew * 2 + b) * (kBoxBytes / 4);
                    float4 *row4 = reinterpret_cast<float4 *>(box + lane * 16);
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        row4[q] = make_float4(v[4 * q], v[4 * q + 1],
                                              v[4 * q + 2],
                                              v[4 * q + 3]);
                    if (ops && kResAhead) {
                        __syncwarp();  // the pass reads the other lanes' rows
                        const int n = n0 + c0 + (lane & 15);
                        float bb = 0.0f;
                        if constexpr (kPreOps)
                            bb = bias_of(c0 + (lane & 15));
                        else
                            bb = (e.bias && n < pN) ? __ldg(e.bias + n) : 0.0f;
#pragma unroll
                        for (int i = 0; i < (kResAhead ? 16 : 1); i++) {
                            const int idx = i * 32 + lane;
                            float x = box[idx];
                            if (e.alpha != 1.0f) x = x * e.alpha;
                            if (e.bias) x = x + bb;
                            if (e.res_mode) x = x + rres[i];
                            box[idx] = x;
                        }
                    } else if (ops) {
                        __syncwarp();  // the pass reads the other lanes' rows
                        // a lane's elements share one column: one bias for all
                        const int n = n0 + c0 + (lane & 15);
                        float bb = 0.0f;
                        if constexpr (kPreOps)
                            bb = bias_of(c0 + (lane & 15));
                        else
                            bb = (e.bias && n < pN) ? __ldg(e.bias + n) : 0.0f;
#pragma unroll 1
                        for (int i0 = 0; i0 < 16; i0 += 4) {
                            float rr[4];
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const int mr = m0 + quad * 32 + 2 * (i0 + u) + (lane >> 4);
                                rr[u] = (e.res_mode && n < pN && mr < pM)
                                            ? R[(long long)mr * e.res_ldm + (long long)n * e.res_ldn]
                                            : 0.0f;
                            }
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const int idx = (i0 + u) * 32 + lane;
                                float x = box[idx];
                                if (e.alpha != 1.0f) x = x * e.alpha;
                                if (e.bias) x = x + bb;
                                if (e.res_mode == 1) x = x + rr[u];
                                x = act_apply(x, ACT);
                                if (e.res_mode == 2) x = x + rr[u];
                                box[idx] = x;
                            }
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) {
                        if (m0 + quad * 32 < pM && n0 + c0 < pN)
                            tma_store_3d(&tmC, staging + (uint32_t)((ew * 2 + b) * kBoxBytes),
                                         n0 + c0, m0 + quad * 32, z);
                        bulk_commit();
                    }
                    nbox++;
                    return;
                }
                // any other layout (strides that TMA cannot take): the raw
                // values go through the thread's own column of a box, then a
                // rolled loop applies the ops and stores with the output strides
                // (all lanes run it when the bias comes by warp shuffle)
                if (!kPreOps && !row_ok) return;
                float *box = staging_ptr + (size_t)(ew * 2) * (kBoxBytes / 4);
#pragma unroll
                for (int j = 0; j < 16; j++) box[j * 32 + lane] = v[j];
#pragma unroll 1
                for (int j = 0; j < 16; j++) {
                    const int n = n0 + c0 + j;
                    float bj = 0.0f;
                    if constexpr (kPreOps) bj = bias_of(c0 + j);
                    if (n < pN && row_ok) {
                        float x = box[j * 32 + lane];
                        if (e.alpha != 1.0f) x = x * e.alpha;
                        if (e.bias) x = x + (kPreOps ? bj : __ldg(e.bias + n));
                        if (e.res_mode == 1) x = x + Rrow[(long long)n * e.res_ldn];
                        x = act_apply(x, ACT);
                        if (e.res_mode == 2) x = x + Rrow[(long long)n * e.res_ldn];
                        Crow[(long long)n * e.ldc_n] = x;
                    }
                }
            };
#pragma unroll
            for (int cq = 0; cq < kHalfCols / 16; cq++) {
                if (c_lo + 16 * cq < c_hi) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; j++) v[j] = tot[16 * cq + j];
                    store_chunk(c_lo + 16 * cq, v);
                }
            }
        }
        // the staging boxes must be read and the stores complete before exit
        if (ptma && lane == 0) bulk_wait_all();
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
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = w[i];
    const float h = tf32_rna(v);
    hi[i] = h;
    lo[i] = v - h;
}

__global__ void tf32_split_pad_kernel(const float *__restrict__ w, float *__restrict__ hi,
                                      float *__restrict__ lo, int rows, int K, int Kp) {
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * Kp) return;
    const int n = (int)(i / Kp), k = (int)(i - (long long)n * Kp);
    const float v = k < K ? w[(long long)n * K + k] : 0.0f;
    const float h = tf32_rna(v);
    hi[i] = h;
    lo[i] = v - h;
}

// Box-mode repack: hi/lo[n][k], k = (bx * kbpb * 32) + kw * CB + c with
// bx = cb * KS + kh, from w[n][ic = cb * CB + c][kh][kw]; zero where kw >= KS
// (window padding) or ic >= IC.
__global__ void tf32_split_box_kernel(const float *__restrict__ w, float *__restrict__ hi,
                                      float *__restrict__ lo, int OC, int IC, int KS, int CB,
                                      int kbpb, int Kb) {
    pdl_begin();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)OC * Kb) return;
    const int n = (int)(i / Kb), k = (int)(i - (long long)n * Kb);
    const int per = kbpb * 32;
    const int bx = k / per, kin = k - bx * per;
    const int kw = kin / CB, c = kin - kw * CB;
    const int kh = bx % KS, ic = (bx / KS) * CB + c;
    float v = 0.0f;
    if (kw < KS && ic < IC) v = w[(((long long)n * IC + ic) * KS + kh) * KS + kw];
    const float h = tf32_rna(v);
    hi[i] = h;
    lo[i] = v - h;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, resolved once (a function-local static
// initialiser runs exactly once even when several host threads make their
// first call together).
EncodeTiledFn encode_fn() {
    static const EncodeTiledFn fn = []() -> EncodeTiledFn {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (EncodeTiledFn)p;
        cudaGetLastError();
        return nullptr;
    }();
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
    pdl_launch(tf32_split_kernel, (int)((n + 255) / 256), 256, 0, st, w, hi, lo, n);
    return cuda_status();
}

Status launch_tf32_split_pad(const float *w, float *hi, float *lo, int rows, int K, int Kp,
                             cudaStream_t st) {
    if (rows <= 0 || K <= 0 || Kp < K) return ERR_SHAPE;
    const long long n = (long long)rows * Kp;
    pdl_launch(tf32_split_pad_kernel, (int)((n + 255) / 256), 256, 0, st, w, hi, lo, rows, K, Kp);
    return cuda_status();
}

Status launch_tf32_split_box(const float *w, float *hi, float *lo, int OC, int IC, int KS,
                             cudaStream_t st) {
    if (OC <= 0 || IC <= 0 || KS <= 0) return ERR_SHAPE;
    int CB, kbpb, nbx;
    tc_conv_box_blocks(IC, KS, &CB, &kbpb, &nbx);
    const int Kb = nbx * kbpb * 32;
    const long long n = (long long)OC * Kb;
    pdl_launch(tf32_split_box_kernel, (int)((n + 255) / 256), 256, 0, st, w, hi, lo, OC, IC, KS, CB,
               kbpb, Kb);
    return cuda_status();
}

namespace {

// Tile and stage sizing shared by the planners.  a_bytes: the A region of
// a stage (0 when A does not pass through the stages); ring_bytes: shared
// memory held beside the stages (box mode: the window ring); row_tiles:
// M tiles over all pages (0 = from M and batch).
bool plan_common(TcGemm *g, int M, int N, int K, int batch, int planes, const TcEpilogue &epi,
                 uint32_t a_bytes = kABytes, uint32_t ring_bytes = 0, long long row_tiles = 0) {
    g->ok = false;
    g->bits = 0;
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || planes <= 0) return false;
    // N tile (multiple of 16, <= 128 so that the partial slots and the A
    // stages fit in the 512 TMEM columns); cost model: the tiles one CTA
    // runs, ceil(tiles / SMs), x (bn + 64), the 64 standing for the per-tile
    // A traffic and epilogue overhead in column equivalents.  A GEMM of a
    // few dozen row tiles (the decoder's 2400 rows) thus takes narrower N
    // tiles and spreads over more SMs.
    if (row_tiles <= 0) row_tiles = (long long)((M + kBM - 1) / kBM) * batch;
    const long long sms = sm_count();
    int bn = 16;
    long long best = -1;
    for (int c = 16; c <= kMaxBN; c += 16) {
        const long long tiles = row_tiles * ((N + c - 1) / c);
        const long long cost = (tiles + sms - 1) / sms * (c + 64);
        if (best < 0 || cost < best || (cost == best && c > bn)) {
            best = cost;
            bn = c;
        }
    }
    const uint32_t stage_bytes = a_bytes + 2 * 128 * bn;
    const long long room = (long long)kSmemMax - kCtrlBytes - kStagingBytes - ring_bytes;
    int stages = room > 0 ? (int)(room / stage_bytes) : 0;
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < kMinStages) return false;
    g->M = M; g->N = N; g->K = K; g->batch = batch; g->planes = planes;
    g->bn = bn; g->stages = stages;
    g->smem = kCtrlBytes + (size_t)stages * stage_bytes + ring_bytes + kStagingBytes;
    if (g->smem < 120 * 1024) g->smem = 120 * 1024;  // one CTA per SM: TMEM is not shared
    g->m_tiles = (M + kBM - 1) / kBM;
    g->n_tiles = (N + bn - 1) / bn;
    g->tiles = g->m_tiles * g->n_tiles * batch;
    g->epi = epi;
    return true;
}

// An output whose strides are 16-byte multiples — CHW (pixels contiguous)
// or token-major (columns contiguous) — is stored by TMA through the
// staging boxes; any other output keeps the direct global stores.
void encode_c(TcGemm *g) {
    const TcEpilogue &e = g->epi;
    g->tma_c = 0;
    if (e.c_bs < 0 || ((uintptr_t)e.C & 15) || (e.c_bs * 4) % 16 ||
        (g->batch > 1 && e.c_bs == 0))
        return;
    if (g->box) {
        // box mode, CHW output [N][OH][OW]: 4-D map, boxes of 32 pixels of
        // one output row x 16 channels (output rows must be 16-byte multiples)
        const TcConvBox &b = g->cb;
        EncodeTiledFn fn = encode_fn();
        if (!fn || e.ldc_m != 1 || b.OW % 4 || (e.ldc_n * 4) % 16 ||
            e.ldc_n != (long long)b.OH * b.OW)
            return;
        const cuuint64_t dims[4] = {(cuuint64_t)b.OW, (cuuint64_t)b.OH, (cuuint64_t)g->N,
                                    (cuuint64_t)g->batch};
        const cuuint64_t strides[3] = {(cuuint64_t)b.OW * 4, (cuuint64_t)e.ldc_n * 4,
                                       (cuuint64_t)(e.c_bs ? e.c_bs : e.ldc_n * g->N) * 4};
        const cuuint32_t box[4] = {32, 1, kBoxN, 1};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        if (fn(&g->tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, e.C, dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
            CUDA_SUCCESS)
            g->tma_c = 3;
        return;
    }
    if (e.ldc_m == 1 && e.ldc_n > 0 && (e.ldc_n * 4) % 16 == 0) {
        // CHW: pixels contiguous, boxes of 32 pixels x 16 channels
        if (encode3d(&g->tmC, e.C, (uint64_t)g->M, (uint64_t)g->N, (uint64_t)g->batch,
                     (uint64_t)e.ldc_n * 4, (uint64_t)e.c_bs * 4, 32, kBoxN,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
            g->tma_c = 1;
    } else if (e.ldc_n == 1 && e.ldc_m > 0 && (e.ldc_m * 4) % 16 == 0) {
        // token-major: columns contiguous, boxes of 16 columns x 32 rows
        if (encode3d(&g->tmC, e.C, (uint64_t)g->N, (uint64_t)g->M, (uint64_t)g->batch,
                     (uint64_t)e.ldc_m * 4, (uint64_t)e.c_bs * 4, kBoxN, 32,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
            g->tma_c = 2;
    }
}

// B hi/lo tensor maps over [planes][N][ldk] halves, k < ldk (16-byte rows).
bool encode_b(TcGemm *g, const float *Bhi, const float *Blo, int ldk) {
    const uint64_t N = (uint64_t)g->N;
    return encode3d(&g->tmBhi, Bhi, (uint64_t)ldk, N, (uint64_t)g->planes, (uint64_t)ldk * 4,
                    (uint64_t)ldk * N * 4, 32, (uint32_t)g->bn, CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode3d(&g->tmBlo, Blo, (uint64_t)ldk, N, (uint64_t)g->planes, (uint64_t)ldk * 4,
                    (uint64_t)ldk * N * 4, 32, (uint32_t)g->bn, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

bool tc_gemm_plan(TcGemm *g, int M, int N, int K, int batch, const float *A, int a_mn,
                  long long lda, long long a_bs, const float *Bhi, const float *Blo, int planes,
                  const TcEpilogue &epi) {
    if (K % 4) {  // B rows must be 16-byte multiples
        g->ok = false;
        return false;
    }
    if (!plan_common(g, M, N, K, batch, planes, epi)) return false;
    g->a_mn = a_mn;
    g->gather = 0;
    g->box = 0;
    g->rows = 0;
    bool ok;
    if (a_mn)
        ok = encode3d(&g->tmA, A, (uint64_t)M, (uint64_t)K, (uint64_t)batch, (uint64_t)lda * 4,
                      (uint64_t)a_bs * 4, kBM, kBK, CU_TENSOR_MAP_SWIZZLE_NONE);
    else
        ok = encode3d(&g->tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)batch, (uint64_t)lda * 4,
                      (uint64_t)a_bs * 4, 32, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
    g->ok = ok && encode_b(g, Bhi, Blo, K);
    if (g->ok) encode_c(g);
    return g->ok;
}

bool tc_gemm_plan_split_k(TcGemm *g, int M, int N, int K, const float *A, int a_mn, long long lda,
                          const float *Bhi, const float *Blo, const TcEpilogue &epi, int splits,
                          float *ws) {
    g->ok = false;
    const int kbl = (K + kBK - 1) / kBK;
    if (K % 4 || splits < 2 || !ws || ((uintptr_t)ws & 15) || N % 4) return false;
    const int kps = (kbl + splits - 1) / splits;
    splits = (kbl + kps - 1) / kps;
    if (splits < 2) return false;
    // the raw totals' epilogue: token-major [splits][M][N]
    TcEpilogue raw;
    raw.C = ws; raw.ldc_m = N; raw.ldc_n = 1; raw.c_bs = (long long)M * N;
    if (!plan_common(g, M, N, K, splits, 1, raw)) return false;
    g->a_mn = a_mn;
    g->gather = 0;
    g->box = 0;
    g->rows = 0;
    // every split reads the one A: a map of one batch entry
    bool ok;
    if (a_mn)
        ok = encode3d(&g->tmA, A, (uint64_t)M, (uint64_t)K, 1, (uint64_t)lda * 4, 0, kBM, kBK,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    else
        ok = encode3d(&g->tmA, A, (uint64_t)K, (uint64_t)M, 1, (uint64_t)lda * 4, 0, 32, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    g->ok = ok && encode_b(g, Bhi, Blo, K);
    if (!g->ok) return false;
    encode_c(g);
    if (g->tma_c != 2) {  // the raw totals leave by TMA stores of token-major boxes
        g->ok = false;
        return false;
    }
    g->kps = kps;
    g->ws = ws;
    g->ws_bs = (long long)M * N;
    g->epi = epi;  // applied by the reduction
    return true;
}

bool tc_gemm_split_k_shape(int M, int N, int K, int splits, int *splits_out, int *kps, int *tiles,
                           int *bn) {
    const int kbl = (K + kBK - 1) / kBK;
    if (K % 4 || splits < 2 || N % 4) return false;
    const int k = (kbl + splits - 1) / splits;
    splits = (kbl + k - 1) / k;
    if (splits < 2) return false;
    TcGemm h;
    TcEpilogue raw;
    if (!plan_common(&h, M, N, K, splits, 1, raw)) return false;
    *splits_out = splits;
    *kps = k;
    *tiles = h.tiles;
    *bn = h.bn;
    return true;
}

bool tc_gemm_plan_gather(TcGemm *g, int M, int N, int K, int batch, const TcGather &gg,
                         const float *Bhi, const float *Blo, const TcEpilogue &epi) {
    g->ok = false;
    // geometry limits of the gather: taps 1..8 (the -64 row sentinel must
    // stay below every tap), 1x1 only as a plain pointwise conv, int offsets
    if (!gg.x || gg.KS < 1 || gg.KS > 8 || gg.S < 1 || gg.P < 0 || gg.P >= gg.KS ||
        gg.H <= 0 || gg.W <= 0 || gg.OW <= 0 || gg.plane <= 0 || M % gg.OW != 0)
        return false;
    if (gg.KS == 1 && (gg.S != 1 || gg.P != 0 || gg.OW != gg.W)) return false;
    if (K % (gg.KS * gg.KS) != 0 || (long long)K / (gg.KS * gg.KS) * gg.plane >= (1LL << 31))
        return false;
    if (!plan_common(g, M, N, K, batch, 1, epi)) return false;
    g->a_mn = 0;  // the gathered tile is K-major
    g->gather = 1;
    g->box = 0;
    g->rows = 0;
    g->gg = gg;
    g->ok = encode_b(g, Bhi, Blo, (K + 3) / 4 * 4);
    if (g->ok) encode_c(g);
    return g->ok;
}

bool tc_gemm_plan_box(TcGemm *g, int N, int batch, const TcConvBox &cbin, const float *Bhi,
                      const float *Blo, const TcEpilogue &epi) {
    g->ok = false;
    TcConvBox b = cbin;
    if (!b.x || b.IC <= 0 || b.H <= 0 || b.W <= 0 || b.OH <= 0 || b.OW <= 0 || b.KS < 1 ||
        b.KS > 4 || b.P < 0 || b.P >= b.KS || (b.S != 1 && b.S != 2))
        return false;
    // TMA: 16-byte aligned base, rows, planes and pages
    if (((uintptr_t)b.x & 15) || b.W % 4 || (b.x_bs * 4) % 16 || (b.S == 2 && b.H % 2))
        return false;
    if ((long long)b.OH * b.OW >= (1LL << 31)) return false;
    tc_conv_box_blocks(b.IC, b.KS, &b.CB, &b.kbpb, &b.nbx);
    b.lcb = 2;
    while ((1 << b.lcb) < b.CB) b.lcb++;
    // window: columns from the 16-byte boundary at or below ox0*S - P (ox0
    // is a multiple of 32, so the remainder o is (-P) mod 4) through the
    // last tap of column 31
    b.o = ((-b.P) % 4 + 4) % 4;
    b.Wb = (b.o + 31 * b.S + b.KS + 3) / 4 * 4;
    b.tiles_x = (b.OW + 31) / 32;
    b.tiles_y = (b.OH + 3) / 4;
    const uint32_t raw_bytes = (uint32_t)b.Wb * 4 * (uint32_t)b.CB * 4;
    b.box_tx = raw_bytes;
    b.box_bytes = (raw_bytes + 1023) / 1024 * 1024;
    const int K = b.nbx * b.kbpb * 32;
    const long long row_tiles = (long long)b.tiles_x * b.tiles_y * batch;
    // two windows in flight at least, three when they fit beside the stages
    bool planned = false;
    for (int nb = 3; nb >= 2 && !planned; nb--) {
        b.nbox = nb;
        planned = plan_common(g, b.OH * b.OW, N, K, batch, 1, epi, 0, (uint32_t)nb * b.box_bytes,
                              row_tiles);
    }
    if (!planned) return false;
    g->m_tiles = b.tiles_x * b.tiles_y;
    g->tiles = g->m_tiles * g->n_tiles * batch;
    g->a_mn = 1;
    g->gather = 0;
    g->rows = 0;
    g->box = 1;
    g->cb = b;
    // the input as [B][C][H][W] (S = 1) or [B][C][2][H/2][W] with the row
    // parity as its own axis (S = 2: a window's rows are 2*oy + d for four
    // consecutive oy, i.e. four consecutive H/2 rows of one parity)
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t W = (cuuint64_t)b.W, H = (cuuint64_t)b.H, IC = (cuuint64_t)b.IC;
    CUresult rc;
    if (b.S == 1) {
        const cuuint64_t dims[4] = {W, H, IC, (cuuint64_t)batch};
        const cuuint64_t strides[3] = {W * 4, W * H * 4, (cuuint64_t)b.x_bs * 4};
        const cuuint32_t box[4] = {(cuuint32_t)b.Wb, 4, (cuuint32_t)b.CB, 1};
        const cuuint32_t es[4] = {1, 1, 1, 1};
        rc = fn(&g->tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(b.x), dims,
                strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[5] = {W, H / 2, 2, IC, (cuuint64_t)batch};
        const cuuint64_t strides[4] = {2 * W * 4, W * 4, W * H * 4, (cuuint64_t)b.x_bs * 4};
        const cuuint32_t box[5] = {(cuuint32_t)b.Wb, 4, 1, (cuuint32_t)b.CB, 1};
        const cuuint32_t es[5] = {1, 1, 1, 1, 1};
        rc = fn(&g->tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float *>(b.x), dims,
                strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (rc != CUDA_SUCCESS) return false;
    g->ok = encode_b(g, Bhi, Blo, K);
    if (g->ok) encode_c(g);
    return g->ok;
}

bool tc_gemm_plan_rows(TcGemm *g, int M, int N, int K, int batch, const float *x, long long plane,
                       long long x_bs, const float *Bhi, const float *Blo, const TcEpilogue &epi,
                       int planes) {
    g->ok = false;
    if (!x || plane < M || K % 4 || ((uintptr_t)x & 3) || (x_bs * 4) % 16 ||
        (batch > 1 && x_bs <= 0) || 4 * plane + 4 >= (1LL << 31))
        return false;
    if (!plan_common(g, M, N, K, batch, planes, epi, kRowsBytes)) return false;
    // the map starts at the 16-byte boundary at or below x; delta = the
    // floats between them
    const float *base = reinterpret_cast<const float *>((uintptr_t)x & ~(uintptr_t)15);
    g->rows_delta = (int)(x - base);
    g->rows_plane = plane;
    g->a_mn = 1;
    g->gather = 0;
    g->box = 0;
    g->rows = 1;
    // each page as [K / 4][4 * plane (+ the slack)]: row q of group g is
    // channel 4g + q; boxes of kRowsBox floats x 8 groups
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)(4 * plane + g->rows_delta), (cuuint64_t)(K / 4),
                                (cuuint64_t)batch};
    // (one page: any 16-byte multiple at least the page's length)
    const cuuint64_t page_bytes =
        x_bs > 0 ? (cuuint64_t)(x_bs * 4) : (cuuint64_t)(K * plane * 4 + 15) / 16 * 16;
    const cuuint64_t strides[2] = {(cuuint64_t)(16 * plane), page_bytes};
    const cuuint32_t box[3] = {kRowsBox, 8, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    if (fn(&g->tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides,
           box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    g->ok = encode_b(g, Bhi, Blo, K);
    if (g->ok) encode_c(g);
    return g->ok;
}

bool tc_gemm_set_bits_output(TcGemm *g, uint32_t *bits, long long words_per_n, long long bits_bs) {
    const TcEpilogue &e = g->epi;
    if (!g->ok || g->box || g->rows || g->gather || g->M % 32 || e.bias || e.res_mode ||
        e.act != ACT_NONE || e.alpha != 1.0f || !bits || words_per_n * 32 < g->M)
        return false;
    g->bits = 1;
    g->tma_c = 0;
    g->epi.C = reinterpret_cast<float *>(bits);
    g->epi.ldc_m = 0;
    g->epi.ldc_n = words_per_n;
    g->epi.c_bs = bits_bs;
    return true;
}

namespace {
// Split-K reduction: out(m, n) = epilogue(sum over splits in order of
// ws[z][m][n]) with the ops in the tensor-core epilogue's order (alpha,
// + bias, + residual mode 1, activation, + residual mode 2).
__global__ void splitk_reduce_kernel(const float *__restrict__ ws, long long ws_bs, int splits,
                                     int M, int N, TcEpilogue e) {
    pdl_begin();
    const long long n_all = (long long)M * N;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n_all;
         i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i - (long long)m * N);
        float x = ws[i];
        for (int z = 1; z < splits; z++) x = x + ws[z * ws_bs + i];
        if (e.alpha != 1.0f) x = x * e.alpha;
        if (e.bias) x = x + __ldg(e.bias + n);
        const float r = e.res_mode ? e.res[(long long)m * e.res_ldm + (long long)n * e.res_ldn] : 0.0f;
        if (e.res_mode == 1) x = x + r;
        x = act_apply(x, e.act);
        if (e.res_mode == 2) x = x + r;
        e.C[(long long)m * e.ldc_m + (long long)n * e.ldc_n] = x;
    }
}
}  // namespace

Status launch_tc_gemm(const TcGemm &g, cudaStream_t st) {
    if (!g.ok || g.epi.act < 0 || g.epi.act > 3) return ERR_SHAPE;
    // per device, once: the kernels' register count is checked and their
    // shared-memory limit raised (under a mutex: host threads may launch
    // their first GEMMs on a device together)
    static std::mutex mu;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return ERR_CUDA;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr[dev]) {
            const void *fns[14] = {
                (const void *)tc_gemm_kernel<0, kModeTile, true>,
                (const void *)tc_gemm_kernel<0, kModeBits>,
                (const void *)tc_gemm_kernel<0, kModeTile>, (const void *)tc_gemm_kernel<1, kModeTile>,
                (const void *)tc_gemm_kernel<2, kModeTile>, (const void *)tc_gemm_kernel<3, kModeTile>,
                (const void *)tc_gemm_kernel<0, kModeBox>,  (const void *)tc_gemm_kernel<1, kModeBox>,
                (const void *)tc_gemm_kernel<2, kModeBox>,  (const void *)tc_gemm_kernel<3, kModeBox>,
                (const void *)tc_gemm_kernel<0, kModeRows>, (const void *)tc_gemm_kernel<1, kModeRows>,
                (const void *)tc_gemm_kernel<2, kModeRows>, (const void *)tc_gemm_kernel<3, kModeRows>};
            for (const void *f : fns) {
                // the setmaxnreg split needs exactly kLaunchRegs per thread at launch
                cudaFuncAttributes fa;
                if (cudaFuncGetAttributes(&fa, f) != cudaSuccess || fa.numRegs != kLaunchRegs ||
                    cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemMax) != cudaSuccess) {
                    cudaGetLastError();
                    return ERR_CUDA;
                }
            }
            attr[dev] = true;
        }
    }
    Args a;
    a.M = g.M; a.N = g.N; a.K = g.K; a.batch = g.batch; a.planes = g.planes;
    a.a_mn = g.a_mn; a.bn = g.bn; a.stages = g.stages;
    a.m_tiles = g.m_tiles; a.n_tiles = g.n_tiles; a.tiles = g.tiles;
    a.gather = g.gather;
    a.tma_c = g.tma_c;
    a.gg = g.gg;
    a.box = g.box;
    a.cb = g.cb;
    if (!g.box) a.cb.nbox = 1;  // the window ring is unused
    a.rows = g.rows;
    a.rows_plane = g.rows_plane;
    a.rows_offmul = (int)(g.rows_plane & 3);
    a.rows_delta = g.rows_delta;
    a.kps = g.kps;
    const int splits = g.kps ? ((g.K + kBK - 1) / kBK + g.kps - 1) / g.kps : 1;
    if (g.kps) {
        // all splits run as batch entries; the raw totals go to the workspace
        a.batch = splits;
        a.tiles = g.m_tiles * g.n_tiles * splits;
    }
    const uint32_t b_bytes = 2u * 128u * (uint32_t)g.bn;
    if (g.box) {
        a.stage_bytes = b_bytes;
        a.tx_bytes = b_bytes;
    } else if (g.rows) {
        a.stage_bytes = kRowsBytes + b_bytes;
        a.tx_bytes = 4u * kRowsQBytes + b_bytes;
    } else {
        a.stage_bytes = kABytes + b_bytes;
        a.tx_bytes = (g.gather ? 0 : kABytes) + b_bytes;
    }
    a.staging_off = (uint32_t)g.stages * a.stage_bytes +
                    (g.box ? (uint32_t)g.cb.nbox * g.cb.box_bytes : 0u);
    if ((size_t)kCtrlBytes + a.staging_off + kStagingBytes > g.smem) return ERR_SHAPE;
    // FP32 accumulate, TF32 A and B, both K-major (A comes from TMEM), N, M
    a.idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(g.bn >> 3) << 17) |
              ((uint32_t)(kBM >> 4) << 24);
    a.epi = g.epi;
    if (g.kps) {
        TcEpilogue raw;
        raw.C = g.ws; raw.ldc_m = g.N; raw.ldc_n = 1; raw.c_bs = g.ws_bs;
        a.epi = raw;
    }
    int grid = sm_count();
    if (g.max_ctas > 0 && grid > g.max_ctas) grid = g.max_ctas;
    if (grid > a.tiles) grid = a.tiles;
    if (g.kps) {
        if (g.gather || g.box || g.rows || g.bits || g.batch < 1) return ERR_SHAPE;
        pdl_launch(tc_gemm_kernel<ACT_NONE, kModeTile>, grid, kThreads, g.smem, st, g.tmA, g.tmBhi,
                   g.tmBlo, g.tmC, a);
        const Status s0 = cuda_status();
        if (s0 != OK) return s0;
        const long long n_all = (long long)g.M * g.N;
        int rb = (int)((n_all + 255) / 256);
        if (rb > 8 * sm_count()) rb = 8 * sm_count();
        pdl_launch(splitk_reduce_kernel, rb, 256, 0, st, g.ws, g.ws_bs, splits, g.M, g.N, g.epi);
        return cuda_status();
    }
    if (g.bits) {
        // packed output: tile A, no epilogue ops (checked by the planner)
        pdl_launch(tc_gemm_kernel<ACT_NONE, kModeBits>, grid, kThreads, g.smem, st, g.tmA, g.tmBhi,
                   g.tmBlo, g.tmC, a);
        return cuda_status();
    }
    const int mode = g.box ? kModeBox : (g.rows ? kModeRows : kModeTile);
    // alternate-tile epilogue: tile-mode identity outputs in N tiles of at
    // most kHalfCols columns and at most two k-blocks, at least four tiles per
    // CTA (the forward's stage-0 Winograd GEMMs, 48 -> 48 channels)
    if (mode == kModeTile && g.epi.act == ACT_NONE && g.bn <= kHalfCols &&
        (g.K + kBK - 1) / kBK <= 2 && a.tiles >= 4 * grid) {
        pdl_launch(tc_gemm_kernel<ACT_NONE, kModeTile, true>, grid, kThreads, g.smem, st, g.tmA,
                   g.tmBhi, g.tmBlo, g.tmC, a);
        return cuda_status();
    }
    switch (mode * 4 + g.epi.act) {
#define PPDL_TC_CASE(M_, A_)                                                                  \
    case M_ * 4 + A_:                                                                      \
        pdl_launch(tc_gemm_kernel<A_, M_>, grid, kThreads, g.smem, st, g.tmA, g.tmBhi, g.tmBlo, g.tmC, \
                                                               a);                          \
        break;
        PPDL_TC_CASE(kModeTile, ACT_NONE)
        PPDL_TC_CASE(kModeTile, ACT_RELU)
        PPDL_TC_CASE(kModeTile, ACT_SILU)
        PPDL_TC_CASE(kModeTile, ACT_GELU)
        PPDL_TC_CASE(kModeBox, ACT_NONE)
        PPDL_TC_CASE(kModeBox, ACT_RELU)
        PPDL_TC_CASE(kModeBox, ACT_SILU)
        PPDL_TC_CASE(kModeBox, ACT_GELU)
        PPDL_TC_CASE(kModeRows, ACT_NONE)
        PPDL_TC_CASE(kModeRows, ACT_RELU)
        PPDL_TC_CASE(kModeRows, ACT_SILU)
        PPDL_TC_CASE(kModeRows, ACT_GELU)
#undef PPDL_TC_CASE
        default:
            return ERR_SHAPE;
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
