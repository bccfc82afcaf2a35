// select.cuh — the nq largest of n unique 64-bit keys held in shared memory,
// by one block: the top-300 query selection (op_topk300,
// src/ppdoclayout.cpp:73-96) and the postprocess's top-300 of the 7500 class
// scores (src/ppdoclayout.cpp:927-993) both order by such keys (value bits
// << 32 | ~index, so ties go to the lower index and every key is unique).
//
// A radix select finds the nq-th largest key: eight passes over the keys,
// each building a 256-bin histogram of the next byte among the keys that
// match the prefix found so far (lanes of a warp with the same bin add once),
// and one scan of the bins from the top; the passes stop early once every
// key of the chosen bin is needed (the threshold is then the bin's lowest
// possible key).  The nq keys >= it are compacted and bitonic-sorted
// descending in a 512-entry buffer.
#pragma once

#include <cstdint>

namespace ppdl {

constexpr int kSelectMax = 512;  // largest nq handled

// order-preserving bits of a float (-0 folded to +0, which the reference's
// value comparison ties with it) << 32 | ~index
__device__ __forceinline__ unsigned long long select_key(float v, unsigned index) {
    if (v == 0.0f) v = 0.0f;
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - index);
}
__device__ __forceinline__ unsigned select_index(unsigned long long key) {
    return 0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull);
}

// Called by all threads of the block (blockDim.x a multiple of 32) after the
// keys are written and synchronised; on return sel[0 .. nq) holds the nq
// largest keys, descending, visible to the whole block.  n >= nq, nq <= 512.
__device__ __forceinline__ void block_select_top(const unsigned long long *keys, int n, int nq,
                                                 unsigned long long *sel) {
    __shared__ unsigned s_hist[256];
    __shared__ unsigned long long s_prefix, s_mask;
    __shared__ unsigned s_need, s_cnt, s_done;
    const int nt = blockDim.x, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_prefix = 0ull;
        s_mask = 0ull;
        s_need = (unsigned)nq;
        s_cnt = 0;
        s_done = 0;
    }
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int b = threadIdx.x; b < 256; b += nt) s_hist[b] = 0;
        __syncthreads();
        const unsigned long long prefix = s_prefix, mask = s_mask;
        for (int q0 = 0; q0 < n; q0 += nt) {
            const int q = q0 + threadIdx.x;
            const bool in = q < n && (keys[q] & mask) == prefix;
            const unsigned bin = in ? (unsigned)(keys[q] >> shift) & 255u : 256u;
            const unsigned same = __match_any_sync(0xffffffffu, bin);
            if (in && lane == __ffs(same) - 1) atomicAdd(&s_hist[bin], __popc(same));
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            // the bin holding the need-th largest of the matching keys
            unsigned above = 0, need = s_need;
            int b = 255;
            for (; b > 0; b--) {
                if (above + s_hist[b] >= need) break;
                above += s_hist[b];
            }
            s_prefix = prefix | ((unsigned long long)b << shift);
            s_mask = mask | (255ull << shift);
            s_need = need - above;
            // every matching key of bin b is needed: the bin's smallest
            // possible key (lower bytes zero) already separates the nq largest
            s_done = s_hist[b] == need - above;
        }
        __syncthreads();
        if (s_done) break;
    }
    const unsigned long long thr = s_prefix;  // the nq-th largest key, or a bound just below it
    for (int q = threadIdx.x; q < n; q += nt)
        if (keys[q] >= thr) sel[atomicAdd(&s_cnt, 1u)] = keys[q];
    for (int i = nq + threadIdx.x; i < kSelectMax; i += nt) sel[i] = 0ull;
    __syncthreads();
    for (int k = 2; k <= kSelectMax; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < kSelectMax; i += nt) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = sel[i], c = sel[ixj];
                    if (((i & k) == 0) ? (a < c) : (a > c)) {
                        sel[i] = c;
                        sel[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

}  // namespace ppdl
