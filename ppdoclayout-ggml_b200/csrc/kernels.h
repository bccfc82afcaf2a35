// kernels.h — internal launchers of the B200 PP-DocLayoutV3 kernels.
//
// Every launcher enqueues on `stream`, allocates nothing and returns a
// ppdl::Status.  Pointers are device pointers; "B" is the number of pages.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace ppdl {

// ---- decoder / selection ops ------------------------------------------------
// MSDeformAttn.  In-model: p1 = offsets [B*nq][192], p2 = logits [B*nq][96],
// ref [B*nq][4].  Canonical: p1 = locations, p2 = softmax weights, ref unused.
// val [B][13125][ldv] (256 channels used), out [B*nq][256].  Rows of p1 /
// p2 lie ld1 / ld2 floats apart (192 / 96 when dense; the model's fused
// projection writes both into one [B*nq][288] buffer); value rows ldv
// floats apart (256 when dense; the six decoder layers' projections share
// one [B][13125][1536] buffer).
Status launch_msda(const float *val, const float *p1, const float *p2, const float *ref,
                   float *out, int nq, int batch, bool canon, int ld1, int ld2,
                   cudaStream_t stream, int ldv = 256);

// mask logits [rows][40000] -> [rows][4]
Status launch_mask_box(const float *ml, float *out, int rows, cudaStream_t stream);
// the same on packed masks [rows][1250] (bit p & 31 of word p >> 5 = pixel p)
Status launch_mask_box_bits(const uint32_t *bits, float *out, int rows, cudaStream_t stream);

// class logits [B][ntok][nc] -> [B][nq] token indices
Status launch_topk(const float *lg, int32_t *out, int ntok, int nc, int nq, int batch,
                   cudaStream_t stream);

// ---- elementwise ----------------------------------------------------------------
// y = act(x + bias[(i / plane) % C]) over n elements; bias may be null.
Status launch_bias_act(const float *x, const float *bias, float *y, long long n,
                       long long plane, int C, int act, cudaStream_t stream);

Status launch_copy(const float *x, float *y, long long n, cudaStream_t stream);

}  // namespace ppdl
