// dec.h — launchers of dec.cu (row-wise decoder kernels, GPU postprocess).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace ppdl {

// y = LayerNorm(x (+ r)) * g + b over rows of 256 (eps 1e-5)
Status launch_layernorm256(const float *x, const float *r, const float *g, const float *b,
                           float *y, long long rows, cudaStream_t st);
// the same, also writing y2 = y + q (rows of 256)
Status launch_layernorm256_add(const float *x, const float *r, const float *g, const float *b,
                               float *y, const float *q, float *y2, long long rows,
                               cudaStream_t st);
// softmax over rows of length L, in place
Status launch_softmax_rows(float *x, long long rows, int L, cudaStream_t st);

// Fused attention core (attn.cu): o = softmax(q k^T * scale) v per head of 32
// dims over token-major [B][T][ld] tensors (page stride bs), heads x 32 <= ld;
// o must not alias q, k or v.
Status launch_attention(const float *q, const float *k, const float *v, float *o, int T, int heads,
                        int ldqk, long long bsqk, int ldvo, long long bsvo, float scale, int B,
                        cudaStream_t st);
Status launch_add(const float *a, const float *b, float *y, long long n, cudaStream_t st);
// y = a + b over `pages` pages of n_per_page elements, b shared by all pages
Status launch_add_bcast(const float *a, const float *b, float *y, long long n_per_page,
                        int pages, cudaStream_t st);
Status launch_sigmoid(const float *x, float *y, long long n, cudaStream_t st);
// ref = sigmoid(delta + inverse_sigmoid(ref))
// rows of h [rows][256] -> delta = h w^T + b (w [4][256]); ref [rows][4]
// refined in place; qp [rows][nqp] = relu(ref wq^T + bq) (wq [nqp][4]) unless
// qp is null.  h, w, ref and wq 16-byte aligned.
Status launch_box_refine(const float *h, const float *w, const float *b, float *ref,
                         const float *wq, const float *bq, float *qp, int rows, int nqp,
                         cudaStream_t st);
// y[b][t][:] = x[b][t][:] * v[t]
Status launch_row_scale(const float *x, const float *v, float *y, long long rows_per_page, int D,
                        int B, cudaStream_t st);
// y[b][i][:] = x[b][idx[b][i]][:]
Status launch_gather_rows(const float *x, const int32_t *idx, float *y, int rows_in, int rows_out,
                          int D, int B, cudaStream_t st);
// reading-order ranks (rank: scratch of B * 300 words for the votes),
// top-300 selection, dets rows and (each if non-null)
// the thresholded, reordered masks of B pages as int32 [B][300][40000]
// (from mask_logits) and packed [B][300][1250] words (bit i of word w =
// pixel 32w + i; from the queries' packed masks mask_bits_q when given,
// else from mask_logits)
Status launch_postprocess(const float *logits, const float *boxes, const float *order,
                          const float *mask_logits, const uint32_t *mask_bits_q,
                          const int32_t *ori_hw, int32_t *rank, float *dets, int32_t *sel,
                          int32_t *masks, uint32_t *mask_bits, int B, cudaStream_t st);

// packed masks [B][300][1250] of mask logits [B][300][40000] (logit > 0)
Status launch_pack_mask_bits(const float *ml, uint32_t *bits, int B, cudaStream_t st);

// int32 masks [rows][40000] from packed masks [rows][1250]
Status launch_unpack_mask_bits(const uint32_t *bits, int32_t *masks, long long rows,
                               cudaStream_t st);

}  // namespace ppdl
