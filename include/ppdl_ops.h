/* ppdl_ops.h — operator-level C ABI of the B200 PP-DocLayoutV3 hot path.
 *
 * This is the drop-in replacement for the reference's tagged ggml custom-op
 * hooks (caojiachen1/ppdoclayout-ggml, patches/ggml-ppdl.patch:612-930):
 *
 *   reference                                      here
 *   bool ggml_cuda_compute_forward_ppdl(ctx, dst)  ppdl_op_launch(desc, stream)
 *        (patch:612-817, ppdl-ops.cuh:925)
 *   bool ggml_cuda_supports_ppdl_op(op)            ppdl_op_supported(desc)
 *        (patch:908-917, ppdl-ops.cuh:926)
 *
 * A ggml tensor is described by ppdl_tensor (device pointer + ggml ne[4],
 * contiguous) and a GGML_OP_CUSTOM node by ppdl_op_desc: the destination,
 * up to four sources (ggml dst->src[0..3]) and the node's int32
 * op_params[16], with op_params[12] = PPDL_MAGIC and op_params[13] = the op
 * id, exactly as the reference's graph builder tags them
 * (src/ppdoclayout.cpp:50-53).  op_params[14]/[15] carry the per-op
 * parameters with the reference's encodings (listed per id below).  A
 * ggml-side adapter fills a ppdl_op_desc from a ggml_tensor by copying
 * data, ne[0..3] and op_params[0..15] of the node and of its sources.
 *
 * Batching: the reference runs every op at batch 1.  Here the outermost ne
 * dimension that the reference leaves at 1 may hold several independent
 * pages (noted per op); all pages are processed in one launch.
 *
 * No function in this header allocates device memory; all run asynchronously
 * on the given stream (a cudaStream_t, NULL = legacy default stream).
 */
#ifndef PPDL_OPS_H
#define PPDL_OPS_H

#include <stdint.h>

#if defined(_WIN32)
#  define PPDL_OPS_API __declspec(dllexport)
#else
#  define PPDL_OPS_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PPDL_MAGIC 0x5050444C /* "PPDL", op_params[12] (src/ppdoclayout.cpp:51) */

/* Op ids, op_params[13] (patch:121-134). */
#define PPDL_OP_MASKBOX    1  /* src0 mask logits ne(40000,nq[,B]) -> dst ne(4,nq[,B]) inverse-sigmoid cxcywh */
#define PPDL_OP_MSDEF      2  /* src0 value ne(256,13125[,B]), src1 offsets ne(192,nq[,B]), src2 attn logits
                                 ne(96,nq[,B]), src3 ref ne(4,nq[,B]) -> dst ne(256,nq[,B]).
                                 op_params[14] = 1 selects the canonical form: src1 = sampling locations
                                 in [0,1] (same index order), src2 = softmax-normalised weights, no src3. */
#define PPDL_OP_CONV       3  /* K==1: src0 x ne(IW,IH,IC[,B]) CHW, src1 ".wr" ne(OC,IC,1), dst ne(IW,IH,OC[,B]);
                                 op_params[14] = K | pad<<8, [15] = 0 (CHW store).  The legacy K==3
                                 channel-last form ([15] = 1) is not provided (PPDL_ERR_UNSUPPORTED). */
#define PPDL_OP_CONVDIRECT 4  /* src0 x ne(IW,IH,IC[,B]), src1 ".wr" ne(OC,IC,K*K), src2 bias ne(OC) -> dst
                                 ne(OW,OH,OC[,B]); op_params[14] = K | S<<8 | PAD<<16 | ACT<<24,
                                 (K,S,PAD) in {(3,1,1),(3,2,1),(2,1,0),(1,1,0)}, ACT 0/1/2 = none/ReLU/SiLU */
#define PPDL_OP_BIASACT    5  /* dst = act(src0 + bias[plane]); src0/dst ne(W,H,C[,B]), src1 bias ne(C);
                                 op_params[14] = ACT */
#define PPDL_OP_COPY       6  /* contiguous f32 copy, n = nelements(dst) */
#define PPDL_OP_WG_INPUT   7  /* Winograd F(2,3) stages: not provided (PPDL_ERR_UNSUPPORTED); */
#define PPDL_OP_WG_OUTPUT  8  /*   F(4,3) below is the k3-s1-p1 path                            */
#define PPDL_OP_WG_MADD    9
#define PPDL_OP_WG4_INPUT  10 /* src0 padded x ne(IW_p,IH_p,IC[,B]) -> dst dt ne(T,IC,36[,B]);
                                 op_params[14] = T, [15] = TH (tile rows), TW = T/TH */
#define PPDL_OP_WG4_OUTPUT 11 /* src0 yt ne(T,OC,36[,B]), src1 bias ne(OC) -> dst ne(OW,OH,OC[,B]);
                                 op_params[14] = ACT, [15] = TW */
#define PPDL_OP_WG4_MADD   12 /* src0 dt ne(T,IC,36[,B]), src1 ".wg4" ne(OC,IC,36) -> dst yt ne(T,OC,36[,B]) */
#define PPDL_OP_TOPK       13 /* src0 class logits ne(nc,ntok[,B]) -> dst i32 ne(nq[,B]): tokens with the
                                 largest max-class logit, descending, ties to the lower index */

/* Status codes of ppdl_op_launch. */
#define PPDL_OK               0
#define PPDL_ERR_UNSUPPORTED  1  /* not a PPDL op or a form this build does not provide
                                    (the reference hook returns false) */
#define PPDL_ERR_SHAPE        2  /* shape / parameter violation (the reference aborts via GGML_ASSERT) */
#define PPDL_ERR_CUDA         3  /* the launch failed; cudaGetLastError() was consumed */

typedef struct {
    void *  data;   /* device pointer, f32 unless stated, contiguous */
    int64_t ne[4];  /* ggml element counts, ne[0] fastest */
} ppdl_tensor;

typedef struct {
    ppdl_tensor dst;
    ppdl_tensor src[4];
    int32_t     op_params[16];
} ppdl_op_desc;

/* Non-zero when desc is a tagged PPDL op that this build provides
   (ggml_cuda_supports_ppdl_op, patch:908-917). */
PPDL_OPS_API int ppdl_op_supported(const ppdl_op_desc * desc);

/* Enqueue the op on stream (ggml_cuda_compute_forward_ppdl, patch:612-817).
   Returns a PPDL_OK / PPDL_ERR_* status. */
PPDL_OPS_API int ppdl_op_launch(const ppdl_op_desc * desc, void * stream);

/* Extension (no counterpart in the reference, which calls cuBLAS SGEMM with
   TF32 off at patch:650-665 and 787-802): the FP32-faithful tensor-core GEMM
   that the 1x1 convs, the Winograd madd and the linears run on.
     C[z](m, n) = sum_k A[z](m, k) * B(n, k)
   A: a_m_major != 0 -> A(m, k) = A[z*a_bs + k*lda + m] (CHW activations);
      otherwise     A(m, k) = A[z*a_bs + m*lda + k] (row-major).
   B: [N][K] row-major, shared by all z.  C(m, n) at C[z*c_bs + m*ldc_m + n*ldc_n].
   b_split: caller-provided device workspace of 2*N*K floats for the TF32
   halves of B.  Requirements (TMA): b_split 16-byte aligned, a_bs and K
   multiples of 4; a K-major A also 16-byte aligned with lda a multiple of 4
   (an M-major A with another lda or alignment, e.g. CHW planes of 25 x 25
   pixels, is loaded as one TMA row per k).  Returns PPDL_OK /
   PPDL_ERR_SHAPE / PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_gemm_tf32x3(int M, int N, int K, int batch, const float * A,
                                  int a_m_major, long long lda, long long a_bs,
                                  const float * B, float * b_split, float * C,
                                  long long ldc_m, long long ldc_n, long long c_bs,
                                  void * stream);

/* Extension (no single counterpart: the reference's conv dispatcher,
   builder::conv at src/ppdoclayout.cpp:388-543, lowers k3-s2 and k2 convs
   to im2col + cuBLAS SGEMM, patch:845-906, and 1x1 convs to op 3): a direct
   convolution on the FP32-faithful tensor-core GEMM with no im2col buffer —
   the path the forward's k3-s2 / k2 convs take.
     y[z][oc][oy][ox] = act(bias[oc] + sum_{ic,kh,kw} weight[oc][ic][kh][kw]
                          * x[z][ic][oy*S + kh - P][ox*S + kw - P])
   with zero outside H x W (padding P at the top/left; the bottom/right
   padding follows from OH/OW, as for the stem's k2 convs with padding
   (0, 1); the last window of each axis must start inside the input,
   (OH-1)*S - P < H).  x: pages of dense [IC][H][W] at stride x_bs;
   y: pages of [OC][OH][OW] at stride y_bs; bias may be NULL; act 0/1/2/3 =
   none/ReLU/SiLU/GELU.  When W and x_bs are multiples of 4, x is 16-byte
   aligned, S is 1 or 2 (H even for 2) and K is 2..4, the A operand comes
   from TMA windows of the input (one per kernel row and 32 channels);
   otherwise the kernel's converter warps gather it.  b_split: device
   workspace of ppdl_conv2d_tf32x3_workspace(IC, OC, K) floats, 16-byte
   aligned.  K 1..8 with P < K; K = 1 needs S = 1, P = 0.
   Returns PPDL_OK / PPDL_ERR_SHAPE / PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_conv2d_tf32x3(const float * x, int batch, int IC, int H, int W,
                                    long long x_bs, const float * weight, const float * bias,
                                    int OC, int K, int S, int P, int OH, int OW, int act,
                                    float * b_split, float * y, long long y_bs, void * stream);

/* No counterpart in the reference (its stem convs are im2col + mul_mat,
   src/ppdoclayout.cpp:535-542): the direct FP32 convolution the forward uses
   for narrow convs — at most 128 products per output (IC*K*K) into at most
   32 channels, K 2..3, S 1..2 (the stem's 3 -> 32 k3-s2 and its 32 -> 16 /
   16 -> 32 k2 convs) — on the CUDA cores; the forward routes its first
   conv (27 products per output) here.  Same arguments and formula as
   ppdl_conv2d_tf32x3 minus b_split; each output sums over ic, kh, kw in that
   order in FP32.  Returns PPDL_OK, PPDL_ERR_UNSUPPORTED (outside the narrow
   shapes), PPDL_ERR_SHAPE or PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_conv2d_direct(const float * x, int batch, int IC, int H, int W,
                                    long long x_bs, const float * weight, const float * bias,
                                    int OC, int K, int S, int P, int OH, int OW, int act,
                                    float * y, long long y_bs, void * stream);

/* No counterpart in the reference (its attention is ggml_mul_mat(k, q) ->
   ggml_scale -> ggml_soft_max -> ggml_mul_mat with v, src/ppdoclayout.cpp:
   572-587): the fused attention core of the forward, per head of 32 dims,
     o[b][i][h*32 + d] = sum_j softmax_j(scale * q[b][i][h*32 ..] . k[b][j][h*32 ..]) v[b][j][h*32 + d]
   in FP32 on the CUDA cores.  q, k: rows of ldqk floats (page stride bsqk),
   v, o: rows of ldvo floats (page stride bsvo); heads * 32 <= ld; pointers
   16-byte aligned, ld and page strides multiples of 4.  T <= 320 (the
   decoder's 300 queries) keeps all keys on chip; longer sequences (AIFI's
   625 tokens) stream 64-key tiles.  Returns PPDL_OK, PPDL_ERR_SHAPE or
   PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_attention_f32(const float * q, const float * k, const float * v, float * o,
                                    int batch, int T, int heads, int ldqk, long long bsqk,
                                    int ldvo, long long bsvo, float scale, void * stream);

/* Floats of b_split that ppdl_conv2d_tf32x3 needs for these sizes (0 for
   non-positive sizes). */
PPDL_OPS_API long long ppdl_conv2d_tf32x3_workspace(int IC, int OC, int K);

/* Extension (replaces the node chain pad_ext -> op 10 -> op 12 -> op 11 of
   the reference's k3-s1-p1 convs, src/ppdoclayout.cpp:430-464 and
   patch:496-610, 778-812): one 3x3, stride-1, padding-1 convolution by
   Winograd F(4,3) exactly as the forward runs it — filter transform with the
   reference's G (src/ppdoclayout.cpp:313-320), input transform with the
   padding fused, the 36-plane product on the 3xTF32 tensor-core GEMM, output
   transform with bias and activation.
     y[z][oc][oy][ox] = act(bias[oc] + sum_{ic,kh,kw} weight[oc][ic][kh][kw]
                          * x[z][ic][oy + kh - 1][ox + kw - 1])
   x: pages of dense [IC][H][W] at stride x_bs; y: pages of [OC][H][W] at
   stride y_bs; bias may be NULL; act 0/1/2/3 = none/ReLU/SiLU/GELU.  IC a
   multiple of 4.  work: device workspace of
   ppdl_conv3x3_wg4_workspace(batch, IC, OC, H, W) floats, 16-byte aligned
   (transformed filter and its TF32 halves, the 36 input and output planes).
   Returns PPDL_OK / PPDL_ERR_SHAPE / PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_conv3x3_wg4_tf32x3(const float * x, int batch, int IC, int H, int W,
                                         long long x_bs, const float * weight,
                                         const float * bias, int OC, int act, float * work,
                                         float * y, long long y_bs, void * stream);

/* Floats of work that ppdl_conv3x3_wg4_tf32x3 needs (0 for non-positive sizes). */
PPDL_OPS_API long long ppdl_conv3x3_wg4_workspace(int batch, int IC, int OC, int H, int W);

/* ppdl_conv3x3_wg4_tf32x3 in two parts, for weights used many times (the
   reference transforms its filters once at load, repack_convs at
   src/ppdoclayout.cpp:251-346): _prepare writes the transformed filter and
   its TF32 halves into the head of work; _run then convolves with them
   (same arguments minus weight).  work as for ppdl_conv3x3_wg4_tf32x3, with
   batch, H and W of the largest _run. */
PPDL_OPS_API int ppdl_conv3x3_wg4_prepare(const float * weight, int IC, int OC, float * work,
                                          void * stream);
PPDL_OPS_API int ppdl_conv3x3_wg4_run(const float * x, int batch, int IC, int H, int W,
                                      long long x_bs, const float * bias, int OC, int act,
                                      float * work, float * y, long long y_bs, void * stream);

/* ppdl_gemm_tf32x3 in two parts, for a B used many times: ppdl_tf32_split
   writes the TF32 halves of the n floats of B into b_split (2n floats: hi,
   then lo); ppdl_gemm_tf32x3_presplit multiplies with them (arguments as
   ppdl_gemm_tf32x3, b_split read only). */
PPDL_OPS_API int ppdl_tf32_split(const float * B, long long n, float * b_split, void * stream);
PPDL_OPS_API int ppdl_gemm_tf32x3_presplit(int M, int N, int K, int batch, const float * A,
                                           int a_m_major, long long lda, long long a_bs,
                                           const float * b_split, float * C,
                                           long long ldc_m, long long ldc_n, long long c_bs,
                                           void * stream);

/* Extension (the reference's depthwise conv is ggml_conv_2d_dw_direct,
   src/ppdoclayout.cpp:400-404, a ggml op rather than a tagged PPDL op):
   the depthwise conv of the backbone's downsampling and light blocks.
     y[z][c][oy][ox] = act(sum_{kh,kw} weight[c][kh][kw]
                           * x[z][c][oy*S + kh - P][ox*S + kw - P] + bias[c])
   in FP32, taps accumulated by fma in (kh, kw) order, zero outside H x W,
   OH = (H + 2P - K) / S + 1 (same for OW).  x: pages of [C][H][W] at stride
   x_bs; y: pages of [C][OH][OW] at stride y_bs; bias may be NULL; act
   0/1/2/3 = none/ReLU/SiLU/GELU.  K 3 or 5, S 1 or 2 (else
   PPDL_ERR_UNSUPPORTED), 0 <= P < K.  Returns PPDL_OK / PPDL_ERR_SHAPE /
   PPDL_ERR_UNSUPPORTED / PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_depthwise_conv2d(const float * x, int batch, int C, int H, int W,
                                       long long x_bs, const float * weight, const float * bias,
                                       int K, int S, int P, int act, float * y, long long y_bs,
                                       void * stream);

/* No counterpart in the reference.  ppdl_gemm_tf32x3 for callers that
   cannot allocate device memory — e.g. a ggml custom-op hook, which runs
   inside ggml's graph compute where ggml's allocator owns every buffer and
   the node sees only its own tensors.  Same arguments and result as
   ppdl_gemm_tf32x3 minus b_split: the TF32 halves of B go to a workspace
   that is a file-scope device array of this library (16 MiB on every device
   that loads it, kept until the process exits), so N*K may be at most
   2097152 (larger -> PPDL_ERR_SHAPE).  Nothing is allocated.  The first call
   on a device resolves the array's address for that device; make it before
   any stream capture on the device.  All calls share the array: calls whose
   GPU work overlaps in time race on it and must be serialised by the caller. */
PPDL_OPS_API int ppdl_gemm_tf32x3_static(int M, int N, int K, int batch, const float * A,
                                         int a_m_major, long long lda, long long a_bs,
                                         const float * B, float * C,
                                         long long ldc_m, long long ldc_n, long long c_bs,
                                         void * stream);

/* No counterpart in the reference.  ppdl_gemm_tf32x3_presplit for a K-major
   A (rows of lda floats) and a token-major C [M][N], with K split into
   `splits` ranges of 32-wide k-blocks: one launch computes every range's
   totals into ws (splits * M * N floats, 16-byte aligned), a second sums
   them in range order and applies C = act(total + bias) + res (bias and
   res may be NULL; res [M][N]; act 0/1/2/3 = none/ReLU/SiLU/GELU) — the
   forward's path for its long-K linears (K = 2048).  Returns PPDL_OK,
   PPDL_ERR_SHAPE or PPDL_ERR_CUDA. */
PPDL_OPS_API int ppdl_gemm_tf32x3_split_k(int M, int N, int K, const float * A, long long lda,
                                          const float * b_split, const float * bias,
                                          const float * res, int act, int splits, float * ws,
                                          float * C, void * stream);

/* Human-readable text of the last error of ppdl_op_launch on this thread. */
PPDL_OPS_API const char * ppdl_op_last_error(void);

/* Extension (the reference aborts through GGML_ASSERT and has no device-side
   error state): the tensor-core kernels bound every wait inside the kernel
   (about 2 s); a wait that gives up leaves its output unwritten, and the
   kernel raises a device-wide flag.  After synchronising the stream of the
   launches in question, this returns 1 if the flag was raised since the last
   call (and clears it), else 0.  The flag is per device (the current one). */
PPDL_OPS_API int ppdl_op_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* PPDL_OPS_H */
