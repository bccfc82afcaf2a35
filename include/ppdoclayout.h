/* ppdoclayout.h — public C ABI of the B200 PP-DocLayoutV3 hot path.
 *
 * Drop-in for the reference's C API (caojiachen1/ppdoclayout-ggml,
 * include/ppdoclayout.h:1-69): the same constants, result struct and
 * functions with the same argument meaning, ownership and error codes.
 * Additions for batched / multi-GPU use are marked "extension"; the
 * reference functions keep batch 1.
 *
 * Backend: only PPDL_BACKEND_CUDA is provided (a B200, sm_100a).  There is no
 * CPU path: ppdl_init with PPDL_BACKEND_CPU returns NULL with a message.
 */
#ifndef PPDOCLAYOUT_H
#define PPDOCLAYOUT_H

#include <stdint.h>

#if defined(_WIN32)
#  define PPDL_API __declspec(dllexport)
#else
#  define PPDL_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PPDL_IMG_SIZE   800  /* fixed input resolution (square)          */
#define PPDL_NUM_DETS   300  /* rows in every result                     */
#define PPDL_DET_FIELDS 7    /* label, score, x1, y1, x2, y2, order       */
#define PPDL_MASK_HW    200  /* per-detection mask is 200 x 200           */

#define PPDL_BACKEND_CPU  0
#define PPDL_BACKEND_CUDA 1

typedef struct ppdl_ctx ppdl_ctx;

/* reference include/ppdoclayout.h:31-38.  Pointers stay valid until the next
   ppdl_infer / ppdl_infer_batch or ppdl_free on the same ctx. */
typedef struct {
    const float   * dets;     /* [300 * 7], score-descending                */
    int32_t         num_dets; /* always 300                                  */
    const int32_t * masks;    /* [300 * 200 * 200] 0/1, row i <-> dets row i */
    double          infer_ms; /* device time of the forward of this call     */
} ppdl_result;

/* reference :40-42 (src/ppdoclayout.cpp:1148-1150).  Loads an F32 GGUF
   (BN folded, the reference converter's layout) onto the current CUDA device
   and prepares the batch-1 forward.  NULL on failure (message on stderr). */
PPDL_API ppdl_ctx * ppdl_init(const char * model_path, int backend);

/* reference :44-45 (src/ppdoclayout.cpp:1082-1146): as ppdl_init, keeping the
   intermediate tensors of the last call available to ppdl_dump. */
PPDL_API ppdl_ctx * ppdl_init_ex(const char * model_path, int backend, int enable_dumps);

/* extension: explicit device ordinal and batch capacity (pages per forward,
   1..64).  device < 0 keeps the current device. */
PPDL_API ppdl_ctx * ppdl_init_dev(const char * model_path, int backend, int device,
                                  int max_batch, int enable_dumps);

/* reference :47-52 (src/ppdoclayout.cpp:1152-1191).  image_chw: float32 CHW
   3 x 800 x 800, RGB, /255.  Returns 0 on success, 1 on bad arguments (null
   pointer, ori_h or ori_w <= 0), 2 on a compute failure. */
PPDL_API int ppdl_infer(ppdl_ctx * ctx, const float * image_chw,
                        int ori_h, int ori_w, ppdl_result * result);

/* extension: n pages (n <= max_batch) from host memory, images back to back;
   ori_hw holds n (ori_h, ori_w) pairs; results[n] are filled as by ppdl_infer
   and share the ctx-owned buffers.  Same return codes. */
PPDL_API int ppdl_infer_batch(ppdl_ctx * ctx, const float * images_chw, int n,
                              const int32_t * ori_hw, ppdl_result * results);

/* extension: n pages already in device memory (d_images, n x 3 x 800 x 800
   f32), ori_hw in host memory.  Enqueues the forward and the postprocess on
   the ctx stream and returns without copying results back; the device
   outputs are then read with ppdl_device_outputs after a stream sync
   (ppdl_sync).  Same return codes. */
PPDL_API int ppdl_infer_device(ppdl_ctx * ctx, const float * d_images, int n,
                               const int32_t * ori_hw);

/* extension: device pointers of the last ppdl_infer_device outputs:
   dets [n][300][7] f32 and masks [n][300][40000] i32. */
PPDL_API int ppdl_device_outputs(ppdl_ctx * ctx, const float ** d_dets,
                                 const int32_t ** d_masks);

/* extension: waits for the ctx stream; returns 2 if the GPU work failed. */
PPDL_API int ppdl_sync(ppdl_ctx * ctx);

/* extension: as ppdl_infer_device, but the masks stay packed (the forward's
   own mask output, 1 bit per pixel, see ppdl_result_bits); they are read with
   ppdl_device_mask_bits after ppdl_sync.  ppdl_device_outputs' int32 masks
   are not refreshed by this call. */
PPDL_API int ppdl_infer_device_bits(ppdl_ctx * ctx, const float * d_images, int n,
                                    const int32_t * ori_hw);

/* extension: device pointer of the packed masks of the last forward,
   [n][300][1250] 32-bit words (layout as ppdl_result_bits.mask_bits). */
PPDL_API int ppdl_device_mask_bits(ppdl_ctx * ctx, const uint32_t ** d_bits);

/* extension (no counterpart in the reference, whose result masks are
   300 x 200 x 200 int32 per page, src/ppdoclayout.cpp:985-990): one page's
   result with the masks packed 1 bit per pixel — 1.5 MB instead of 48 MB.
   Pixel p = y * 200 + x of detection i is bit (p & 31) of
   mask_bits[i * 1250 + (p >> 5)]; ppdl_expand_mask_bits restores the int32
   form.  dets and infer_ms as in ppdl_result. */
typedef struct {
    const float *    dets;       /* 300 x 7, score-descending */
    int32_t          num_dets;   /* 300 */
    const uint32_t * mask_bits;  /* 300 x 1250 words */
    double           infer_ms;   /* device time of the forward */
} ppdl_result_bits;

/* extension: pipelined batches.  Enqueues n pages (host memory; pinned
   memory lets the copy overlap the previous batch's forward) and returns at
   once with *ticket.  The copy in, the forward and the copy out of the
   results (dets + packed masks) run on three streams, so up to two batches
   are in flight: batch t's copies overlap batch t-1's forward.  The pages
   must stay unchanged until ppdl_wait_batch(ticket) returns.  Results of
   ticket t live in ctx-owned pinned buffers until ticket t + 2 is submitted
   (a submission waits for ticket t - 2's copy-out first).  The first call
   allocates the pipeline's buffers (two device staging copies of the pages
   and outputs, two pinned result slots).  Returns 0, 1 (bad args), 2
   (failure). */
PPDL_API int ppdl_submit_batch(ppdl_ctx * ctx, const float * images_chw, int n,
                               const int32_t * ori_hw, int64_t * ticket);

/* extension: waits for the batch of ticket and fills results[n] (n of that
   submission).  Returns 0, 1 (unknown or overwritten ticket), 2 (failure). */
PPDL_API int ppdl_wait_batch(ppdl_ctx * ctx, int64_t ticket, ppdl_result_bits * results);

/* extension: host expansion of packed masks into the reference's int32
   format: masks[i * 40000 + p] = bit p of detection i, for n_dets rows. */
PPDL_API void ppdl_expand_mask_bits(const uint32_t * mask_bits, int32_t * masks, int n_dets);

/* extension: the CUDA stream (cudaStream_t) the ctx enqueues on, for callers
   that time or order their own work against it. */
PPDL_API void * ppdl_stream(ppdl_ctx * ctx);

/* extension: per-step device profile — the counterpart of the reference's
   PPDL_PROFILE phase profile (src/ppdoclayout.cpp:995-1050).  Runs the
   forward of the n pages of the last call once more with a CUDA event after
   every step — captured into a CUDA graph and replayed, so the times are
   device time without host launch gaps (eagerly if the capture fails) — and
   fills up to max entries.  The steps run one after another here, so each
   time is the step alone.  Returns the number of steps written, or -1. */
#define PPDL_STEP_OTHER         0
#define PPDL_STEP_GEMM_1X1      1   /* 1x1 conv GEMM                     */
#define PPDL_STEP_WG_MADD       2   /* Winograd 36-plane GEMM            */
#define PPDL_STEP_GEMM_IMPLICIT 3   /* k3-s2 / k2 implicit-GEMM conv     */
#define PPDL_STEP_GEMM_LINEAR   4   /* linears and mask GEMMs            */
#define PPDL_STEP_WG_INPUT      5   /* Winograd input transform          */
#define PPDL_STEP_WG_OUTPUT     6   /* Winograd output transform         */
#define PPDL_STEP_DWCONV        7   /* depthwise conv                    */
#define PPDL_STEP_MSDA          8   /* MSDeformAttn                      */
#define PPDL_STEP_MASKBOX       9   /* mask -> box                       */
#define PPDL_STEP_TOPK          10  /* top-300 selection                 */
#define PPDL_STEP_POSTPROCESS   11  /* order votes, top-300, masks       */
#define PPDL_STEP_GLUE          12  /* LN, softmax, add, interp, pool... */
#define PPDL_STEP_IM2COL        13  /* conv operand packing for the GEMM */
#define PPDL_STEP_ATTENTION     14  /* q-k products on SIMT FP32: fused
                                       softmax(q k^T) v, reading-order scores */
#define PPDL_STEP_CONV_DIRECT   15  /* narrow convs on SIMT FP32 (the stem's
                                       first three: IC*K*K <= 128, OC <= 32) */
typedef struct {
    char    name[48];
    int32_t kind;   /* PPDL_STEP_* */
    float   ms;     /* device time of the step for all n pages */
    double  flops;  /* algorithmic FLOPs per page */
    double  bytes;  /* algorithmic bytes per page */
} ppdl_step_stat;
PPDL_API int ppdl_profile_steps(ppdl_ctx * ctx, int n, ppdl_step_stat * out, int max);

/* extension: timeline of the forward as it runs — its steps on their lanes
   (CUDA streams inside the captured forward: lane 0 the decoder chain, 1 the
   value projections, 2 projections beside the chain), with an event after
   every step on its own lane.  end_ms[i] = end of step i (the order of
   ppdl_profile_steps) from the start of the forward, lane[i] its lane.
   Returns the number of steps written, or -1 (also when the capture fails). */
PPDL_API int ppdl_profile_timeline(ppdl_ctx * ctx, int n, float * end_ms, int32_t * lane,
                                   int max);

/* reference :54-56 (src/ppdoclayout.cpp:1193-1213): writes the intermediate
   tensors of page 0 of the last call plus shapes.txt.  Non-zero when dumps
   were not enabled or nothing was computed yet. */
PPDL_API int ppdl_dump(ppdl_ctx * ctx, const char * dir);

/* reference :58-62 (src/ppdoclayout.cpp:1215-1223): <pfx>logits.bin (300x25),
   <pfx>boxes.bin (300x4 sigmoid cxcywh), <pfx>order.bin (300x300,
   [j + 300 i] = q_i . k_j / 8), <pfx>sel.bin (300 i32 flat q*25+c) of page 0
   of the last call.  Extension: <pfx>topk.bin (300 i32), the encoder tokens
   chosen as decoder queries, in query order (op_topk300's output). */
PPDL_API int ppdl_dump_raw(ppdl_ctx * ctx, const char * pfx);

/* reference :64 (src/ppdoclayout.cpp:1225-1236) */
PPDL_API void ppdl_free(ppdl_ctx * ctx);

#ifdef __cplusplus
}
#endif

#endif /* PPDOCLAYOUT_H */
