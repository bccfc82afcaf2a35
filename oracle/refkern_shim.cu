// refkern_shim.cu — the reference's own CUDA kernels for MSDeformAttn and
// mask->box, compiled for sm_100a as the same-box bar.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile extracts the kernel bodies
// from the reference's ggml patch at build time (patches/ggml-ppdl.patch
// lines 197-312: the model constants, ppdl_invsig, ppdl_mask_box_kernel and
// ppdl_msdeform_kernel, with the patch's leading '+' removed) into
// oracle/_ref/refkern_body.inc, which is never committed.  This file adds
// only launch wrappers with the reference's launch shapes (patch:618-631:
// one block per query, 256 threads; batch 1 per launch, so a batch of pages
// is one launch per page), so bench.py can time the unmodified reference
// kernels beside this build's on the same B200.  The product library never
// loads it.
#include <cuda_runtime.h>

#include <cmath>

#include "refkern_body.inc"

extern "C" int refkern_msdeform(const float *val, const float *off, const float *awr,
                                const float *ref, float *out, int nq, int pages,
                                void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    for (int b = 0; b < pages; b++)
        ppdl_msdeform_kernel<<<nq, PPDL_NH * 32, 0, st>>>(
            val + (size_t)b * 13125 * PPDL_DM, off + (size_t)b * nq * 192,
            awr + (size_t)b * nq * 96, ref + (size_t)b * nq * 4, out + (size_t)b * nq * PPDL_DM,
            nq);
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

extern "C" int refkern_mask_box(const float *ml, float *out, int rows, void *stream) {
    ppdl_mask_box_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(ml, out, rows);
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
