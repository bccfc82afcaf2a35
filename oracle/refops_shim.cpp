// refops_shim.cpp — builds the reference's own CPU custom ops as a checker.
//
// TEST INFRASTRUCTURE ONLY (see ppdl_oracle.c).  oracle/Makefile extracts
// the operator bodies from the reference sources at build time
// (src/ppdoclayout.cpp:29-44 model constants and :61-198 op_topk300,
// op_mask_box, op_msdeform) into oracle/_ref/refops_body.inc, which is never
// committed.  This file supplies the one ggml type those bodies touch
// (ggml_tensor: data and src[] only) and exports plain C entry points so the
// tests and bench.py can run the unmodified reference arithmetic.
#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

struct ggml_tensor {
    void * data = nullptr;
    ggml_tensor * src[4] = {nullptr, nullptr, nullptr, nullptr};
};

#include "refops_body.inc"

namespace {
// The reference runs its ops on ggml's CPU threads as op(dst, ith, nth); the
// same striding is reproduced with std::thread.
template <typename F>
void run_threads(F fn, ggml_tensor * dst, int nth) {
    if (nth <= 1) { fn(dst, 0, 1, nullptr); return; }
    std::vector<std::thread> ts;
    for (int i = 0; i < nth; i++) ts.emplace_back([=] { fn(dst, i, nth, nullptr); });
    for (auto & t : ts) t.join();
}
}  // namespace

extern "C" {

// value [13125][256], off [300][192], awr [300][96], ref [300][4] -> out [300][256]
void ref_msdeform(const float * val, const float * off, const float * awr, const float * ref,
                  float * out, int nth) {
    ggml_tensor s0, s1, s2, s3, d;
    s0.data = (void *) val; s1.data = (void *) off; s2.data = (void *) awr; s3.data = (void *) ref;
    d.data = out;
    d.src[0] = &s0; d.src[1] = &s1; d.src[2] = &s2; d.src[3] = &s3;
    run_threads(op_msdeform, &d, nth);
}

// mask logits [300][40000] -> out [300][4]
void ref_mask_box(const float * ml, float * out, int nth) {
    ggml_tensor s0, d;
    s0.data = (void *) ml; d.data = out; d.src[0] = &s0;
    run_threads(op_mask_box, &d, nth);
}

// class logits [13125][25] -> out [300] i32
void ref_topk300(const float * lg, int32_t * out) {
    ggml_tensor s0, d;
    s0.data = (void *) lg; d.data = out; d.src[0] = &s0;
    op_topk300(&d, 0, 1, nullptr);
}

}  // extern "C"
