// common.cuh — shared definitions of the B200 PP-DocLayoutV3 kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

namespace ppdl {

// Model constants (reference src/ppdoclayout.cpp:31-44).
constexpr int kImg = 800;
constexpr int kNQ = 300;
constexpr int kNC = 25;
constexpr int kDM = 256;
constexpr int kNH = 8;
constexpr int kHD = 32;
constexpr int kNLvl = 3;
constexpr int kNPts = 4;
constexpr int kMaskHW = 200;
constexpr int kMaskPix = kMaskHW * kMaskHW;
constexpr int kMaskWords = kMaskPix / 32;  // packed mask: 1250 32-bit words
constexpr int kNTok = 13125;

enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_SILU = 2, ACT_GELU = 3 };

// Round-to-nearest a / d for d = 1 + exp(-a) (d in [1, 2^128) or +inf), with
// no branch, so that a loop over several values keeps them all in flight.
// Markstein's method (P. Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Develop. 34(1), 1990):
// an approximate reciprocal y of d refined by one Newton step
// y += y (1 - d y), the quotient q = a y, then one correction with the exact
// remainder, q += y (a - d q), both residuals taken with a single rounding
// by fma.  Denominators above 2^64 scale a and d by 2^-64 first (exact), so
// that 1/d stays a normal number; d = +inf gives a signed zero, as a / inf.
__device__ __forceinline__ float silu_quotient(float a, float d) {
    const bool big = d > 0x1p64f;
    const float s = big ? 0x1p-64f : 1.0f;
    const float as = a * s, ds = d * s;
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(ds));
    y = __fmaf_rn(__fmaf_rn(-ds, y, 1.0f), y, y);
    float q = __fmul_rn(as, y);
    q = __fmaf_rn(__fmaf_rn(-ds, q, as), y, q);
    if (d == 1.0f || a == 0.0f) q = a;  // exact quotients (a zero keeps its sign)
    if (d == INFINITY) q = copysignf(0.0f, a);
    return q;
}

// Activation exactly as the reference evaluates it: ReLU fmaxf, SiLU
// x / (1 + exp(-x)) (patch:383-386, 426-430; ggml_silu; the quotient
// correctly rounded by silu_quotient), GELU with erf (ggml_gelu_erf,
// src/ppdoclayout.cpp:687).
__device__ __forceinline__ float act_apply(float v, int act) {
    if (act == ACT_RELU) return fmaxf(v, 0.0f);
    if (act == ACT_SILU) return silu_quotient(v, __fadd_rn(1.0f, expf(-v)));
    if (act == ACT_GELU) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
    return v;
}

// Status returned by the internal launchers.
enum Status : int { OK = 0, ERR_UNSUPPORTED = 1, ERR_SHAPE = 2, ERR_CUDA = 3 };

// Raise kernel fn's dynamic shared-memory limit to `bytes` on the current
// device, once per process, kernel and device (host threads may make their
// first launches together, so the record is kept under a mutex).
inline bool smem_attr_once(const void *fn, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({fn, dev})) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess)
        return false;
    done.insert({fn, dev});
    return true;
}

// ---- programmatic dependent launch -------------------------------------------
// Every kernel of the library starts with pdl_begin(): it waits until the
// grids it depends on in its stream have completed and their writes are
// visible (at once for a launch without the attribute).  Launched through
// pdl_launch, a kernel's launch and its blocks' set-up overlap the end of the
// previous kernel, while all of its global-memory reads and writes follow the
// wait.  No kernel signals its dependents early (griddepcontrol.
// launch_dependents): the next grid launches as the blocks exit; an early
// signal at block start measured slower in the forward (dependent blocks
// holding SMs while they wait).
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// PPDL_PDL=0 in the environment launches without the attribute
inline bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("PPDL_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// kernel<<<g, b, smem, st>>>(args...) with programmatic stream
// serialization allowed; errors surface through cudaGetLastError as for the
// triple-chevron launch
template <typename... KArgs, typename... Args>
inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 g, dim3 b, size_t smem,
                              cudaStream_t st, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = g;
    cfg.blockDim = b;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline Status cuda_status() {
    return cudaGetLastError() == cudaSuccess ? OK : ERR_CUDA;
}

inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }

}  // namespace ppdl
