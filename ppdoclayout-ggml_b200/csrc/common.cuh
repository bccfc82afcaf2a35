// common.cuh — shared definitions of the B200 PP-DocLayoutV3 kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

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

// Activation exactly as the reference evaluates it: ReLU fmaxf, SiLU
// x / (1 + exp(-x)) (patch:383-386, 426-430; ggml_silu), GELU with erf
// (ggml_gelu_erf, src/ppdoclayout.cpp:687).
__device__ __forceinline__ float act_apply(float v, int act) {
    if (act == ACT_RELU) return fmaxf(v, 0.0f);
    if (act == ACT_SILU) return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
    if (act == ACT_GELU) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
    return v;
}

// Status returned by the internal launchers.
enum Status : int { OK = 0, ERR_UNSUPPORTED = 1, ERR_SHAPE = 2, ERR_CUDA = 3 };

inline Status cuda_status() {
    return cudaGetLastError() == cudaSuccess ? OK : ERR_CUDA;
}

inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }

}  // namespace ppdl
