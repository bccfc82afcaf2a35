// gemm_static.cu — ppdl_gemm_tf32x3_static: the FP32-faithful tensor-core
// GEMM for callers that cannot allocate device memory.
//
// ppdl_gemm_tf32x3 needs a workspace for the TF32 halves of its B operand
// (2*N*K floats) and takes it from the caller.  Some callers have no way to
// provide one: a ggml custom-op hook (ggml_cuda_compute_forward_ppdl) runs
// inside ggml's graph compute, where every device buffer belongs to ggml's
// allocator and the node sees only its own dst and src tensors, so it can
// neither cudaMalloc a workspace nor receive one.  This variant keeps that
// workspace in a file-scope device array instead.
//
// Contract:
//   * the array holds kStaticMaxNK split weights (2 x 2,097,152 floats =
//     16 MiB) and lives on every device that loads this library until the
//     process exits; N*K above kStaticMaxNK is rejected (PPDL_ERR_SHAPE);
//   * the first call on a device resolves the array's device address
//     (cudaGetSymbolAddress, once per device, with that device current); make
//     that first call before any stream capture on the device;
//   * nothing is allocated or freed (no cudaMalloc/cudaFree, no allocating
//     library routine);
//   * all calls share the array and it keeps the last call's contents; every
//     call overwrites the N*K hi/lo entries it reads before reading them, so
//     nothing has to start at zero; calls whose GPU work overlaps (other
//     streams, other host threads on the same device) race on the array and
//     must be serialised by the caller.
#include <mutex>

#include "../../include/ppdl_ops.h"
#include "gemm_tc.h"

namespace ppdl {
void set_op_error(const char *msg);
}

namespace {

constexpr long long kStaticMaxNK = 1LL << 21;

// [0, N*K): hi halves of B; [kStaticMaxNK, kStaticMaxNK + N*K): lo halves
__device__ __align__(256) float g_gemm_static_scratch[2 * kStaticMaxNK];

std::mutex g_mu;
constexpr int kMaxDevices = 64;
float *g_scratch_addr[kMaxDevices] = {};

// Device address of the array on the current device (resolved once per device).
float *scratch_on_current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemm_static_scratch) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_scratch_addr[dev] = static_cast<float *>(p);
    }
    return g_scratch_addr[dev];
}

}  // namespace

namespace ppdl {
// The same array for the operator hooks of ops_conv.cu (ops 3 and 12 split
// their weights into it in chunks): hi at [0, cap), lo at [cap, 2 cap).
// Shared with ppdl_gemm_tf32x3_static: their GPU work must not overlap.
float *static_split_workspace(long long *cap) {
    *cap = kStaticMaxNK;
    return scratch_on_current_device();
}
}  // namespace ppdl

extern "C" PPDL_OPS_API int ppdl_gemm_tf32x3_static(int M, int N, int K, int batch, const float *A,
                                                    int a_m_major, long long lda, long long a_bs,
                                                    const float *B, float *C, long long ldc_m,
                                                    long long ldc_n, long long c_bs,
                                                    void *stream) {
    ppdl::set_op_error("");  // a PPDL_OK leaves no older message behind
    if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || !A || !B || !C) {
        ppdl::set_op_error("gemm_static: bad sizes or null pointer");
        return PPDL_ERR_SHAPE;
    }
    if ((long long)N * K > kStaticMaxNK) {
        ppdl::set_op_error("gemm_static: N*K exceeds the static workspace (2097152 weights)");
        return PPDL_ERR_SHAPE;
    }
    float *ws = scratch_on_current_device();
    if (!ws) {
        ppdl::set_op_error("gemm_static: cudaGetSymbolAddress of the static workspace failed");
        return PPDL_ERR_CUDA;
    }
    cudaStream_t st = (cudaStream_t)stream;
    float *hi = ws, *lo = ws + kStaticMaxNK;
    if (ppdl::launch_tf32_split(B, hi, lo, (long long)N * K, st) != ppdl::OK) {
        ppdl::set_op_error("gemm_static: split launch failed");
        return PPDL_ERR_CUDA;
    }
    ppdl::TcEpilogue e;
    e.C = C; e.ldc_m = ldc_m; e.ldc_n = ldc_n; e.c_bs = c_bs;
    ppdl::TcGemm g;
    if (!ppdl::tc_gemm_plan(&g, M, N, K, batch, A, a_m_major ? 1 : 0, lda, a_bs, hi, lo, 1, e)) {
        ppdl::set_op_error("gemm_static: operands violate the TMA rules (16-byte alignment, "
                           "strides and K multiples of 4)");
        return PPDL_ERR_SHAPE;
    }
    if (ppdl::launch_tc_gemm(g, st) != ppdl::OK) {
        ppdl::set_op_error("gemm_static: GEMM launch failed");
        return PPDL_ERR_CUDA;
    }
    return PPDL_OK;
}
