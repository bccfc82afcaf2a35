// ops_internal.h — the conv-family op ids of the operator ABI (3, 4, 10, 11,
// 12), implemented next to the conv kernels in ops_conv.cu.
#pragma once

#include <cuda_runtime.h>

#include "../../include/ppdl_ops.h"

namespace ppdl {

// True when op id `id` is one of the conv-family ops this build provides.
bool ops_ext_provided(int id);

// Launches a conv-family op.  Returns false when `d` is not one of them;
// otherwise stores the PPDL_* status in *status (and a message in err).
bool ops_ext_launch(const ppdl_op_desc *d, cudaStream_t stream, int *status, char *err,
                    size_t err_len);

}  // namespace ppdl
