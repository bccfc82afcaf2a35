// ops_conv.cu — conv-family op ids of the operator ABI (3, 4, 10, 11, 12).
#include "ops_internal.h"

namespace ppdl {

bool ops_ext_provided(int) { return false; }

bool ops_ext_launch(const ppdl_op_desc *, cudaStream_t, int *, char *, size_t) { return false; }

}  // namespace ppdl
