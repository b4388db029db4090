// status.h -- error reporting shared by the C-ABI entry points: a status code
// is returned, and a human-readable detail is kept per calling thread.
#pragma once
#include <cuda_runtime.h>

#include "../../include/rk_b200.h"

namespace rk {
rk_status fail(rk_status s, const char* what);
// appends cudaGetLastError()'s text (and clears it)
rk_status fail_cuda(rk_status s, const char* what);
rk_status fail_cuda_err(rk_status s, const char* what, cudaError_t e);
}  // namespace rk
