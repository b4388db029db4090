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
// Sets the conv kernels' shared-memory attributes on the current device, once per
// device for the whole process (the stateless conv seams call it before launching).
rk_status conv_seam_init_device();
}  // namespace rk
