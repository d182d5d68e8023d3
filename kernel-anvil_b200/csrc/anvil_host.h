// anvil_host.h -- host helpers shared by the translation units of libanvil.so (defined in
// anvil_abi.cu): error reporting into anvil_last_error() and per-device queries.
#pragma once

#include <cuda_runtime.h>

namespace anvil {

// Records a printf-style message as the calling thread's last error; returns `status`.
int fail(int status, const char *fmt, ...);
// ANVIL_ERR_CUDA with the CUDA error's name and text.
int cuda_fail(cudaError_t e, const char *what);
// Current device (rejects ids beyond the library's per-device tables).
int current_device(int *dev);
// Multiprocessor count of `dev` (cached).
int sm_count(int dev, int *out);
// Bound on every device-side wait of the kernels launched from now on (anvil_set_wait_limit_ns).
unsigned long long wait_limit_ns();

}  // namespace anvil
