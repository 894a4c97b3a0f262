// dk_internal.h -- shared declarations of the library's host code (not part of the C ABI).
#pragma once

#include "../../include/diolkos.h"
#include "dk_kernels.h"

namespace dk {

// Record an error message for dk_last_error() and return `code`.
int set_error(int code, const char *fmt, ...);
// DK_OK for cudaSuccess, else DK_ERR_CUDA with the CUDA error string.
int cuda_status(cudaError_t e, const char *what);
int current_num_sms();
// A zero-initialised device int on the current device, used as the error word of standalone
// kernel calls (allocated once per device, never freed).
int *device_error_word();

}  // namespace dk
