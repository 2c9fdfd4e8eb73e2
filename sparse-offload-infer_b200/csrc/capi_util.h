// Error-state helpers shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>

namespace soinfer {

// Records a formatted message as the calling thread's last error; returns status.
int set_error(int status, const char* fmt, ...);
// SOINFER_OK for cudaSuccess, else SOINFER_ERR_CUDA with the CUDA message.
int cuda_result(cudaError_t e, const char* what);
const char* last_error();

}  // namespace soinfer
