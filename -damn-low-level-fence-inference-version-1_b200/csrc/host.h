// host.h — host-side error plumbing shared by every translation unit of libfence_b200.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <cuda_runtime.h>

#define FENCE_BUILDING_LIBRARY 1
#include "../../include/fence_b200.h"

namespace fence {

// Records a formatted message as this thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
// Maps a CUDA status to the C-ABI status (0 or the cudaError_t value), recording the message.
int cuda_status(cudaError_t e, const char* what);

}  // namespace fence

#define FENCE_CUDA_TRY(expr)                                                   \
    do {                                                                       \
        cudaError_t _e = (expr);                                               \
        if (_e != cudaSuccess) return ::fence::cuda_status(_e, #expr);         \
    } while (0)
