// Host-side helpers shared by the C-ABI entry points.
#pragma once
#include <cuda_runtime.h>

namespace omni {

// Records the calling thread's last error message and returns code.
int set_error(int code, const char* msg);
// Maps a launch result to OMNI_OK / OMNI_ERR_CUDA (recording the message).
int check_launch(cudaError_t e);

}  // namespace omni
