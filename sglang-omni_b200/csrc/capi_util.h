// Host-side helpers shared by the C-ABI entry points.
#pragma once
#include <cuda_runtime.h>

#include <functional>

namespace omni {

// Records the calling thread's last error message and returns code.
int set_error(int code, const char* msg);
// Maps a launch result to OMNI_OK / OMNI_ERR_CUDA (recording the message).
int check_launch(cudaError_t e);

// The current device's ordinal (0 when the runtime cannot report one).
int current_device();
// Streaming multiprocessors of the current device, cached per device ordinal.
int device_sm_count();
// Runs `set` (a kernel-attribute setter: cudaFuncSetAttribute applies to the
// device that is current) the first time the pair (kernel, what) is seen on the
// current device, and again on a later call if it failed.  Thread-safe.
enum AttrKind : int { kAttrSmem = 0, kAttrCarveout = 1, kAttrCluster = 2 };
cudaError_t once_per_device(const void* kernel, int what, const std::function<cudaError_t()>& set);

}  // namespace omni
