// Library-level C-ABI entry points: version, error messages, device status,
// and the programmatic-dependent-launch switch shared by every launcher.
#include <cstdlib>
#include <cstring>
#include <cstdio>
#include <map>
#include <mutex>
#include <set>
#include <utility>
#include <vector>

#include "common.cuh"
#include "capi_util.h"

namespace omni {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
  return code;
}

int check_launch(cudaError_t e) {
  if (e == cudaSuccess) return OMNI_OK;
  std::snprintf(g_last_error, sizeof(g_last_error), "CUDA launch failed: %s", cudaGetErrorString(e));
  return OMNI_ERR_CUDA;
}

static std::vector<StatusReader>& readers() {
  static std::vector<StatusReader> r;
  return r;
}
static std::mutex& readers_mu() {
  static std::mutex m;
  return m;
}

int register_status_reader(StatusReader r) {
  std::lock_guard<std::mutex> g(readers_mu());
  readers().push_back(r);
  return (int)readers().size();
}

// OMNI_PDL=0 disables programmatic dependent launch (every launch then waits
// for its predecessor in the stream, as a plain launch does).
bool pdl_enabled() {
  static int enabled = [] {
    const char* v = std::getenv("OMNI_PDL");
    return (v && v[0] == '0') ? 0 : 1;
  }();
  return enabled != 0;
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return dev;
}

int device_sm_count() {
  static std::mutex mu;
  static std::map<int, int> sms;
  const int dev = current_device();
  std::lock_guard<std::mutex> g(mu);
  auto it = sms.find(dev);
  if (it != sms.end()) return it->second;
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) {
    cudaGetLastError();
    return 148;  // not cached: asked again on the next call
  }
  sms[dev] = v;
  return v;
}

cudaError_t once_per_device(const void* kernel, int what, const std::function<cudaError_t()>& set) {
  static std::mutex mu;
  static std::set<std::pair<std::pair<const void*, int>, int>> done;
  const auto key = std::make_pair(std::make_pair(kernel, what), current_device());
  std::lock_guard<std::mutex> g(mu);
  if (done.count(key)) return cudaSuccess;
  const cudaError_t e = set();
  if (e == cudaSuccess) done.insert(key);
  return e;
}

// Every kernel of the library asks for the largest shared-memory carveout, so
// that all SMs keep one L1/shared split: an SM can only change its split while
// it is idle, so kernels that prefer different splits cannot overlap through
// programmatic dependent launch.
void prefer_max_shared(const void* fn) {
  const cudaError_t e = once_per_device(fn, kAttrCarveout, [fn] {
    return cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared);
  });
  if (e != cudaSuccess) cudaGetLastError();
}

}  // namespace omni

extern "C" OMNI_API const char* omni_version(void) { return "omni_b200 0.1.0 sm_100a"; }

extern "C" OMNI_API const char* omni_last_error(void) { return omni::g_last_error; }

extern "C" OMNI_API unsigned int omni_device_status(int reset) {
  std::lock_guard<std::mutex> g(omni::readers_mu());
  unsigned int v = 0;
  for (auto r : omni::readers()) {
    unsigned int s = r(reset);
    if (s && !v) v = s;
  }
  return v;
}
