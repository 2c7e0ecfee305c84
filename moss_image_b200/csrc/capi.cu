// Library-level C ABI entry points: version, last error, the host-visible status copy and
// the GEMM timeout test hook.
#include <cstring>
#include <mutex>
#include <string>

#include "errors.cuh"

namespace moss {
std::string& last_error_slot() {
  static thread_local std::string slot;
  return slot;
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mirror_mu;
int* g_mirror_host[kMaxDevices] = {};
int* g_mirror_dev[kMaxDevices] = {};
thread_local bool t_debug_stall = false;
}  // namespace

int* status_mirror_for_current_device() {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mirror_mu);
  return g_mirror_dev[device];
}

bool take_debug_stall() {
  const bool stall = t_debug_stall;
  t_debug_stall = false;
  return stall;
}
}  // namespace moss

extern "C" int moss_version(void) { return 101; }

extern "C" const char* moss_last_error(void) { return moss::last_error_slot().c_str(); }

extern "C" int moss_status_mirror(int** host_word) {
  using namespace moss;
  if (host_word == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null host_word pointer");
  int device = -1;
  MOSS_CUDA_TRY(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices)
    return fail(MOSS_ERR_UNSUPPORTED, "device ordinal %d is beyond the %d devices this library tracks", device,
                kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mirror_mu);
  if (g_mirror_host[device] == nullptr) {
    void* host = nullptr;
    MOSS_CUDA_TRY(cudaHostAlloc(&host, 64, cudaHostAllocMapped | cudaHostAllocPortable));
    std::memset(host, 0, 64);
    void* dev = nullptr;
    const cudaError_t e = cudaHostGetDevicePointer(&dev, host, 0);
    if (e != cudaSuccess) {
      cudaFreeHost(host);
      return check_cuda(e, "cudaHostGetDevicePointer");
    }
    g_mirror_host[device] = static_cast<int*>(host);
    g_mirror_dev[device] = static_cast<int*>(dev);
  }
  *host_word = g_mirror_host[device];
  return clear_ok();
}

extern "C" int moss_debug_stall_next_gemm(void) {
  moss::t_debug_stall = true;
  return moss::clear_ok();
}
