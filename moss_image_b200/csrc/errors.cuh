// Host-side error plumbing for the C ABI: a thread-local message and helpers that turn
// CUDA failures into MOSS_ERR_* codes.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/moss_w8.h"

namespace moss {

std::string& last_error_slot();

// Device-visible address of the current device's host-visible status copy (set up by
// moss_status_mirror), or nullptr when the caller has not asked for one.
int* status_mirror_for_current_device();

// Whether the calling thread asked for a debug stall of its next GEMM
// (moss_debug_stall_next_gemm); the request is consumed by this call.
bool take_debug_stall();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error_slot() = buf;
  return code;
}

inline int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MOSS_OK;
  return fail(MOSS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline int clear_ok() {
  last_error_slot().clear();
  return MOSS_OK;
}

inline bool is_float_kind(int k) {
  return k == MOSS_DTYPE_F16 || k == MOSS_DTYPE_BF16 || k == MOSS_DTYPE_F32;
}

inline int dtype_size(int k) { return k == MOSS_DTYPE_F32 ? 4 : 2; }

}  // namespace moss

#define MOSS_CUDA_TRY(expr)                               \
  do {                                                    \
    int _rc = ::moss::check_cuda((expr), #expr);          \
    if (_rc != MOSS_OK) return _rc;                       \
  } while (0)
