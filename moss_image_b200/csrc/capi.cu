// Library-level C ABI entry points (version, last error).
#include <string>

#include "errors.cuh"

namespace moss {
std::string& last_error_slot() {
  static thread_local std::string slot;
  return slot;
}
}  // namespace moss

extern "C" int moss_version(void) { return 100; }

extern "C" const char* moss_last_error(void) { return moss::last_error_slot().c_str(); }
