// C ABI plumbing shared by every entry point: the thread-local error slot and
// the version string.
#include <string>

#include "capi_util.h"
#include "omg_b200.h"

namespace omg {

std::string& last_error_slot() {
  static thread_local std::string slot;
  return slot;
}

}  // namespace omg

extern "C" const char* omg_last_error(void) { return omg::last_error_slot().c_str(); }

extern "C" const char* omg_version(void) { return "omg_b200 0.1.0 (sm_100a)"; }
