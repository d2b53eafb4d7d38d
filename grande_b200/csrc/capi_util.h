// Error plumbing for the C ABI: a thread-local last-error string, a status
// code per call (0 = ok, -1 = error), and a guard that turns C++ exceptions
// into that status so nothing unwinds across the ABI.
#pragma once
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <exception>
#include <stdexcept>
#include <string>

namespace omg {

std::string& last_error_slot();

inline int set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  last_error_slot() = buf;
  return -1;
}

// An engine error carrying the message the reference's anyhow error would.
struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] inline void fail(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Error(buf);
}

inline void cuda_check(cudaError_t e, const char* what, const char* file, int line) {
  if (e != cudaSuccess) fail("%s: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
}

template <class F>
int guarded(F&& f) {
  try {
    last_error_slot().clear();
    return f();
  } catch (const std::exception& e) {
    last_error_slot() = e.what();
    return -1;
  } catch (...) {
    last_error_slot() = "unknown error";
    return -1;
  }
}

}  // namespace omg

#define CUDA_TRY(expr) ::omg::cuda_check((expr), #expr, __FILE__, __LINE__)
