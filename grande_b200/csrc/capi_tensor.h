// Helpers the C ABI entry points share: a HostTensor from the caller's
// buffers and the copy of a string result into a caller buffer.
#pragma once
#include <algorithm>
#include <cstring>
#include <string>

#include "capi_util.h"
#include "engine.h"

namespace omg {

inline HostTensor make_tensor(int dtype, const int64_t* shape, int ndim, const void* data,
                              size_t nbytes, const void* scales, size_t nscales) {
  if (ndim < 0 || ndim > 4) fail("tensor rank %d", ndim);
  if (nbytes && !data) fail("tensor data is null");
  if (nscales && !scales) fail("tensor scales are null");
  HostTensor t;
  t.dtype = dtype;
  t.shape.assign(shape, shape + ndim);
  t.data.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + nbytes);
  if (nscales)
    t.scales.assign(static_cast<const uint8_t*>(scales),
                    static_cast<const uint8_t*>(scales) + nscales);
  return t;
}

inline int copy_out(const std::string& s, char* buf, size_t cap, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (buf && cap) {
    const size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return 0;
}

}  // namespace omg
