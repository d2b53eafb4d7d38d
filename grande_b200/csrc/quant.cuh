// Device-side reading of the reference's weight storage (model.rs:338-371:
// f16, Q8_0 = 32 int8 codes + f16 scale, Q4_0 = 16 bytes of nibbles + f16
// scale, codes and scales in separate runs) as the f32 values QTensor::get
// returns (model.rs:508-525).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "kernels.cuh"

namespace omg {

__device__ __forceinline__ float half_bits_to_float(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

// Dequantized 32-element block `b` of a row-major table (f32, exact as
// QTensor::get).
template <int DT>
__device__ __forceinline__ void load_block_f32(const uint8_t* codes, const uint8_t* scales,
                                               size_t b, float (&v)[32]) {
  if constexpr (DT == kF16) {
    __align__(16) uint16_t h[32];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      reinterpret_cast<uint4*>(h)[i] = reinterpret_cast<const uint4*>(codes + b * 64)[i];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = half_bits_to_float(h[j]);
  } else {
    const uint16_t sb =
        static_cast<uint16_t>(scales[2 * b]) | (static_cast<uint16_t>(scales[2 * b + 1]) << 8);
    const float d = half_bits_to_float(sb);
    if constexpr (DT == kQ8) {
      __align__(16) int8_t q[32];
      reinterpret_cast<uint4*>(q)[0] = reinterpret_cast<const uint4*>(codes + b * 32)[0];
      reinterpret_cast<uint4*>(q)[1] = reinterpret_cast<const uint4*>(codes + b * 32)[1];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = static_cast<float>(q[j]) * d;
    } else {
      __align__(16) uint8_t q[16];
      reinterpret_cast<uint4*>(q)[0] = reinterpret_cast<const uint4*>(codes + b * 16)[0];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[j] = (static_cast<float>(q[j] & 0xf) - 8.0f) * d;
        v[j + 16] = (static_cast<float>(q[j] >> 4) - 8.0f) * d;
      }
    }
  }
}

}  // namespace omg
