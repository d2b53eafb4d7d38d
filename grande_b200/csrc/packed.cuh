// Q4_0 / Q8_0 projection weights kept packed in HBM and decoded per tile in
// shared memory by the tensor-core GEMMs (the reference keeps its weights
// packed in device memory too and decodes them per use:
// crates/omg-wgpu/src/shaders/weight.wgsl:29-54, matmul.wgsl:1-9).
//
// Layout: a weight [rows, k] is cut into chunks of 128 rows x one 64-wide K
// step, stored chunk-row-major ([ceil(rows / 128)][ceil(k / 64)] chunks), so
// the GEMM stages one K step of 128 weight rows with a single contiguous
// bulk copy. Inside a chunk, for the two 32-element blocks b of the K step:
//   codes  [b][row][16 B]  (Q4_0: low nibbles = elements 0..15, high 16..31)
//          [b][row][32 B]  (Q8_0: int8)
//   scales [b][row] f16
// (4,608 bytes per Q4_0 chunk, 8,704 per Q8_0 chunk: the weight's own
// 18 / 34 bytes per 32 values, nothing more). Rows past the weight's end, up
// to a whole 256 (the widest tile a GEMM stages), and K blocks past k are
// zero (code 0, scale 0: the value 0).
//
// Decoding gives f16(QTensor::get) exactly (model.rs:508-525): the code
// becomes an exact f16 by writing it into the mantissa of 1024 (f16 bits
// 0x6400 | q) and subtracting 1024 + offset, and one f16 multiply by the
// block's f16 scale rounds the exact product (at most 4 + 11 or 8 + 11
// significant bits) once, as the f32 product rounded to f16 does.
#pragma once
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

#include "kernels.cuh"

namespace omg {

template <int DT>
struct PackChunk {
  static constexpr int CODE_BYTES = DT == kQ4 ? 16 : 32;  // per row per 32-block
  static constexpr int CODES = 2 * 128 * CODE_BYTES;
  static constexpr int SCALES = 2 * 128 * 2;
  static constexpr int BYTES = CODES + SCALES;
};

constexpr int kPackRows = 128;  // weight rows per chunk
constexpr int kPackK = 64;      // K values per chunk

inline size_t pack_chunk_bytes(int dtype) {
  return dtype == kQ4 ? PackChunk<kQ4>::BYTES : PackChunk<kQ8>::BYTES;
}

// Bytes of a packed [rows, k] weight (rows padded to a multiple of 256).
inline size_t packed_bytes(int dtype, int rows, int k) {
  return static_cast<size_t>((rows + 255) / 256 * 2) *
         static_cast<size_t>((k + kPackK - 1) / kPackK) * pack_chunk_bytes(dtype);
}

#if defined(__CUDACC__)
// A half2 from its bit pattern (no conversion instruction: constants built
// with __float2half2_rn are converted at run time).
__device__ __forceinline__ __half2 bits_half2(uint32_t b) {
  return *reinterpret_cast<const __half2*>(&b);
}

// Values 8 PC .. 8 PC + 7 of a block (its codes `c`, its scale `d2` in both
// halves) as eight f16, one 16-byte piece of an f16 row.
template <int DT, int PC>
__device__ __forceinline__ uint4 unpack_piece(const uint4* c, __half2 d2) {
  uint32_t w0, w1;
  __half2 bias;
  if constexpr (DT == kQ8) {
    const uint4 q = c[PC / 2];
    w0 = (PC & 1) ? q.z : q.x;
    w1 = (PC & 1) ? q.w : q.y;
    bias = bits_half2(0x64806480u);  // 1152 = 1024 + 128: (int8 ^ 0x80) is the code + 128
  } else {
    const uint4 q = c[0];
    w0 = (PC & 1) ? q.z : q.x;
    w1 = (PC & 1) ? q.w : q.y;
    if (PC >= 2) {
      w0 >>= 4;
      w1 >>= 4;
    }
    bias = bits_half2(0x64086408u);  // 1032 = 1024 + 8: w = (q - 8) d
  }
  uint32_t h[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t w = e < 2 ? w0 : w1;
    // Bytes 0, 1 (or 2, 3) of w into the low byte of each 16-bit lane.
    uint32_t x = __byte_perm(w, 0u, (e & 1) ? 0x4342u : 0x4140u);
    if constexpr (DT == kQ8)
      x ^= 0x64806480u;
    else
      x = (x & 0x000F000Fu) | 0x64006400u;
    const __half2 code = __hsub2(*reinterpret_cast<const __half2*>(&x), bias);
    const __half2 v = __hmul2(code, d2);
    h[e] = *reinterpret_cast<const uint32_t*>(&v);
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// Block b (0 or 1) of row r (0..127) of the chunk at `raw` (shared or global
// memory) as its four f16 pieces.
template <int DT>
__device__ __forceinline__ void unpack_block(const uint8_t* raw, int r, int b, uint4 (&out)[4]) {
  using P = PackChunk<DT>;
  uint4 c[DT == kQ4 ? 1 : 2];
  const uint4* src = reinterpret_cast<const uint4*>(raw + (b * 128 + r) * P::CODE_BYTES);
  c[0] = src[0];
  if constexpr (DT == kQ8) c[1] = src[1];
  const uint16_t sb = *reinterpret_cast<const uint16_t*>(raw + P::CODES + (b * 128 + r) * 2);
  const __half d = __ushort_as_half(sb);
  const __half2 d2 = __halves2half2(d, d);
  out[0] = unpack_piece<DT, 0>(c, d2);
  out[1] = unpack_piece<DT, 1>(c, d2);
  out[2] = unpack_piece<DT, 2>(c, d2);
  out[3] = unpack_piece<DT, 3>(c, d2);
}

// Both blocks of chunk row r into row `tr` of a 128-byte-swizzled K-major f16
// tile (the layout a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes and the
// MMA's shared-memory descriptor reads: piece p of row tr at
// tr * 128 + ((p ^ (tr & 7)) << 4)).
template <int DT>
__device__ __forceinline__ void unpack_row_to_tile(const uint8_t* raw, int r, uint8_t* tile,
                                                   int tr) {
  uint8_t* row = tile + tr * 128;
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    uint4 pc[4];
    unpack_block<DT>(raw, r, b, pc);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(row + (((4 * b + i) ^ (tr & 7)) << 4)) = pc[i];
  }
}

#endif  // __CUDACC__

// Host launchers (kernels.cu).
// Repack a pushed weight (codes and f16 scales as QTensor holds them:
// row-major runs, model.rs:338-371) into chunks at `out`, which the caller
// zeroes once (gate and up land in one buffer); `out_rows` its row count.
// remap 1 / 2 puts row r of a gate / up weight at row (r / 128) * 256 +
// (0 / 128) + r % 128 of the interleaved gate_up weight.
void launch_pack_weight(int dtype, const void* codes, const void* scales, int rows, int k,
                        int remap, int out_rows, uint8_t* out, cudaStream_t s);
// Decode a packed weight to row-major f16 [rows, k] with the GEMM's decoder.
void launch_unpack_weight(int dtype, const uint8_t* packed, int rows, int k, __half* out,
                          cudaStream_t s);

}  // namespace omg
