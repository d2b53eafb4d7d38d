// Checkpoint description and host-side tensor encodings, mirroring
// crates/omg-wgpu/src/model.rs: Config (:28-314), Dtype (:338-371) and the
// Q8_0 / Q4_0 quantizers and decoder (:409-525).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace omg {

enum class Arch { Gemma3, Gemma4 };

// model.rs:28-63. Per-layer vectors have `layers` entries.
struct Config {
  Arch arch = Arch::Gemma3;
  int vocab = 0, d = 0, layers = 0, heads = 0, kv_heads = 0;
  std::vector<int> head_dim, ff, kv_source, rope_dims;
  std::vector<bool> sliding;
  float eps = 1e-6f;
  int window = 512;
  float theta_global = 1e6f, theta_local = 1e4f, query_scale = 1.f, norm_offset = 0.f;
  bool v_norm = false;
  int per_layer_dim = 0;
  float softcap = 0.f;
  uint32_t bos = 2;

  // model.rs:66-210 (HF config.json, nested text_config allowed).
  static Config from_json(const std::string& text);
  // model.rs:213-254: what the kernels can run; throws Error otherwise.
  void validate() const;
  bool has_kv(int l) const { return kv_source[l] == l; }
  // model.rs:263-270
  int qkv_width(int l) const {
    return has_kv(l) ? (heads + 2 * kv_heads) * head_dim[l] : heads * head_dim[l];
  }
  int max_head_dim() const;
  int max_ff() const;

  struct TensorSpec {
    std::string name;
    std::vector<int64_t> shape;
  };
  // model.rs:277-314: every tensor the engine expects, in catalogue order.
  std::vector<TensorSpec> tensors() const;
};

// Payload bytes for n elements (model.rs:365-371).
size_t payload_bytes(int dtype, size_t n);

// model.rs:409-427 / 431-466: n a multiple of 32.
void quantize_q8(const float* v, size_t n, uint8_t* codes, uint8_t* scales);
void quantize_q4(const float* v, size_t n, uint8_t* codes, uint8_t* scales);
// model.rs:508-525 for every element.
void dequantize(int dtype, const uint8_t* codes, const uint8_t* scales, size_t n, float* out);

uint16_t f32_to_f16(float v);
float f16_to_f32(uint16_t h);

}  // namespace omg
