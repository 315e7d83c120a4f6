// Host-side checkpoint access: a minimal safetensors reader (src/st.rs semantics: u64-LE header
// length, JSON directory, little-endian payload; F32/F64/I64 accepted) and the weight resolution
// rules of src/weights.rs (plain `.weight` or weight_norm(weight_v, weight_g); AdaIN affine
// defaults).
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace kk {

struct KKError : std::runtime_error {
  int status;
  KKError(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

struct HostTensor {
  std::vector<int64_t> shape;
  std::vector<float> data;  // converted to f32 (F64 / I64 payloads are cast)
};

class Checkpoint {
 public:
  explicit Checkpoint(const std::string& path);
  bool has(const std::string& name) const { return map_.count(name) != 0; }
  // f32 tensor with its exact shape asserted (Weights::get, src/weights.rs:53-60)
  std::vector<float> get(const std::string& name, const std::vector<int64_t>& shape) const;
  // `prefix.weight` if present, else weight_norm(weight_v, weight_g) (src/weights.rs:62-70)
  std::vector<float> conv_weight(const std::string& prefix, const std::vector<int64_t>& shape) const;
  // AdaIN InstanceNorm affine: defaults to `init` when absent (src/weights.rs:76-84)
  std::vector<float> norm_affine(const std::string& name, int64_t c, float init) const;
  size_t size() const { return map_.size(); }

 private:
  std::unordered_map<std::string, HostTensor> map_;
};

// torch._weight_norm(v, g, dim=0) (src/ops.rs:9-23): f64 row norm cast to f32, scale = g / norm.
std::vector<float> weight_norm(const std::vector<float>& v, const std::vector<float>& g);

}  // namespace kk
