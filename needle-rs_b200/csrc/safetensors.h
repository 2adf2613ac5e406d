// safetensors.h — SafeTensors reader for needle weight files.
//
// Mirrors crates/needle-infer/src/safetensors.rs: 8-byte LE header length, a
// JSON header of {name: {dtype, shape, data_offsets}} plus a string-valued
// __metadata__ object, then the raw tensor bytes.  Dtypes F32, BF16, F16, I8
// and the custom packed I4 (two signed nibbles per byte).
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ndl {

enum class DType { F32, BF16, F16, I8, I4 };

struct TensorMeta {
  DType dtype;
  std::vector<size_t> shape;
  size_t start = 0, end = 0;
};

class SafeTensors {
 public:
  // Parses `raw` (takes ownership).  Returns false with `err` set on a
  // malformed file (safetensors.rs:43-69, 140-214).
  bool parse(std::vector<uint8_t> raw, std::string &err);

  // Tensor converted to f32 (safetensors.rs:72-122).  False if absent, or an
  // I4 tensor whose byte count does not match its shape.
  bool get_f32(const std::string &name, std::vector<float> &out) const;
  // Raw bytes of a tensor (safetensors.rs:125-128).
  const uint8_t *get_raw(const std::string &name, size_t *len) const;
  const TensorMeta *meta(const std::string &name) const;
  const std::string *metadata(const std::string &key) const;

  // True when every value of a BF16 tensor (or an F32 tensor whose low 16
  // bits are all zero) is exactly representable in bf16.
  bool is_bf16_exact(const std::string &name) const;

 private:
  std::vector<uint8_t> data_;
  size_t data_off_ = 0;
  std::map<std::string, TensorMeta> tensors_;
  std::map<std::string, std::string> meta_;
};

float f16_to_f32(uint16_t bits);  // safetensors.rs:376-398

}  // namespace ndl
