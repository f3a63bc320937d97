// safetensors file reader (header JSON + raw little-endian tensor bytes).
//
// Replaces WeightStore (Weights.swift:23-58) / mlx-swift loadArrays for this path:
// every tensor of one file, keyed by name, with dtype and shape.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "gdc.h"

namespace gdc {

struct TensorInfo {
  std::string dtype;            // "F16", "F32", "BF16", "I64", ...
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte offsets relative to the data section
};

class SafetensorsFile {
 public:
  // Reads and parses the whole file. GDC_ERR_IO on a missing / truncated / malformed file.
  gdc_status open(const std::string& path);

  bool has(const std::string& key) const { return tensors_.count(key) != 0; }
  const TensorInfo* info(const std::string& key) const;
  const uint8_t* data(const TensorInfo& t) const { return bytes_.data() + data_offset_ + t.begin; }
  const std::map<std::string, TensorInfo>& tensors() const { return tensors_; }

  // Converts a floating tensor (F16 / BF16 / F32) to fp16 bits. Key and shape checks
  // follow WeightStore.array(_:shape:) (Weights.swift:34-57).
  gdc_status get_f16(const std::string& key, const std::vector<int64_t>* expected_shape,
                     std::vector<uint16_t>* out, std::vector<int64_t>* shape_out = nullptr) const;

 private:
  std::vector<uint8_t> bytes_;
  size_t data_offset_ = 0;
  std::map<std::string, TensorInfo> tensors_;
};

// Parses the JSON header of a safetensors file (exposed for tests of malformed input).
gdc_status parse_safetensors_header(const char* json, size_t len, uint64_t data_bytes,
                                    std::map<std::string, TensorInfo>* out);

}  // namespace gdc
