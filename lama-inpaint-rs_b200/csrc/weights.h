// The checkpoint container: a safetensors file (u64 LE header length, JSON
// header, payloads).  Same checks as the reference's weight store
// (lama-rs/src/weights.rs:80-106): every tensor F32, every payload inside the
// file; lookups fail with the reference's "missing tensor in weight blob" text.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace lama {

struct TensorRec {
  std::vector<int64_t> shape;
  size_t begin = 0, end = 0;  // payload-relative byte range
};

class WeightFile {
 public:
  // Returns false with a message in `err`.
  bool open(const std::string& path, std::string& err);
  bool has(const std::string& name) const { return recs_.count(name) != 0; }
  // Copies a tensor out as f32; checks the shape when `want` is non-empty.
  bool f32(const std::string& name, const std::vector<int64_t>& want, std::vector<float>& out,
           std::string& err) const;
  size_t count() const { return recs_.size(); }
  size_t payload_bytes() const;

 private:
  std::vector<uint8_t> data_;
  size_t base_ = 0;
  std::map<std::string, TensorRec> recs_;
};

}  // namespace lama
