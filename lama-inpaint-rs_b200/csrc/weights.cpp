// safetensors reader for the engine (see weights.h).
#include "weights.h"

#include <cstdio>
#include <cstring>

namespace lama {

namespace {

struct Json {
  const std::string& s;
  size_t i = 0;
  explicit Json(const std::string& str) : s(str) {}
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) i++;
  }
  bool eat(char c) {
    ws();
    if (i < s.size() && s[i] == c) {
      i++;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (i >= s.size() || s[i] != '"') return false;
    i++;
    out.clear();
    while (i < s.size() && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < s.size()) i++;
      out += s[i++];
    }
    if (i >= s.size()) return false;
    i++;
    return true;
  }
  bool num(int64_t& v) {
    ws();
    bool neg = false;
    if (i < s.size() && s[i] == '-') { neg = true; i++; }
    if (i >= s.size() || s[i] < '0' || s[i] > '9') return false;
    v = 0;
    while (i < s.size() && s[i] >= '0' && s[i] <= '9') {
      const int d = s[i++] - '0';
      if (v > (INT64_MAX - d) / 10) return false;  // does not fit int64: malformed for this container
      v = v * 10 + d;
    }
    if (neg) v = -v;
    return true;
  }
  bool skip_value() {
    ws();
    if (i >= s.size()) return false;
    if (s[i] == '"') { std::string t; return str(t); }
    if (s[i] == '{' || s[i] == '[') {
      int depth = 0;
      while (i < s.size()) {
        if (s[i] == '"') { std::string t; if (!str(t)) return false; continue; }
        if (s[i] == '{' || s[i] == '[') depth++;
        if (s[i] == '}' || s[i] == ']') { depth--; if (depth == 0) { i++; return true; } }
        i++;
      }
      return false;
    }
    while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') i++;
    return true;
  }
  bool int_list(std::vector<int64_t>& v) {
    v.clear();
    if (!eat('[')) return false;
    if (eat(']')) return true;
    do {
      int64_t x;
      if (!num(x)) return false;
      v.push_back(x);
    } while (eat(','));
    return eat(']');
  }
};

}  // namespace

bool WeightFile::open(const std::string& path, std::string& err) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) { err = path + ": cannot open weight file"; return false; }
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (n < 8) { fclose(f); err = path + ": too short for a safetensors header"; return false; }
  data_.resize((size_t)n);
  size_t got = fread(data_.data(), 1, (size_t)n, f);
  fclose(f);
  if (got != (size_t)n) { err = path + ": short read"; return false; }
  uint64_t hl = 0;
  memcpy(&hl, data_.data(), 8);
  if (hl > (uint64_t)n - 8) { err = path + ": header length past end of file"; return false; }
  base_ = 8 + (size_t)hl;
  std::string header((const char*)data_.data() + 8, (size_t)hl);
  Json j(header);
  if (!j.eat('{')) { err = path + ": malformed safetensors header"; return false; }
  if (!j.eat('}')) {
    do {
      std::string name;
      if (!j.str(name) || !j.eat(':')) { err = path + ": malformed safetensors header"; return false; }
      if (name == "__metadata__") {
        if (!j.skip_value()) { err = path + ": malformed __metadata__"; return false; }
        continue;
      }
      if (!j.eat('{')) { err = path + ": malformed entry for " + name; return false; }
      TensorRec r;
      std::string dtype;
      std::vector<int64_t> offs;
      bool have_shape = false;
      if (!j.eat('}')) {
        do {
          std::string key;
          if (!j.str(key) || !j.eat(':')) { err = path + ": malformed entry for " + name; return false; }
          if (key == "dtype") { if (!j.str(dtype)) return (err = "bad dtype for " + name, false); }
          else if (key == "shape") { if (!j.int_list(r.shape)) return (err = "bad shape for " + name, false); have_shape = true; }
          else if (key == "data_offsets") { if (!j.int_list(offs)) return (err = "bad data_offsets for " + name, false); }
          else if (!j.skip_value()) return (err = "bad entry for " + name, false);
        } while (j.eat(','));
        if (!j.eat('}')) { err = path + ": malformed entry for " + name; return false; }
      }
      if (dtype != "F32") {
        err = "tensor " + name + " is " + dtype + ", not F32 - is this a big-lama checkpoint?";
        return false;
      }
      if (!have_shape || offs.size() != 2 || offs[0] < 0 || offs[1] < offs[0] ||
          base_ + (size_t)offs[1] > data_.size()) {
        err = "tensor " + name + ": data_offsets outside the file (truncated?)";
        return false;
      }
      int64_t numel = 1;
      for (int64_t d : r.shape) {
        if (d < 0 || (d > 0 && numel > INT64_MAX / 4 / d)) {
          err = "tensor " + name + ": shape has a negative or oversized dimension";
          return false;
        }
        numel *= d;
      }
      if ((int64_t)(offs[1] - offs[0]) != numel * 4) {
        err = "tensor " + name + ": payload size does not match its shape";
        return false;
      }
      r.begin = (size_t)offs[0];
      r.end = (size_t)offs[1];
      recs_[name] = r;
    } while (j.eat(','));
    if (!j.eat('}')) { err = path + ": malformed safetensors header"; return false; }
  }
  if (recs_.empty()) { err = "no tensors found in " + path; return false; }
  return true;
}

bool WeightFile::f32(const std::string& name, const std::vector<int64_t>& want, std::vector<float>& out,
                     std::string& err) const {
  auto it = recs_.find(name);
  if (it == recs_.end()) { err = "missing tensor in weight blob: " + name; return false; }
  const TensorRec& r = it->second;
  if (!want.empty() && r.shape != want) {
    std::string a, b;
    for (auto d : r.shape) a += std::to_string(d) + ",";
    for (auto d : want) b += std::to_string(d) + ",";
    err = "tensor " + name + " has shape [" + a + "], expected [" + b + "]";
    return false;
  }
  out.resize((r.end - r.begin) / 4);
  memcpy(out.data(), data_.data() + base_ + r.begin, r.end - r.begin);
  return true;
}

size_t WeightFile::payload_bytes() const {
  size_t s = 0;
  for (auto& kv : recs_) s += kv.second.end - kv.second.begin;
  return s;
}

}  // namespace lama
