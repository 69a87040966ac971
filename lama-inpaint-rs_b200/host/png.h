// PNG codec of the CLI (png.cpp).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <string>
#include <vector>

namespace lama_host {

struct Rgb8 {
  int width = 0, height = 0;
  std::vector<uint8_t> data;  // row-major HWC
};

bool png_decode(const std::vector<uint8_t>& file, const std::string& source, Rgb8& img, std::string& err);
bool png_encode(const Rgb8& img, std::vector<uint8_t>& out, std::string& err);

}  // namespace lama_host
