// Minimal PNG codec over zlib for the CLI.
//
// Decoding follows what the reference CLI accepts (lama-rs/src/image.rs:80-130):
// 8- and 16-bit samples (16-bit keeps the high byte), greyscale, grey+alpha,
// RGB, RGBA and palette images, converted to 8-bit RGB (alpha dropped, grey
// replicated, palette indices clamped to the palette); other bit depths are
// an error.  Adam7-interlaced files are de-interlaced.  Chunk CRCs are
// checked.  Encoding writes 8-bit RGB (image.rs:132-155).
#include "png.h"

#include <zlib.h>

#include <cstdio>
#include <cstring>

namespace lama_host {

namespace {

const uint8_t kSig[8] = {137, 80, 78, 71, 13, 10, 26, 10};

uint32_t be32(const uint8_t* p) { return ((uint32_t)p[0] << 24) | ((uint32_t)p[1] << 16) | ((uint32_t)p[2] << 8) | p[3]; }

void put32(std::vector<uint8_t>& v, uint32_t x) {
  v.push_back((uint8_t)(x >> 24));
  v.push_back((uint8_t)(x >> 16));
  v.push_back((uint8_t)(x >> 8));
  v.push_back((uint8_t)x);
}

uint8_t paeth(int a, int b, int c) {
  const int p = a + b - c;
  const int pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
  if (pa <= pb && pa <= pc) return (uint8_t)a;
  if (pb <= pc) return (uint8_t)b;
  return (uint8_t)c;
}

// Undo the per-row filters of a (sub)image in place: rows of `stride` bytes,
// each preceded by its filter byte.  Returns false on a bad filter type.
bool unfilter(uint8_t* data, int rows, size_t stride, int bpp, std::vector<uint8_t>& out) {
  out.assign((size_t)rows * stride, 0);
  for (int r = 0; r < rows; r++) {
    const uint8_t ft = data[(size_t)r * (stride + 1)];
    const uint8_t* src = data + (size_t)r * (stride + 1) + 1;
    uint8_t* cur = out.data() + (size_t)r * stride;
    const uint8_t* prev = r ? cur - stride : nullptr;
    for (size_t i = 0; i < stride; i++) {
      const int a = i >= (size_t)bpp ? cur[i - bpp] : 0;
      const int b = prev ? prev[i] : 0;
      const int c = (prev && i >= (size_t)bpp) ? prev[i - bpp] : 0;
      int v;
      switch (ft) {
        case 0: v = src[i]; break;
        case 1: v = src[i] + a; break;
        case 2: v = src[i] + b; break;
        case 3: v = src[i] + ((a + b) >> 1); break;
        case 4: v = src[i] + paeth(a, b, c); break;
        default: return false;
      }
      cur[i] = (uint8_t)v;
    }
  }
  return true;
}

}  // namespace

bool png_decode(const std::vector<uint8_t>& f, const std::string& source, Rgb8& img, std::string& err) {
  if (f.size() < 8 || memcmp(f.data(), kSig, 8) != 0) { err = source + ": not a PNG file"; return false; }
  size_t pos = 8;
  uint32_t w = 0, h = 0;
  int depth = 0, ctype = -1, interlace = 0;
  std::vector<uint8_t> idat, palette;
  bool seen_ihdr = false, seen_iend = false;
  while (pos + 12 <= f.size() && !seen_iend) {
    const uint32_t len = be32(&f[pos]);
    if (pos + 12 + (size_t)len > f.size()) { err = source + ": truncated chunk"; return false; }
    const uint8_t* type = &f[pos + 4];
    const uint8_t* data = &f[pos + 8];
    const uint32_t crc = be32(&f[pos + 8 + len]);
    if ((uint32_t)crc32(crc32(0L, Z_NULL, 0), type, len + 4) != crc) { err = source + ": chunk CRC mismatch"; return false; }
    if (!memcmp(type, "IHDR", 4)) {
      if (len < 13) { err = source + ": bad IHDR"; return false; }
      w = be32(data);
      h = be32(data + 4);
      depth = data[8];
      ctype = data[9];
      interlace = data[12];
      seen_ihdr = true;
    } else if (!memcmp(type, "PLTE", 4)) {
      palette.assign(data, data + len);
    } else if (!memcmp(type, "IDAT", 4)) {
      idat.insert(idat.end(), data, data + len);
    } else if (!memcmp(type, "IEND", 4)) {
      seen_iend = true;
    }
    pos += 12 + (size_t)len;
  }
  if (!seen_ihdr) { err = source + ": missing IHDR"; return false; }
  if (w == 0 || h == 0 || w > (1u << 16) || h > (1u << 16)) { err = source + ": unsupported PNG size"; return false; }
  if (depth != 8 && depth != 16) { err = "unsupported PNG bit depth " + std::to_string(depth); return false; }
  int channels;
  switch (ctype) {
    case 0: channels = 1; break;
    case 2: channels = 3; break;
    case 3: channels = 1; break;
    case 4: channels = 2; break;
    case 6: channels = 4; break;
    default: err = source + ": bad PNG color type"; return false;
  }
  const int sb = depth / 8;
  const int bpp = channels * sb;

  // Adam7 pass geometry (x0, y0, dx, dy); a non-interlaced image is one pass.
  const int passes_i[7][4] = {{0, 0, 8, 8}, {4, 0, 8, 8}, {0, 4, 4, 8}, {2, 0, 4, 4}, {0, 2, 2, 4}, {1, 0, 2, 2}, {0, 1, 1, 2}};
  const int pass_one[1][4] = {{0, 0, 1, 1}};
  const int npass = interlace ? 7 : 1;
  size_t need = 0;
  for (int p = 0; p < npass; p++) {
    const int* g = interlace ? passes_i[p] : pass_one[0];
    const size_t pw = (w > (uint32_t)g[0]) ? (w - g[0] + g[2] - 1) / g[2] : 0;
    const size_t ph = (h > (uint32_t)g[1]) ? (h - g[1] + g[3] - 1) / g[3] : 0;
    if (pw && ph) need += ph * (1 + pw * bpp);
  }
  std::vector<uint8_t> raw(need);
  z_stream zs;
  memset(&zs, 0, sizeof(zs));
  if (inflateInit(&zs) != Z_OK) { err = "zlib init failed"; return false; }
  // zlib counts in 32-bit uInt: feed and drain at most 1 GiB per call so that
  // images whose compressed or raw data exceed 4 GiB are read whole
  const size_t kStep = size_t(1) << 30;
  size_t in_pos = 0, out_pos = 0;
  int zr = Z_OK;
  while (zr == Z_OK) {
    if (zs.avail_in == 0 && in_pos < idat.size()) {
      const size_t n = std::min(kStep, idat.size() - in_pos);
      zs.next_in = idat.data() + in_pos;
      zs.avail_in = (uInt)n;
      in_pos += n;
    }
    if (zs.avail_out == 0 && out_pos < raw.size()) {
      const size_t n = std::min(kStep, raw.size() - out_pos);
      zs.next_out = raw.data() + out_pos;
      zs.avail_out = (uInt)n;
      out_pos += n;
    }
    const uInt in_before = zs.avail_in, out_before = zs.avail_out;
    zr = inflate(&zs, Z_NO_FLUSH);
    if (zr == Z_OK && zs.avail_in == in_before && zs.avail_out == out_before) break;  // no progress
    if (zr == Z_BUF_ERROR) break;
  }
  const size_t got = out_pos - zs.avail_out;
  inflateEnd(&zs);
  if ((zr != Z_STREAM_END && zr != Z_BUF_ERROR) || got < need) { err = source + ": corrupt image data"; return false; }

  // full-resolution samples, bpp bytes per pixel
  std::vector<uint8_t> px((size_t)w * h * bpp);
  size_t off = 0;
  std::vector<uint8_t> rows;
  for (int p = 0; p < npass; p++) {
    const int* g = interlace ? passes_i[p] : pass_one[0];
    const size_t pw = (w > (uint32_t)g[0]) ? (w - g[0] + g[2] - 1) / g[2] : 0;
    const size_t ph = (h > (uint32_t)g[1]) ? (h - g[1] + g[3] - 1) / g[3] : 0;
    if (!pw || !ph) continue;
    const size_t stride = pw * bpp;
    if (!unfilter(raw.data() + off, (int)ph, stride, bpp, rows)) { err = source + ": bad PNG filter"; return false; }
    off += ph * (stride + 1);
    for (size_t r = 0; r < ph; r++)
      for (size_t c = 0; c < pw; c++) {
        const size_t y = g[1] + r * g[3], x = g[0] + c * g[2];
        memcpy(&px[(y * w + x) * bpp], &rows[r * stride + c * bpp], bpp);
      }
  }
  img.width = (int)w;
  img.height = (int)h;
  img.data.assign((size_t)w * h * 3, 0);
  const size_t pal_entries = palette.size() / 3;
  for (size_t i = 0; i < (size_t)w * h; i++) {
    auto s = [&](int c) { return px[i * bpp + c * sb]; };  // high byte of 16-bit samples
    uint8_t r, gg, b;
    switch (ctype) {
      case 2: case 6: r = s(0); gg = s(1); b = s(2); break;
      case 0: case 4: r = gg = b = s(0); break;
      default: {
        const size_t idx = std::min<size_t>(s(0), pal_entries ? pal_entries - 1 : 0);
        const size_t o = idx * 3;
        if (o + 2 < palette.size()) { r = palette[o]; gg = palette[o + 1]; b = palette[o + 2]; }
        else { r = gg = b = 0; }
      }
    }
    img.data[i * 3] = r;
    img.data[i * 3 + 1] = gg;
    img.data[i * 3 + 2] = b;
  }
  return true;
}

bool png_encode(const Rgb8& img, std::vector<uint8_t>& out, std::string& err) {
  const size_t stride = (size_t)img.width * 3;
  std::vector<uint8_t> filtered((size_t)img.height * (stride + 1));
  for (int y = 0; y < img.height; y++) {
    uint8_t* d = &filtered[(size_t)y * (stride + 1)];
    const uint8_t* s = &img.data[(size_t)y * stride];
    d[0] = 1;  // Sub
    for (size_t i = 0; i < stride; i++) d[1 + i] = (uint8_t)(s[i] - (i >= 3 ? s[i - 3] : 0));
  }
  uLongf zlen = compressBound((uLong)filtered.size());
  std::vector<uint8_t> z(zlen);
  if (compress2(z.data(), &zlen, filtered.data(), (uLong)filtered.size(), 6) != Z_OK) {
    err = "zlib compression failed";
    return false;
  }
  z.resize(zlen);
  out.assign(kSig, kSig + 8);
  auto chunk = [&](const char* type, const uint8_t* data, size_t len) {
    put32(out, (uint32_t)len);
    const size_t start = out.size();
    out.insert(out.end(), type, type + 4);
    out.insert(out.end(), data, data + len);
    put32(out, (uint32_t)crc32(crc32(0L, Z_NULL, 0), &out[start], (uInt)(len + 4)));
  };
  std::vector<uint8_t> ihdr;
  put32(ihdr, (uint32_t)img.width);
  put32(ihdr, (uint32_t)img.height);
  ihdr.push_back(8);  // depth
  ihdr.push_back(2);  // RGB
  ihdr.push_back(0);
  ihdr.push_back(0);
  ihdr.push_back(0);
  chunk("IHDR", ihdr.data(), ihdr.size());
  // a chunk's length field tops out at 2^31 - 1: the stream goes out in 1 MiB IDAT chunks
  const size_t kIdat = size_t(1) << 20;
  for (size_t o = 0; o < z.size(); o += kIdat) chunk("IDAT", z.data() + o, std::min(kIdat, z.size() - o));
  chunk("IEND", nullptr, 0);
  return true;
}

}  // namespace lama_host
