// Window and section geometry of the --tile and --sections modes.
//
// Restates the host-side helpers of the reference CLI (lama-rs/src/main.rs):
//   window_origin  main.rs:722-727
//   tile_rect      main.rs:740-777
//   section_rects  main.rs:597-659
//   mask_depth     main.rs:664-717
// with the same constants (TILE_MIN 512, SECTION_BLOCK 256, PAD_MOD 8) and
// the same deterministic ordering, so that --tile and --sections choose the
// same windows and passes as the reference.
#include <algorithm>
#include <climits>
#include <cstdint>
#include <deque>
#include <vector>

#include "lama_b200.h"

namespace {

constexpr int kPadMod = 8;
constexpr int kTileMin = 512;
constexpr int kSectionBlock = 256;

struct BBox {
  int min_x, min_y, max_x, max_y;
  long long count;
};

BBox bbox(const uint8_t* m, int w, int h) {
  BBox b{w, h, 0, 0, 0};
  for (int y = 0; y < h; y++)
    for (int x = 0; x < w; x++)
      if (m[(size_t)y * w + x]) {
        b.min_x = std::min(b.min_x, x);
        b.min_y = std::min(b.min_y, y);
        b.max_x = std::max(b.max_x, x);
        b.max_y = std::max(b.max_y, y);
        b.count++;
      }
  return b;
}

}  // namespace

extern "C" {

int lama_window_origin(int c, int side, int extent) {
  const int max0 = std::max(extent - side, 0);
  return std::clamp(c - side / 2, 0, max0);
}

int lama_tile_rect(const uint8_t* mask, int w, int h, int* out) {
  if (!mask || !out || w < 1 || h < 1) return LAMA_EINVAL;
  const BBox b = bbox(mask, w, h);
  if (b.count == 0) return 0;
  const int bw = b.max_x - b.min_x + 1, bh = b.max_y - b.min_y + 1;
  const int want = std::max(kTileMin, 2 * std::max(bw, bh));
  const int cap = std::min(w, h) / kPadMod * kPadMod;
  int side = cap >= kPadMod ? std::min((want + kPadMod - 1) / kPadMod * kPadMod, cap) : std::min(w, h);
  side = std::max(side, 1);
  const int cx = b.min_x + bw / 2, cy = b.min_y + bh / 2;
  out[0] = lama_window_origin(cx, side, w);
  out[1] = lama_window_origin(cy, side, h);
  out[2] = side;
  out[3] = bw;
  out[4] = bh;
  return 1;
}

int lama_mask_depth(const uint8_t* mask, int w, int h, uint32_t* depth) {
  if (!mask || !depth || w < 1 || h < 1) return LAMA_EINVAL;
  const size_t n = (size_t)w * h;
  std::fill(depth, depth + n, UINT32_MAX);
  std::deque<size_t> q;
  for (int y = 0; y < h; y++)
    for (int x = 0; x < w; x++) {
      const size_t i = (size_t)y * w + x;
      if (!mask[i]) continue;
      const bool rim = x == 0 || y == 0 || x + 1 == w || y + 1 == h || !mask[i - 1] || !mask[i + 1] ||
                       !mask[i - w] || !mask[i + w];
      if (rim) {
        depth[i] = 0;
        q.push_back(i);
      }
    }
  while (!q.empty()) {
    const size_t i = q.front();
    q.pop_front();
    const uint32_t d = depth[i];
    const int x = (int)(i % w), y = (int)(i / w);
    size_t nb[4];
    int k = 0;
    if (x > 0) nb[k++] = i - 1;
    if (x + 1 < w) nb[k++] = i + 1;
    if (y > 0) nb[k++] = i - w;
    if (y + 1 < h) nb[k++] = i + w;
    for (int j = 0; j < k; j++)
      if (mask[nb[j]] && depth[nb[j]] == UINT32_MAX) {
        depth[nb[j]] = d == UINT32_MAX ? d : d + 1;
        q.push_back(nb[j]);
      }
  }
  return 0;
}

int lama_section_rects(const uint8_t* mask, int w, int h, int* out, int cap) {
  if (!mask || w < 1 || h < 1) return LAMA_EINVAL;
  const BBox b = bbox(mask, w, h);
  if (b.count == 0) return 0;
  struct Cell {
    uint32_t depth;
    int x0, y0, x1, y1;
  };
  std::vector<Cell> cells;
  if (b.max_x - b.min_x + 1 <= kSectionBlock && b.max_y - b.min_y + 1 <= kSectionBlock) {
    cells.push_back({0, b.min_x, b.min_y, b.max_x + 1, b.max_y + 1});
  } else {
    std::vector<uint32_t> depth((size_t)w * h);
    lama_mask_depth(mask, w, h, depth.data());
    for (int y0 = b.min_y;; y0 += kSectionBlock) {
      for (int x0 = b.min_x;; x0 += kSectionBlock) {
        const int x1 = std::min(x0 + kSectionBlock, b.max_x + 1);
        const int y1 = std::min(y0 + kSectionBlock, b.max_y + 1);
        uint32_t shallowest = UINT32_MAX;
        for (int y = y0; y < y1; y++)
          for (int x = x0; x < x1; x++)
            if (mask[(size_t)y * w + x]) shallowest = std::min(shallowest, depth[(size_t)y * w + x]);
        if (shallowest != UINT32_MAX) cells.push_back({shallowest, x0, y0, x1, y1});
        if (x1 >= b.max_x + 1) break;
      }
      if (y0 + kSectionBlock >= b.max_y + 1) break;
    }
    std::stable_sort(cells.begin(), cells.end(), [](const Cell& a, const Cell& c) {
      if (a.depth != c.depth) return a.depth < c.depth;
      if (a.y0 != c.y0) return a.y0 < c.y0;
      return a.x0 < c.x0;
    });
  }
  const int n = (int)cells.size();
  if (out)
    for (int i = 0; i < n && i < cap; i++) {
      out[4 * i] = cells[i].x0;
      out[4 * i + 1] = cells[i].y0;
      out[4 * i + 2] = cells[i].x1;
      out[4 * i + 3] = cells[i].y1;
    }
  return n;
}

}  // extern "C"
