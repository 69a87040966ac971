// Parameter block of the implicit-GEMM convolution kernel (conv_gemm.cu).
//
// One launch computes  out[pixel][n] = epilogue( sum_k A[pixel][k] * B[n][k] )
// over one or more "tile classes".  A class owns a range of output channels
// and its own K list; K is a concatenation of segments, each a convolution
// (a list of taps) over a channel range of one activation tensor.  This is
// how one launch expresses:
//   * a plain KxK convolution (one class, one segment),
//   * an FFC layer's two outputs with concatenated K (local: 3x3 over all 512
//     channels = l2l|g2l; global: 3x3 over the 128 local channels then the
//     1x1 spectral conv2 = l2g|conv2), as two classes of one launch,
//   * a stride-2 transposed convolution as its four output phases (four
//     classes with 1, 2, 2, 4 taps and strided output placement).
//
// Activations are NHWC and carried as split bf16 pairs: a buffer
// [2][B][H+2h][W+2h][C] holds hi = bf16(v) in part 0 and lo = bf16(v - hi)
// in part 1, with an optional halo h of reflected pixels.  A tensor maps
// address them as 5-D (C, Wp, Hp, B, part).  Weights are [2][N][K] bf16
// (hi/lo), addressed as 3-D (K, N, part).
#pragma once

#include <cuda.h>
#include <cstdint>

namespace lama {

constexpr int GEMM_MAX_TAPS = 49;
constexpr int GEMM_MAX_SEGS = 2;
constexpr int GEMM_MAX_CLASSES = 4;
constexpr int GEMM_MAX_AMAPS = 3;
constexpr int GEMM_MAX_GROUPS = 8;
constexpr int GEMM_MAX_KSPLIT = 8;

enum OutKind : int {
  OUT_SPLIT = 0,     // split bf16 NHWC (optionally halo'd, reflect-filled)
  OUT_F32_NHWC = 1,  // fp32 NHWC
  OUT_F32_NCHW = 2,  // fp32 NCHW, channels < nvalid only
};

struct GemmSeg {
  int amap;    // index into GemmParams::amap
  int c0;      // first channel of this segment in the A tensor
  int nblk;    // CB-channel blocks per tap
  int ntaps;   // taps
  int stride;  // the tile origin is multiplied by this in A coordinates
  int sub0;    // index of the segment's first A sub-box within its class
  int8_t dy[GEMM_MAX_TAPS];  // tap offsets in A map coordinates
  int8_t dx[GEMM_MAX_TAPS];
};

// Row-union mode: taps of one segment that share dx and have consecutive dy
// (up to 3 with 64-channel boxes; 2 or 4 whole K blocks with 32-channel
// boxes) form a group; per channel block the group's A tiles are the row
// windows of ONE box of bh + ndy - 1 rows, loaded once.
struct GemmGroup {
  int8_t seg, dx, dy0, ndy;
  int8_t tap[4];
};

struct GemmClass {
  int n0;        // first output channel (absolute, indexes scale/shift and out)
  int nvalid;    // output channels in this class
  int ntiles_n;  // BN-wide tiles covering nvalid
  int nkb;       // 64-wide K blocks
  int nseg;
  int oy_mul, oy_add, ox_mul, ox_add;  // output pixel = M pixel * mul + add
  int tile0;     // first global tile index of the class
  int ksplit;    // K parts per output tile (split-K; 1 = none)
  int ws_tile0;  // first workspace slice of the class (split-K)
  // K parts [part0, part0 + nparts) of every output tile run in this launch
  // (the others in another launch sharing the workspace and counters; the
  // part that arrives last finishes the tile); part q covers K units
  // [kcut[q], kcut[q + 1]): 64-wide K blocks, or row-union iterations (one
  // per group and channel block, in group order) when GemmParams::uni is set
  int part0, nparts;
  int16_t kcut[GEMM_MAX_KSPLIT + 1];
  GemmSeg seg[GEMM_MAX_SEGS];
  int ngroup;    // row-union mode: groups of the class's taps
  GemmGroup grp[GEMM_MAX_GROUPS];
};

struct GemmParams {
  CUtensorMap amap[GEMM_MAX_AMAPS];
  CUtensorMap bmap[GEMM_MAX_CLASSES];
  // row-union mode (uni = 1; tiles of bh = 4 x bw = 32 pixels, 64- or
  // 32-channel boxes, stride 1, no split-K, BN = 64 or CTA pairs of BN = 128): per A map
  // a map of boxes of urows = bh + (longest group) - 1 rows, both parts
  CUtensorMap amap_u[GEMM_MAX_AMAPS];
  int uni;
  int urows[GEMM_MAX_AMAPS];
  // ostore != 0: the output leaves through TMA tensor stores of one box per
  // epilogue warp and 32-channel chunk (32 channels x obox_w x 32 / obox_w
  // pixels).  omap[c] views class c's output pixels (output = M pixel * mul +
  // add) as a dense grid indexed by M-space (j, i): 1 = split,
  // (C, W/mul, H/mul, B, part) from the class's first interior pixel, 64-byte
  // swizzled (boxes clip at the interior's far edges; reflected halo copies
  // are ordinary stores); 2 = fp32 NCHW (W, H, C, B); 3 = fp32 NHWC
  // (C, W, H, B), 128-byte swizzled.
  CUtensorMap omap[GEMM_MAX_CLASSES];
  int ostore, obox_w;
  GemmClass cls[GEMM_MAX_CLASSES];
  int nclass;
  int swap;                   // 1: M = 128 output channels, N = BN pixels (see conv_gemm.cu)
  int pair;                   // 1: clusters of two CTAs, 256 x BN tiles (see conv_gemm.cu); the grid is
                              //    2 x clusters and tiles count pair tiles
  int cb;                     // channels per A sub-box: 64 (128B swizzle) or 32 (64B swizzle)
  int batch, mh, mw;          // M space: images x rows x cols
  int bh, bw;                 // tile rows x cols, bh * bw == 128
  int tiles_y, tiles_x, m_tiles;
  int total_tiles;
  // epilogue
  const float* scale;         // per absolute output channel
  const float* shift;
  int relu;
  int sigmoid;
  int out_kind;
  void* out;
  long long out_part;         // elements per part of a split output
  int out_c, out_h, out_w;    // output tensor channels and interior extent
  int out_halo, out_reflect;  // halo width; fill it by reflection
  const void* skip;           // split residual, same geometry as out (may alias it)
  // split-K (classes with ksplit > 1): fp32 partial sums, one [BN][128] slice
  // per part of each output tile (with CTA pairs: of each CTA's 128-pixel
  // half), and one arrival counter per output tile (indexed by its part-0
  // slice), zero between launches (the CTA that finishes a tile resets it)
  float* ws;
  int* cnt;
  // optional static schedule: slot s (a CTA, or a CTA pair) runs tiles
  // sched[sched_off[s] .. sched_off[s + 1]) in order; null = round robin
  const int* sched;
  const int* sched_off;
  int* err;                   // device status word (0 = ok)
};

static_assert(sizeof(GemmParams) <= 4096, "GemmParams must fit the kernel parameter space");

// Host launcher (conv_gemm.cu).  `bn` in {16, 32, 64, 128, 192, 256}.
int launch_conv_gemm(const GemmParams& p, int bn, int grid, cudaStream_t stream);
size_t conv_gemm_smem_bytes(int bn);
int conv_gemm_stages(int bn);
int conv_gemm_prepare();
bool conv_gemm_pair_bn(int bn);  // tile widths with a CTA-pair kernel
int conv_gemm_pair_clusters();   // co-resident clusters of the pair kernel (after conv_gemm_prepare)

}  // namespace lama
