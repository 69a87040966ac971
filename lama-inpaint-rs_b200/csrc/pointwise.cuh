// Input / output / layout kernels (pointwise.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace lama {

// One --sections pass on a device-resident image (lama-rs/src/main.rs:465-566):
// the pass's window (side x side at wx0, wy0) of the working image img and
// the mask, with the mask restricted to the section rectangle
// [sx0, sx1) x [sy0, sy1); the fill is written back into img.  Kernels read
// it from device memory at run time, so one captured plan serves every pass.
struct WinDesc {
  uint8_t* img;          // u8 [fh][fw][3], read and updated in place
  const uint8_t* mask;   // u8 [fh][fw]
  int fw, fh;
  int wx0, wy0;
  int sx0, sy0, sx1, sy1;
};

struct UnfoldParams {
  int batch;
  int H, W;                // network input size (multiples of 8)
  int h, w;                // u8 source image size (<= H, W; reflect-extended)
  const float* in;         // f32 NCHW [B][4][H][W]
  const uint8_t* rgb;      // u8 [B][h][w][3]
  const uint8_t* mask;     // u8 [B][h][w]
  void* out;               // split bf16 [2][B][H+6][W][32]
  long long out_part;
  const WinDesc* win;      // window mode (batch 1): read rgb / mask through the descriptor
};

// The u8 path's composite (fused into the OutConv, outconv.cu).
struct CompositeParams {
  int batch, h, w, H, W;
  const uint8_t* rgb;      // [B][h][w][3]
  const uint8_t* mask;     // [B][h][w]
  uint8_t* dst;            // [B][h][w][3]
};

struct ConvertParams {
  int batch, c, h, w, halo, ctot, c0;
  float* nchw;
  void* split;
  long long part;
};

int launch_unfold_f32(const UnfoldParams& p, cudaStream_t st);
int launch_unfold_u8(const UnfoldParams& p, cudaStream_t st);
int launch_nchw_to_split(const ConvertParams& p, cudaStream_t st);
int launch_split_to_nchw(const ConvertParams& p, cudaStream_t st);

}  // namespace lama
