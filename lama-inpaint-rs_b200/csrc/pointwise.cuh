// Input / output / layout kernels (pointwise.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace lama {

struct UnfoldParams {
  int batch;
  int H, W;                // network input size (multiples of 8)
  int h, w;                // u8 source image size (<= H, W; reflect-extended)
  const float* in;         // f32 NCHW [B][4][H][W]
  const uint8_t* rgb;      // u8 [B][h][w][3]
  const uint8_t* mask;     // u8 [B][h][w]
  void* out;               // split bf16 [2][B][H+6][W][32]
  long long out_part;
};

// The u8 path's composite (fused into the OutConv, outconv.cu).
struct CompositeParams {
  int batch, h, w, H, W;
  const uint8_t* rgb;      // [B][h][w][3]
  const uint8_t* mask;     // [B][h][w]
  const float* net;        // [B][3][H][W] sigmoid output (unused by the fused composite)
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
