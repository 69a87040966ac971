// OutConv 7x7 64 -> 3 + bias + sigmoid with every input row read once (outconv.cu).
#pragma once

#include <cstdint>

#include <cuda.h>
#include <cuda_runtime.h>

#include "pointwise.cuh"

namespace lama {

struct OutConvParams {
  CUtensorMap amap;   // input: split bf16 (64, W + 6, H + 6, B, part), boxes of 64 x 32 x 1, 128B swizzle
  CUtensorMap wmap;   // weights: split bf16 [2][160][64], n = ky * 21 + kx * 3 + co, boxes of 64 x 160
  const float* bias;  // [3]
  float* out;         // [B][3][H][W] fp32 (unused when dst is set)
  // Composite + quantise instead of the fp32 store (the u8 path, lama-rs
  // src/main.rs:272-307): for image pixels (y < ih, x < iw) of the padded
  // output where mask != 0, dst = (u8)(int)(clamp(v, 0, 1) * 255 + 0.5); the
  // plan copies rgb into dst beforehand, which gives the unmasked bytes.
  // dst [B][ih][iw][3], mask [B][ih][iw].
  const uint8_t* mask;
  uint8_t* dst;
  int ih, iw;
  // window mode (one --sections pass, batch 1): write the fill into win->img
  // at the window's place, where the mask is set inside the section rectangle
  const WinDesc* win;
  int batch, h, w;
  int strips, segs, seg;  // filled by outconv_units (seg = output rows per segment)
  int* err;           // device status word
};

int outconv_prepare();
void outconv_units(OutConvParams& q, int sms);
int launch_outconv(const OutConvParams& q, int sms, cudaStream_t st);

}  // namespace lama
