// FourierUnit transform kernels (fft.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace lama {

struct FftParams {
  int batch, c;            // images, real channels (the spectrum has 2c)
  int h, w, wh;            // plane, wh = w/2 + 1
  int log2h, log2w;        // log2 of a power-of-two length, else -1
  int cg;                  // channels per CTA
  int lmax;                // max(h, w): line buffer length
  float scale;             // 1/sqrt(h*w)
  const float2* tw_h;      // (cos, sin)(2 pi k / h), k < h
  const float2* tw_w;      // (cos, sin)(2 pi k / w), k < w
  const float* feat;       // [B][c][h][w] fp32 (NCHW): rfft2 input / irfft2 residual
  void* spec;              // rfft2 out: split bf16 [2][B][h][wh][2c]
  long long spec_part;
  const float* fu;         // irfft2 in: fp32 [B][h][wh][2c]
  void* s_out;             // irfft2 out: split bf16 [2][B][h][w][c] = feat + irfft2(fu)
  long long s_part;
};

size_t fft_smem_bytes(const FftParams& p);
int fft_prepare(size_t max_smem);
int launch_rfft2(const FftParams& p, cudaStream_t st);
int launch_irfft2(const FftParams& p, cudaStream_t st);

// Register-resident kernels for power-of-two planes with sides in {8..64}
// (fft_reg.cu).
bool fft_reg_supported(int h, int w);
int fft_reg_prepare();
int launch_fft_reg(const FftParams& p, bool inverse, cudaStream_t st);

}  // namespace lama
