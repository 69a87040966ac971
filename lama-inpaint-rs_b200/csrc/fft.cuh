// FourierUnit transform kernels (fft.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace lama {

// Division by a divisor fixed at plan time (Granlund & Montgomery, "Division
// by invariant integers using multiplication", 1994, round-up variant):
// x / d = (umulhi(x, m) + x) >> s for 0 <= x < 2^31.
struct FastDiv {
  unsigned d, m, s;
};

inline FastDiv make_fastdiv(unsigned d) {
  FastDiv f{d, 0, 0};
  while ((1u << f.s) < d) f.s++;
  f.m = (unsigned)((((unsigned long long)1 << 32) * (((unsigned long long)1 << f.s) - d)) / d + 1);
  return f;
}

#ifdef __CUDACC__
__device__ __forceinline__ unsigned fdiv(unsigned x, const FastDiv& f) { return (__umulhi(x, f.m) + x) >> f.s; }
#endif

// One Stockham stage: radix R, Ns = product of the radices before it, and
// the divisors its index arithmetic needs (m = n / R).
struct FftStage {
  int r;
  FastDiv m, ns, rr, nsr;
};

// The stages of one line length n (product of the radices = n).
struct Radices {
  int n;
  FastDiv len;
  FftStage st[12];
};

struct FftParams {
  int batch, c;            // images, real channels (the spectrum has 2c)
  int h, w, wh;            // plane, wh = w/2 + 1
  int log2h, log2w;        // log2 of a power-of-two length, else -1
  int cg;                  // fft.cu: channels per CTA of the column and inverse-row passes
  int kb;                  // fft.cu: columns (kx) per CTA of the column passes
  int rp;                  // fft.cu: row pairs per CTA of the forward row pass
  int rpi;                 // fft.cu: row pairs per CTA of the inverse row pass
  float scale;             // 1/sqrt(h*w)
  const float2* tw_h;      // (cos, sin)(2 pi k / h), k < h
  const float2* tw_w;      // (cos, sin)(2 pi k / w), k < w
  const float* feat;       // [B][c][h][w] fp32 (NCHW): rfft2 input / irfft2 residual
  void* spec;              // rfft2 out: split bf16 [2][B][h][wh][2c]
  long long spec_part;
  const float* fu;         // irfft2 in: fp32 [B][h][wh][2c]
  void* s_out;             // irfft2 out: split bf16 [2][B][h][w][c] = feat + irfft2(fu)
  long long s_part;
  float2* tmp;             // fft.cu: intermediate, fft_tmp_elems(p) complex values
  Radices rad_h, rad_w;    // fft.cu: stages of the column / row transforms
  FastDiv fd_w, fd_h, fd_cg, fd_kb, fd_rows;  // fft.cu: w, h, cg, kb, 2 * rp
  int* err;                // device status word (bounded waits of the prefetching kernel)
};

// The prefetching rfft2 of 64 x 64 planes (fft_reg.cu): feat_map views feat
// as rows (x: 64 floats, rows: B * c * 64), boxes of 32 x 256, 128-byte swizzle.
struct FftPfParams {
  CUtensorMap feat_map;
  FftParams p;
};

// The tensor-core rfft2 of 64 x 64 planes (fft_tc.cu): map views feat as rows
// of 64 floats with boxes of 32 x 128 (two channels' x-halves), 128-byte
// swizzle; tab is the device copy of fft_tc_table (the two DFT matrices).
struct FftTcParams {
  CUtensorMap map;
  FftParams p;
  const void* tab;
};
bool fft_tc_supported(int c, int h, int w);
size_t fft_tc_table_bytes();
void fft_tc_table(uint8_t* out);  // fft_tc_table_bytes() bytes
int fft_tc_prepare();
int launch_rfft2_tc(const FftTcParams& q, int grid, cudaStream_t st);

// Two-pass kernels for any plane size (fft.cu).  fft_tiles fills cg/kb/rp/rpi
// from c, h, w so that every pass fits max_smem (false if none does);
// pass 0 = rows_fwd, 1 = the column passes, 2 = rows_inv.
bool fft_tiles(FftParams& p, size_t max_smem);
Radices fft_radices(int n);
size_t fft_smem_bytes(const FftParams& p, int pass);
size_t fft_tmp_elems(const FftParams& p);
int fft_prepare(size_t max_smem);
int launch_rfft2(const FftParams& p, cudaStream_t st);
int launch_irfft2(const FftParams& p, cudaStream_t st);

// Register-resident kernels for power-of-two planes with sides in {8..64}
// (fft_reg.cu).
bool fft_reg_supported(int h, int w);
bool fft_pf_supported(int c, int h, int w);
int fft_pf_prepare();
int launch_rfft2_pf(const FftPfParams& q, int grid, cudaStream_t st);
// irfft2 of 64 x 64 planes split by output-row parity, 16 channels per CTA,
// or 4 where 16-channel CTAs would not cover the `sms` SMs (fft_reg.cu);
// needs c % 16 == 0.
int launch_irfft2_par(const FftParams& p, int sms, cudaStream_t st);
bool irfft2_par_narrow(int c, int batch, int sms);
int fft_reg_prepare();
int launch_fft_reg(const FftParams& p, bool inverse, cudaStream_t st);

}  // namespace lama
