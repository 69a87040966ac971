// Data-movement kernels at the two ends of the pass, and layout conversions.
//
// k_unfold_*  : the network input, ReflectionPad2d(3) and model.1's 7x7 taps
//               along x, in one pass.  Replaces the host `build_input`
//               (lama-rs/src/main.rs:175-196, pad to a multiple of 8 at
//               :241-242), the k_reflect_pad launch (lama-rs/src/cuda.rs:1227-1240)
//               and model.1's im2col (K = 196, lama-rs/src/cuda.rs:991-1005).
//               The output U[b][y][x][kx*4 + c] (32 channels, 28 used) is the
//               A operand of model.1: seven taps along x packed into channels,
//               so the 7x7 conv becomes 8 row-taps of 32 channels.
// (The mask composite + u8 quantisation, lama-rs/src/main.rs:272-307, runs in
// the OutConv epilogue, outconv.cu.)
// k_nchw_to_split / k_split_to_nchw : the resblock-stack entry point's layout
//               conversions (fp32 NCHW <-> split-bf16 NHWC with reflect halo).
#include <cstdint>

#include "pointwise.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace lama {

namespace {

__device__ __forceinline__ int reflect_i(int i, int n) {
  if (n == 1) return 0;
  int period = 2 * (n - 1);
  int m = i % period;
  if (m < 0) m += period;
  return m >= n ? period - m : m;
}

// Value of network input channel c (0..3) at padded-image pixel (y, x) of an
// image of the padded size H x W, for the u8 source (build_input semantics:
// the padded image is the reflect extension of the h x w original).
__device__ __forceinline__ void input_px_u8(const uint8_t* rgb, const uint8_t* mask, int h, int w, int y, int x,
                                            float* v4) {
  const int sy = reflect_i(y, h), sx = reflect_i(x, w);
  float m = (float)mask[(size_t)sy * w + sx] / 255.0f;
  m = m > 0.0f ? 1.0f : 0.0f;
  const uint8_t* px = rgb + ((size_t)sy * w + sx) * 3;
  const float om = 1.0f - m;
#pragma unroll
  for (int c = 0; c < 3; c++) {
    const float v = (float)px[c] / 255.0f;
    v4[c] = v * om;
  }
  v4[3] = m;
}

template <bool U8>
__global__ void k_unfold(UnfoldParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const long long total = (long long)p.batch * (p.H + 6) * p.W;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int x = (int)(idx % p.W);
  const long long t = idx / p.W;
  const int y = (int)(t % (p.H + 6));
  const int b = (int)(t / (p.H + 6));
  const int yy = reflect_i(y - 3, p.H);
  float v[32];
#pragma unroll
  for (int kx = 0; kx < 7; kx++) {
    const int xx = reflect_i(x + kx - 3, p.W);
    if constexpr (U8) {
      if (p.win) {
        // window pixel (reflect-extended inside the side x side window) of the working image
        const WinDesc& d = *p.win;
        const int gy = d.wy0 + reflect_i(yy, p.h), gx = d.wx0 + reflect_i(xx, p.w);
        const bool in = gx >= d.sx0 && gx < d.sx1 && gy >= d.sy0 && gy < d.sy1;
        const float m = in && d.mask[(size_t)gy * d.fw + gx] != 0 ? 1.0f : 0.0f;
        const uint8_t* px = d.img + ((size_t)gy * d.fw + gx) * 3;
        const float om = 1.0f - m;
#pragma unroll
        for (int c = 0; c < 3; c++) v[4 * kx + c] = ((float)px[c] / 255.0f) * om;
        v[4 * kx + 3] = m;
        continue;
      }
      const uint8_t* rgb = p.rgb + (size_t)b * p.h * p.w * 3;
      const uint8_t* mask = p.mask + (size_t)b * p.h * p.w;
      input_px_u8(rgb, mask, p.h, p.w, yy, xx, v + 4 * kx);
    } else {
      const float* in = p.in + (size_t)b * 4 * p.H * p.W;
#pragma unroll
      for (int c = 0; c < 4; c++) v[4 * kx + c] = in[((size_t)c * p.H + yy) * p.W + xx];
    }
  }
#pragma unroll
  for (int c = 28; c < 32; c++) v[c] = 0.f;
  uint32_t hi[16], lo[16];
#pragma unroll
  for (int k = 0; k < 16; k++) split_pair(v[2 * k], v[2 * k + 1], hi[k], lo[k]);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
  const size_t off = (size_t)idx * 32;
  uint4* dh = reinterpret_cast<uint4*>(out + off);
  uint4* dl = reinterpret_cast<uint4*>(out + p.out_part + off);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    dh[k] = make_uint4(hi[4 * k], hi[4 * k + 1], hi[4 * k + 2], hi[4 * k + 3]);
    dl[k] = make_uint4(lo[4 * k], lo[4 * k + 1], lo[4 * k + 2], lo[4 * k + 3]);
  }
}

// fp32 NCHW [B][C][h][w] -> channels [c0, c0+C) of split NHWC [2][B][h+2halo][w+2halo][Ct], reflect halo
__global__ void k_nchw_to_split(ConvertParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const long long total = (long long)p.batch * (p.h + 2 * p.halo) * (p.w + 2 * p.halo) * p.c;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = (int)(idx % p.c);
  long long t = idx / p.c;
  const int wp = p.w + 2 * p.halo, hp = p.h + 2 * p.halo;
  const int xp = (int)(t % wp);
  t /= wp;
  const int yp = (int)(t % hp);
  const int b = (int)(t / hp);
  const int y = reflect_i(yp - p.halo, p.h), x = reflect_i(xp - p.halo, p.w);
  const float v = p.nchw[(((size_t)b * p.c + c) * p.h + y) * p.w + x];
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.split);
  const size_t off = (((size_t)b * hp + yp) * wp + xp) * p.ctot + p.c0 + c;
  out[off] = hi;
  out[p.part + off] = __float2bfloat16_rn(v - __bfloat162float(hi));
}

__global__ void k_split_to_nchw(ConvertParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const long long total = (long long)p.batch * p.c * p.h * p.w;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int x = (int)(idx % p.w);
  long long t = idx / p.w;
  const int y = (int)(t % p.h);
  t /= p.h;
  const int c = (int)(t % p.c);
  const int b = (int)(t / p.c);
  const int wp = p.w + 2 * p.halo, hp = p.h + 2 * p.halo;
  const __nv_bfloat16* in = reinterpret_cast<const __nv_bfloat16*>(p.split);
  const size_t off = (((size_t)b * hp + y + p.halo) * wp + x + p.halo) * p.ctot + p.c0 + c;
  p.nchw[idx] = __bfloat162float(in[off]) + __bfloat162float(in[p.part + off]);
}

inline unsigned blocks_for(long long n, int bs) { return (unsigned)((n + bs - 1) / bs); }

}  // namespace

int launch_unfold_f32(const UnfoldParams& p, cudaStream_t st) {
  const long long n = (long long)p.batch * (p.H + 6) * p.W;
  return launch_kernel(k_unfold<false>, dim3(blocks_for(n, 128)), dim3(128), 0, st, 1, p);
}

int launch_unfold_u8(const UnfoldParams& p, cudaStream_t st) {
  const long long n = (long long)p.batch * (p.H + 6) * p.W;
  return launch_kernel(k_unfold<true>, dim3(blocks_for(n, 128)), dim3(128), 0, st, 1, p);
}

int launch_nchw_to_split(const ConvertParams& p, cudaStream_t st) {
  const long long n = (long long)p.batch * (p.h + 2 * p.halo) * (p.w + 2 * p.halo) * p.c;
  return launch_kernel(k_nchw_to_split, dim3(blocks_for(n, 256)), dim3(256), 0, st, 1, p);
}

int launch_split_to_nchw(const ConvertParams& p, cudaStream_t st) {
  const long long n = (long long)p.batch * p.c * p.h * p.w;
  return launch_kernel(k_split_to_nchw, dim3(blocks_for(n, 256)), dim3(256), 0, st, 1, p);
}

}  // namespace lama
