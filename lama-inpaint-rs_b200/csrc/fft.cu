// FourierUnit transforms: rfft2 / irfft2 with norm='ortho' over NHWC planes.
//
// Replaces the reference's spectral transform launches (lama-rs/src/cuda.rs
// :1460-1539: lg_fft2_r2c + k_spec_pack, k_spec_unpack + lg_fft2_c2r, and the
// lg_add_inplace of the FourierUnit residual) and restates the CPU engine's
// transform semantics (lama-rs/src/cpu.rs:769-1011):
//   * forward: row transforms then column transforms, bins 0..w/2, scaled by
//     1/sqrt(h*w); the stacked channel order (c.re, c.im) the 1x1 conv sees
//     (cpu.rs:281-285) is simply channels 2c, 2c+1 of the NHWC output;
//   * inverse: the 2-D Hermitian completion of cpu.rs:801-837, realised as
//     column transforms of the stored bins, then per row a real transform
//     that ignores the imaginary parts of the DC (and, for even w, Nyquist)
//     column - the two constructions are identical;
//   * a transform length that is not a power of two runs in the opposite
//     direction, as the reference's Bluestein code does (cpu.rs:984-1011 pairs
//     a_j = x_j*conj(w_j) with b = w, the conjugate of the chirps its
//     requested direction needs), so non-power-of-two planes match the
//     reference rather than torch.fft.
// The inverse fuses the FourierUnit residual: S = feat + irfft2(fu) is written
// as the split-bf16 operand of the closing 1x1 conv.
//
// One CTA transforms CG channels of one image: 8 warps, each warp owns a line
// buffer in shared memory and transforms one line at a time (radix-2 with
// warp-synchronous stages for powers of two, a direct DFT otherwise).  Two real
// rows are packed into one complex transform.  Arithmetic is fp32 with
// twiddles rounded from double.
#include <cmath>
#include <cstdint>

#include "fft.cuh"
#include "ptx.cuh"

namespace lama {

namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// In-place transform of L[0..n) by one warp.  `sign` = -1: sum x_j e^{-2 pi i jk/n},
// +1: e^{+...}.  `tw` holds (cos, sin)(2 pi k / n), k < n.  `tmp` is a second
// line buffer (used by the direct DFT).
__device__ void warp_line_transform(float2* L, float2* tmp, const float2* tw, int n, int log2n, int sign) {
  const int lane = threadIdx.x & 31;
  if (n <= 1) return;
  if (log2n >= 0) {
    for (int i = lane; i < n; i += 32) {
      int j = (int)(__brev((unsigned)i) >> (32 - log2n));
      if (i < j) {
        float2 t = L[i];
        L[i] = L[j];
        L[j] = t;
      }
    }
    __syncwarp();
    for (int len = 2, stride = n >> 1; len <= n; len <<= 1, stride >>= 1) {
      const int half = len >> 1;
      for (int bfly = lane; bfly < (n >> 1); bfly += 32) {
        const int g = bfly / half, k = bfly - g * half;
        const int i = g * len + k, j = i + half;
        float2 w = tw[k * stride];
        w.y *= (float)sign;
        const float2 v = cmul(L[j], w);
        const float2 u = L[i];
        L[i] = make_float2(u.x + v.x, u.y + v.y);
        L[j] = make_float2(u.x - v.x, u.y - v.y);
      }
      __syncwarp();
    }
  } else {
    for (int k = lane; k < n; k += 32) {
      float2 acc = make_float2(0.f, 0.f);
      int idx = 0;
      for (int j = 0; j < n; j++) {
        float2 w = tw[idx];
        w.y *= (float)sign;
        const float2 v = cmul(L[j], w);
        acc.x += v.x;
        acc.y += v.y;
        idx += k;
        if (idx >= n) idx -= n;
      }
      tmp[k] = acc;
    }
    __syncwarp();
    for (int k = lane; k < n; k += 32) L[k] = tmp[k];
    __syncwarp();
  }
}

__device__ __forceinline__ int direction(int log2n, bool inverse) {
  // powers of two: forward e^{-}, inverse e^{+}; otherwise swapped (see header)
  const bool fwd = (log2n >= 0) ? !inverse : inverse;
  return fwd ? -1 : 1;
}

struct Smem {
  float2* Z;      // [cg][h][wh]
  float2* lines;  // [warp][2][lmax]
  float2* tw_h;   // [h]
  float2* tw_w;   // [w]
};

__device__ Smem carve(const FftParams& p, uint8_t* base) {
  Smem s;
  s.Z = reinterpret_cast<float2*>(base);
  s.lines = s.Z + (size_t)p.cg * p.h * p.wh;
  s.tw_h = s.lines + kWarps * 2 * p.lmax;
  s.tw_w = s.tw_h + p.h;
  return s;
}

__device__ void load_twiddles(const FftParams& p, const Smem& s) {
  for (int i = threadIdx.x; i < p.h; i += blockDim.x) s.tw_h[i] = p.tw_h[i];
  for (int i = threadIdx.x; i < p.w; i += blockDim.x) s.tw_w[i] = p.tw_w[i];
}

__global__ void __launch_bounds__(256) k_rfft2(const FftParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const Smem s = carve(p, smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, c0 = blockIdx.x * p.cg;
  load_twiddles(p, s);
  __syncthreads();
  float2* L = s.lines + warp * 2 * p.lmax;
  float2* T = L + p.lmax;
  const int npairs = (p.h + 1) >> 1;
  const int sgn_w = direction(p.log2w, false), sgn_h = direction(p.log2h, false);
  const float* in = p.feat;  // [B][C][h][w]

  // rows: two real rows per complex transform
  for (int item = warp; item < p.cg * npairs; item += kWarps) {
    const int cg = item / npairs, yp = item - cg * npairs;
    const int c = c0 + cg;
    if (c >= p.c) continue;
    const int ya = 2 * yp, yb = 2 * yp + 1;
    const float* ra = in + (((size_t)b * p.c + c) * p.h + ya) * p.w;
    const float* rb = ra + p.w;
    for (int x = lane; x < p.w; x += 32)
      L[x] = make_float2(ra[x], yb < p.h ? rb[x] : 0.f);
    __syncwarp();
    warp_line_transform(L, T, s.tw_w, p.w, p.log2w, sgn_w);
    float2* za = s.Z + ((size_t)cg * p.h + ya) * p.wh;
    float2* zb = s.Z + ((size_t)cg * p.h + yb) * p.wh;
    for (int k = lane; k < p.wh; k += 32) {
      const float2 zk = L[k], zm = L[k == 0 ? 0 : p.w - k];
      za[k] = make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y - zm.y));
      if (yb < p.h) zb[k] = make_float2(0.5f * (zk.y + zm.y), -0.5f * (zk.x - zm.x));
    }
    __syncwarp();
  }
  __syncthreads();

  // columns, then scale and store the split spectrum (channels 2c = re, 2c+1 = im)
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.spec);
  const int C2 = 2 * p.c;
  for (int item = warp; item < p.cg * p.wh; item += kWarps) {
    const int cg = item / p.wh, kx = item - cg * p.wh;
    const int c = c0 + cg;
    if (c >= p.c) continue;
    const float2* zc = s.Z + (size_t)cg * p.h * p.wh + kx;
    for (int y = lane; y < p.h; y += 32) L[y] = zc[(size_t)y * p.wh];
    __syncwarp();
    warp_line_transform(L, T, s.tw_h, p.h, p.log2h, sgn_h);
    for (int ky = lane; ky < p.h; ky += 32) {
      const float2 v = L[ky];
      uint32_t hi, lo;
      split_pair(v.x * p.scale, v.y * p.scale, hi, lo);
      const size_t off = (((size_t)b * p.h + ky) * p.wh + kx) * C2 + 2 * c;
      *reinterpret_cast<uint32_t*>(out + off) = hi;
      *reinterpret_cast<uint32_t*>(out + p.spec_part + off) = lo;
    }
    __syncwarp();
  }
}

__global__ void __launch_bounds__(256) k_irfft2(const FftParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const Smem s = carve(p, smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, c0 = blockIdx.x * p.cg;
  load_twiddles(p, s);
  __syncthreads();
  float2* L = s.lines + warp * 2 * p.lmax;
  float2* T = L + p.lmax;
  const int sgn_w = direction(p.log2w, true), sgn_h = direction(p.log2h, true);
  const int C2 = 2 * p.c;

  // columns of the stored half-spectrum
  for (int item = warp; item < p.cg * p.wh; item += kWarps) {
    const int cg = item / p.wh, kx = item - cg * p.wh;
    const int c = c0 + cg;
    if (c >= p.c) continue;
    for (int y = lane; y < p.h; y += 32) {
      const float* src = p.fu + (((size_t)b * p.h + y) * p.wh + kx) * C2 + 2 * c;
      L[y] = make_float2(src[0], src[1]);
    }
    __syncwarp();
    warp_line_transform(L, T, s.tw_h, p.h, p.log2h, sgn_h);
    float2* zc = s.Z + (size_t)cg * p.h * p.wh + kx;
    for (int y = lane; y < p.h; y += 32) zc[(size_t)y * p.wh] = L[y];
    __syncwarp();
  }
  __syncthreads();

  // rows: Hermitian completion, two real rows per complex transform, + feat
  const int npairs = (p.h + 1) >> 1;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.s_out);
  for (int item = warp; item < p.cg * npairs; item += kWarps) {
    const int cg = item / npairs, yp = item - cg * npairs;
    const int c = c0 + cg;
    if (c >= p.c) continue;
    const int ya = 2 * yp, yb = 2 * yp + 1;
    const float2* za = s.Z + ((size_t)cg * p.h + ya) * p.wh;
    const float2* zb = s.Z + ((size_t)cg * p.h + (yb < p.h ? yb : ya)) * p.wh;
    for (int k = lane; k < p.w; k += 32) {
      float2 a, bb;
      if (k < p.wh) {
        a = za[k];
        bb = zb[k];
        if (k == 0 || 2 * k == p.w) { a.y = 0.f; bb.y = 0.f; }
      } else {
        a = za[p.w - k];
        bb = zb[p.w - k];
        a.y = -a.y;
        bb.y = -bb.y;
      }
      if (yb >= p.h) bb = make_float2(0.f, 0.f);
      L[k] = make_float2(a.x - bb.y, a.y + bb.x);
    }
    __syncwarp();
    warp_line_transform(L, T, s.tw_w, p.w, p.log2w, sgn_w);
    for (int x = lane; x < p.w; x += 32) {
      const float2 v = L[x];
      const size_t ia = (((size_t)b * p.h + ya) * p.w + x) * p.c + c;
      const size_t fa = (((size_t)b * p.c + c) * p.h + ya) * p.w + x;
      const float va = v.x * p.scale + p.feat[fa];
      const __nv_bfloat16 ha = __float2bfloat16_rn(va);
      out[ia] = ha;
      out[p.s_part + ia] = __float2bfloat16_rn(va - __bfloat162float(ha));
      if (yb < p.h) {
        const size_t ib = ia + (size_t)p.w * p.c;
        const float vb = v.y * p.scale + p.feat[fa + p.w];
        const __nv_bfloat16 hb = __float2bfloat16_rn(vb);
        out[ib] = hb;
        out[p.s_part + ib] = __float2bfloat16_rn(vb - __bfloat162float(hb));
      }
    }
    __syncwarp();
  }
}

}  // namespace

size_t fft_smem_bytes(const FftParams& p) {
  return sizeof(float2) * ((size_t)p.cg * p.h * p.wh + (size_t)kWarps * 2 * p.lmax + p.h + p.w);
}

int fft_prepare(size_t max_smem) {
  cudaError_t e = cudaFuncSetAttribute(k_rfft2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_smem);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaFuncSetAttribute(k_irfft2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_smem);
}

int launch_rfft2(const FftParams& p, cudaStream_t st) {
  dim3 grid((p.c + p.cg - 1) / p.cg, p.batch);
  k_rfft2<<<grid, 256, fft_smem_bytes(p), st>>>(p);
  return (int)cudaGetLastError();
}

int launch_irfft2(const FftParams& p, cudaStream_t st) {
  dim3 grid((p.c + p.cg - 1) / p.cg, p.batch);
  k_irfft2<<<grid, 256, fft_smem_bytes(p), st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace lama
