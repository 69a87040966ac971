// FourierUnit transforms for planes of any size: rfft2 / irfft2 with
// norm='ortho', as two streaming passes joined by a complex fp32 intermediate.
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
// Passes (every CTA: a tile of lines in shared memory, all threads cooperate
// on each stage; powers of two run radix-2 stages over bit-reversed loads,
// other lengths a direct DFT against a twiddle table):
//   rfft2   rows_fwd  feat NCHW rows, two real rows per complex line
//                     -> T[b][c][kx][y]   (columns contiguous)
//           cols_fwd  T columns of 16 channels -> spectrum [b][ky][kx][2c+part]
//   irfft2  cols_inv  fu [b][ky][kx][2c+part] columns -> T[b][y][kx][c]
//           rows_inv  T rows of 16 channels, Hermitian completion, two rows per
//                     complex line, + feat -> S [b][y][x][c] (split bf16)
// T holds B*c*(w/2+1)*h complex values and is shared by every transform of a
// plan.  No plane is ever held whole on chip, so any latent size runs.
// Arithmetic is fp32 with twiddles rounded from double.
#include <algorithm>
#include <cstdint>

#include "fft.cuh"
#include "ptx.cuh"

namespace lama {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Position of element k of a line when it is loaded: bit-reversed for the
// radix-2 stages, natural for the direct DFT.
__device__ __forceinline__ int load_pos(int k, int log2n) {
  return log2n > 0 ? (int)(__brev((unsigned)k) >> (32 - log2n)) : k;
}

// Transforms `nl` lines of length n, line l at buf + l * ls.  Powers of two:
// in place (loaded bit-reversed), returns buf.  Otherwise a direct DFT into
// tmp, returns tmp.  `sign` -1: sum x_j e^{-2 pi i jk/n}, +1: e^{+...}; tw
// holds (cos, sin)(2 pi m / n), m < n.  Ends with __syncthreads.
__device__ float2* transform_lines(float2* buf, float2* tmp, int nl, int ls, int n, int log2n, const float2* tw,
                                   float sign) {
  if (log2n >= 0) {
    const int hn = n >> 1, nb = nl * hn;
    for (int s = 1; s <= log2n; s++) {
      const int half = 1 << (s - 1), tstride = n >> s;
      for (int t = threadIdx.x; t < nb; t += blockDim.x) {
        const int l = t >> (log2n - 1), r = t & (hn - 1);
        const int k = r & (half - 1), i = ((r >> (s - 1)) << s) + k;
        float2* L = buf + l * ls;
        float2 w = tw[k * tstride];
        w.y *= sign;
        const float2 v = cmul(L[i + half], w), u = L[i];
        L[i] = make_float2(u.x + v.x, u.y + v.y);
        L[i + half] = make_float2(u.x - v.x, u.y - v.y);
      }
      __syncthreads();
    }
    return buf;
  }
  for (int t = threadIdx.x; t < nl * n; t += blockDim.x) {
    const int l = t / n, k = t - l * n;
    const float2* L = buf + l * ls;
    float2 acc = make_float2(0.f, 0.f);
    int idx = 0;
    for (int j = 0; j < n; j++) {
      float2 w = tw[idx];
      w.y *= sign;
      const float2 v = cmul(L[j], w);
      acc.x += v.x;
      acc.y += v.y;
      idx += k;
      if (idx >= n) idx -= n;
    }
    tmp[l * ls + k] = acc;
  }
  __syncthreads();
  return tmp;
}

__device__ __forceinline__ float direction(int log2n, bool inverse) {
  // powers of two: forward e^{-}, inverse e^{+}; otherwise swapped (see header)
  const bool fwd = (log2n >= 0) ? !inverse : inverse;
  return fwd ? -1.f : 1.f;
}

__device__ __forceinline__ void load_tw(float2* dst, const float2* src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

// ------------------------------------------------------------------ rfft2
// grid (row-pair blocks, c, b); lines = pairs of rows (a + i b), ls = w + 1
__global__ void __launch_bounds__(kThreads) k_rows_fwd(const FftParams p) {
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c = blockIdx.y, y0 = blockIdx.x * 2 * p.rp;
  const int W = p.w, ls = W + 1;
  const int nrows = min(2 * p.rp, p.h - y0), nl = (nrows + 1) >> 1;
  float2* tw = sm;
  float2* buf = tw + W;
  float2* tmp = buf + p.rp * ls;
  load_tw(tw, p.tw_w, W);
  const float* plane = p.feat + (((size_t)b * p.c + c) * p.h + y0) * W;
  for (int t = threadIdx.x; t < nl * W; t += blockDim.x) {
    const int l = t / W, x = t - l * W;
    const float a = plane[(size_t)(2 * l) * W + x];
    const float bb = 2 * l + 1 < nrows ? plane[(size_t)(2 * l + 1) * W + x] : 0.f;
    buf[l * ls + load_pos(x, p.log2w)] = make_float2(a, bb);
  }
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, W, p.log2w, tw, direction(p.log2w, false));
  // untangle the two real rows; T[b][c][kx][y], y fastest
  float2* T = p.tmp + ((size_t)b * p.c + c) * p.wh * p.h + y0;
  for (int t = threadIdx.x; t < p.wh * nrows; t += blockDim.x) {
    const int kx = t / nrows, r = t - kx * nrows, l = r >> 1;
    const float2 zk = L[l * ls + kx], zm = L[l * ls + (kx == 0 ? 0 : W - kx)];
    T[(size_t)kx * p.h + r] = (r & 1) ? make_float2(0.5f * (zk.y + zm.y), -0.5f * (zk.x - zm.x))
                                      : make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y - zm.y));
  }
}

// grid (kx blocks of kb, channel groups of cg, b); lines = (kx, channel)
// columns, channel fastest (conflict-free smem reads when storing channel-fastest)
__global__ void __launch_bounds__(kThreads) k_cols_fwd(const FftParams p) {
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c0 = blockIdx.y * p.cg, kx0 = blockIdx.x * p.kb;
  const int H = p.h, ls = H + 1;
  const int ncg = min(p.cg, p.c - c0), nkb = min(p.kb, p.wh - kx0), nl = ncg * nkb;
  float2* tw = sm;
  float2* buf = tw + H;
  float2* tmp = buf + p.cg * p.kb * ls;
  load_tw(tw, p.tw_h, H);
  for (int t = threadIdx.x; t < nl * H; t += blockDim.x) {
    const int l = t / H, y = t - l * H;
    const int kl = l / ncg, cl = l - kl * ncg;
    const float2 v = p.tmp[(((size_t)b * p.c + c0 + cl) * p.wh + kx0 + kl) * H + y];
    buf[l * ls + load_pos(y, p.log2h)] = v;
  }
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, H, p.log2h, tw, direction(p.log2h, false));
  // spectrum [b][ky][kx][2c + part], channel fastest
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.spec);
  const int C2 = 2 * p.c;
  for (int t = threadIdx.x; t < nl * H; t += blockDim.x) {
    const int cl = t % ncg, r = t / ncg, kl = r % nkb, ky = r / nkb;
    const float2 v = L[(kl * ncg + cl) * ls + ky];
    uint32_t hi, lo;
    split_pair(v.x * p.scale, v.y * p.scale, hi, lo);
    const size_t off = (((size_t)b * H + ky) * p.wh + kx0 + kl) * C2 + 2 * (c0 + cl);
    *reinterpret_cast<uint32_t*>(out + off) = hi;
    *reinterpret_cast<uint32_t*>(out + p.spec_part + off) = lo;
  }
}

// ------------------------------------------------------------------ irfft2
// grid (kx blocks of kb, channel groups of cg, b); lines = (kx, channel) columns
__global__ void __launch_bounds__(kThreads) k_cols_inv(const FftParams p) {
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c0 = blockIdx.y * p.cg, kx0 = blockIdx.x * p.kb;
  const int H = p.h, ls = H + 1;
  const int ncg = min(p.cg, p.c - c0), nkb = min(p.kb, p.wh - kx0), nl = ncg * nkb;
  float2* tw = sm;
  float2* buf = tw + H;
  float2* tmp = buf + p.cg * p.kb * ls;
  load_tw(tw, p.tw_h, H);
  const int C2 = 2 * p.c;
  for (int t = threadIdx.x; t < nl * H; t += blockDim.x) {
    const int cl = t % ncg, r = t / ncg, kl = r % nkb, ky = r / nkb;
    const float2 v = *reinterpret_cast<const float2*>(p.fu + (((size_t)b * H + ky) * p.wh + kx0 + kl) * C2 +
                                                      2 * (c0 + cl));
    buf[(kl * ncg + cl) * ls + load_pos(ky, p.log2h)] = v;
  }
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, H, p.log2h, tw, direction(p.log2h, true));
  // T[b][y][kx][c], channel fastest
  for (int t = threadIdx.x; t < nl * H; t += blockDim.x) {
    const int cl = t % ncg, r = t / ncg, kl = r % nkb, y = r / nkb;
    p.tmp[(((size_t)b * H + y) * p.wh + kx0 + kl) * p.c + c0 + cl] = L[(kl * ncg + cl) * ls + y];
  }
}

// grid (row-pair blocks of rpi, channel groups of cg, b); lines = (row pair, channel)
__global__ void __launch_bounds__(kThreads) k_rows_inv(const FftParams p) {
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c0 = blockIdx.y * p.cg, y0 = blockIdx.x * 2 * p.rpi;
  const int W = p.w, ls = W + 1, fs = W + 1;
  const int ncg = min(p.cg, p.c - c0), nrows = min(2 * p.rpi, p.h - y0), npair = (nrows + 1) >> 1;
  const int nl = npair * ncg;
  float2* tw = sm;
  float2* buf = tw + W;
  float2* tmp = buf + p.rpi * p.cg * ls;
  float* fe = reinterpret_cast<float*>(p.log2w >= 0 ? tmp : tmp + p.rpi * p.cg * ls);  // [row][channel][x]
  load_tw(tw, p.tw_w, W);
  // Hermitian completion of each row's bins; line (pair, channel) = row a + i row b
  for (int t = threadIdx.x; t < nl * W; t += blockDim.x) {
    const int cl = t % ncg, r = t / ncg, k = r % W, pr = r / W;
    const int ya = y0 + 2 * pr, yb = ya + 1;
    const bool mirror = k >= p.wh;
    const int kk = mirror ? W - k : k;
    const float2* Ta = p.tmp + (((size_t)b * p.h + ya) * p.wh + kk) * p.c + c0 + cl;
    float2 a = Ta[0];
    float2 bb = yb < y0 + nrows ? Ta[(size_t)p.wh * p.c] : make_float2(0.f, 0.f);
    if (k == 0 || 2 * k == W) {
      a.y = 0.f;
      bb.y = 0.f;
    }
    if (mirror) {
      a.y = -a.y;
      bb.y = -bb.y;
    }
    buf[(pr * ncg + cl) * ls + load_pos(k, p.log2w)] = make_float2(a.x - bb.y, a.y + bb.x);
  }
  // feat rows of this tile, coalesced along x
  for (int t = threadIdx.x; t < nrows * ncg * W; t += blockDim.x) {
    const int x = t % W, r = t / W, cl = r % ncg, row = r / ncg;
    fe[(row * ncg + cl) * fs + x] = p.feat[(((size_t)b * p.c + c0 + cl) * p.h + y0 + row) * W + x];
  }
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, W, p.log2w, tw, direction(p.log2w, true));
  // S [b][y][x][c] = feat + scale * row, channel fastest
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.s_out);
  for (int t = threadIdx.x; t < nrows * W * ncg; t += blockDim.x) {
    const int cl = t % ncg, r = t / ncg, x = r % W, row = r / W;
    const float2 v = L[((row >> 1) * ncg + cl) * ls + x];
    const float s = ((row & 1) ? v.y : v.x) * p.scale + fe[(row * ncg + cl) * fs + x];
    const __nv_bfloat16 hs = __float2bfloat16_rn(s);
    const size_t o = (((size_t)b * p.h + y0 + row) * W + x) * p.c + c0 + cl;
    out[o] = hs;
    out[p.s_part + o] = __float2bfloat16_rn(s - __bfloat162float(hs));
  }
}

inline size_t tw_bytes(int n) { return sizeof(float2) * (size_t)n; }

}  // namespace

size_t fft_smem_bytes(const FftParams& p, int pass) {
  const bool pw = p.log2w >= 0, ph = p.log2h >= 0;
  switch (pass) {
    case 0:  // rows_fwd
      return tw_bytes(p.w) + (pw ? 1 : 2) * sizeof(float2) * (size_t)p.rp * (p.w + 1);
    case 1:  // cols_fwd / cols_inv
      return tw_bytes(p.h) + (ph ? 1 : 2) * sizeof(float2) * (size_t)p.cg * p.kb * (p.h + 1);
    default:  // rows_inv: lines (+ tmp) + feat rows
      return tw_bytes(p.w) + (pw ? 1 : 2) * sizeof(float2) * (size_t)p.rpi * p.cg * (p.w + 1) +
             sizeof(float) * (size_t)2 * p.rpi * p.cg * (p.w + 1);
  }
}

bool fft_tiles(FftParams& p, size_t max_smem) {
  constexpr int kElems = 4096;  // complex values per tile
  const int w = std::max(1, p.w), h = std::max(1, p.h), pairs = (h + 1) / 2;
  p.rp = std::max(1, std::min(kElems / w, pairs));
  for (p.cg = std::min(16, p.c); p.cg >= 1; p.cg /= 2) {
    p.kb = std::max(1, std::min(kElems / (p.cg * h), p.wh));
    p.rpi = std::max(1, std::min(kElems / (p.cg * w), pairs));
    if (fft_smem_bytes(p, 1) <= max_smem && fft_smem_bytes(p, 2) <= max_smem) break;
  }
  return p.cg >= 1 && fft_smem_bytes(p, 0) <= max_smem;
}

size_t fft_tmp_elems(const FftParams& p) { return (size_t)p.batch * p.c * p.wh * p.h; }

int fft_prepare(size_t max_smem) {
  const void* fns[] = {(const void*)k_rows_fwd, (const void*)k_cols_fwd, (const void*)k_cols_inv,
                       (const void*)k_rows_inv};
  for (const void* f : fns) {
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_smem);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

int launch_rfft2(const FftParams& p, cudaStream_t st) {
  const dim3 g0((p.h + 2 * p.rp - 1) / (2 * p.rp), p.c, p.batch);
  const dim3 g1((p.wh + p.kb - 1) / p.kb, (p.c + p.cg - 1) / p.cg, p.batch);
  k_rows_fwd<<<g0, kThreads, fft_smem_bytes(p, 0), st>>>(p);
  k_cols_fwd<<<g1, kThreads, fft_smem_bytes(p, 1), st>>>(p);
  return (int)cudaGetLastError();
}

int launch_irfft2(const FftParams& p, cudaStream_t st) {
  const dim3 g1((p.wh + p.kb - 1) / p.kb, (p.c + p.cg - 1) / p.cg, p.batch);
  const dim3 g2((p.h + 2 * p.rpi - 1) / (2 * p.rpi), (p.c + p.cg - 1) / p.cg, p.batch);
  k_cols_inv<<<g1, kThreads, fft_smem_bytes(p, 1), st>>>(p);
  k_rows_inv<<<g2, kThreads, fft_smem_bytes(p, 2), st>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace lama
