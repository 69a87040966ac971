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
#include "launch.cuh"
#include "ptx.cuh"

namespace lama {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }
// i * sign * z
__device__ __forceinline__ float2 rot(float2 z, float sign) { return make_float2(-sign * z.y, sign * z.x); }

// e^{sign * 2 pi i m / n} from the (cos, sin) table of length n
__device__ __forceinline__ float2 twf(const float2* tw, int m, float sign) {
  const float2 w = tw[m];
  return make_float2(w.x, sign * w.y);
}

// In-register DFT of R points: X_k = sum_r v_r e^{sign 2 pi i rk/R}.
template <int R>
__device__ __forceinline__ void dft_small(float2 (&v)[R], float sign);

template <>
__device__ __forceinline__ void dft_small<2>(float2 (&v)[2], float) {
  const float2 a = v[0], b = v[1];
  v[0] = cadd(a, b);
  v[1] = csub(a, b);
}

template <>
__device__ __forceinline__ void dft_small<4>(float2 (&v)[4], float sign) {
  const float2 s02 = cadd(v[0], v[2]), d02 = csub(v[0], v[2]);
  const float2 s13 = cadd(v[1], v[3]), d13 = rot(csub(v[1], v[3]), sign);
  v[0] = cadd(s02, s13);
  v[2] = csub(s02, s13);
  v[1] = cadd(d02, d13);
  v[3] = csub(d02, d13);
}

template <>
__device__ __forceinline__ void dft_small<8>(float2 (&v)[8], float sign) {
  float2 e[4] = {v[0], v[2], v[4], v[6]}, o[4] = {v[1], v[3], v[5], v[7]};
  dft_small<4>(e, sign);
  dft_small<4>(o, sign);
  constexpr float h = 0.70710678118654752f;  // cos(pi/4)
  const float2 o1 = make_float2(h * (o[1].x - sign * o[1].y), h * (o[1].y + sign * o[1].x));
  const float2 o2 = rot(o[2], sign);
  const float2 o3 = make_float2(-h * (o[3].x + sign * o[3].y), h * (sign * o[3].x - o[3].y));
  v[0] = cadd(e[0], o[0]);
  v[4] = csub(e[0], o[0]);
  v[1] = cadd(e[1], o1);
  v[5] = csub(e[1], o1);
  v[2] = cadd(e[2], o2);
  v[6] = csub(e[2], o2);
  v[3] = cadd(e[3], o3);
  v[7] = csub(e[3], o3);
}

template <>
__device__ __forceinline__ void dft_small<3>(float2 (&v)[3], float sign) {
  constexpr float c = -0.5f, s = 0.86602540378443865f;  // cos, sin(2 pi / 3)
  const float2 t = cadd(v[1], v[2]), d = rot(cscale(csub(v[1], v[2]), s), sign);
  const float2 m = make_float2(v[0].x + c * t.x, v[0].y + c * t.y);
  v[0] = cadd(v[0], t);
  v[1] = cadd(m, d);
  v[2] = csub(m, d);
}

template <>
__device__ __forceinline__ void dft_small<5>(float2 (&v)[5], float sign) {
  constexpr float c1 = 0.30901699437494742f, c2 = -0.80901699437494742f;  // cos(2 pi / 5), cos(4 pi / 5)
  constexpr float s1 = 0.95105651629515357f, s2 = 0.58778525229247313f;   // sin(2 pi / 5), sin(4 pi / 5)
  const float2 a1 = cadd(v[1], v[4]), b1 = csub(v[1], v[4]);
  const float2 a2 = cadd(v[2], v[3]), b2 = csub(v[2], v[3]);
  const float2 m1 = make_float2(v[0].x + c1 * a1.x + c2 * a2.x, v[0].y + c1 * a1.y + c2 * a2.y);
  const float2 m2 = make_float2(v[0].x + c2 * a1.x + c1 * a2.x, v[0].y + c2 * a1.y + c1 * a2.y);
  const float2 n1 = rot(make_float2(s1 * b1.x + s2 * b2.x, s1 * b1.y + s2 * b2.y), sign);
  const float2 n2 = rot(make_float2(s2 * b1.x - s1 * b2.x, s2 * b1.y - s1 * b2.y), sign);
  v[0] = cadd(v[0], cadd(a1, a2));
  v[1] = cadd(m1, n1);
  v[4] = csub(m1, n1);
  v[2] = cadd(m2, n2);
  v[3] = csub(m2, n2);
}

// One Stockham autosort stage of radix R over nl lines of length n (line l
// at src/dst + l * ls); Ns = product of the radices already applied.
// Butterfly j reads src[j + r n/R], twiddles input r by
// e^{sign 2 pi i r (j mod Ns) / (Ns R)}, and writes its R-point DFT to
// dst[(j / Ns) Ns R + (j mod Ns) + k Ns].
template <int R>
__device__ __forceinline__ void stage(const float2* src, float2* dst, int nl, int ls, int n, const FftStage& sg,
                                      const float2* tw, float sign) {
  const int m = (int)sg.m.d, Ns = (int)sg.ns.d, nb = nl * m, tstep = n / (Ns * R);
  for (int t = threadIdx.x; t < nb; t += blockDim.x) {
    const int l = (int)fdiv(t, sg.m), j = t - l * m;
    const int jq = (int)fdiv(j, sg.ns), jm = j - jq * Ns;
    const float2* S = src + l * ls + j;
    float2 v[R];
    v[0] = S[0];
#pragma unroll
    for (int r = 1; r < R; r++) v[r] = cmul(S[r * m], twf(tw, r * jm * tstep, sign));
    dft_small<R>(v, sign);
    float2* D = dst + l * ls + jq * Ns * R + jm;
#pragma unroll
    for (int k = 0; k < R; k++) D[k * Ns] = v[k];
  }
}

// Stage of any radix R: every thread computes single outputs as length-R sums
// (used for prime factors above 5, including a prime length itself, where it
// is the direct DFT).
__device__ void stage_generic(const float2* src, float2* dst, int nl, int ls, int n, const Radices& rad,
                              const FftStage& sg, const float2* tw, float sign) {
  const int R = sg.r, Ns = (int)sg.ns.d, m = (int)sg.m.d, tstep = n / (Ns * R);
  for (int t = threadIdx.x; t < nl * n; t += blockDim.x) {
    const int l = (int)fdiv(t, rad.len), q = t - l * n;
    const int qn = (int)fdiv(q, sg.ns), jm = q - qn * Ns;
    const int qr = (int)fdiv(qn, sg.rr), k = qn - qr * R, j = qr * Ns + jm;
    const float2* S = src + l * ls + j;
    const int step = (tstep * (jm + k * Ns)) % n;
    float2 acc = S[0];
    int idx = step;
    for (int r = 1; r < R; r++) {
      const float2 v = cmul(S[r * m], twf(tw, idx, sign));
      acc.x += v.x;
      acc.y += v.y;
      idx += step;
      if (idx >= n) idx -= n;
    }
    dst[l * ls + q] = acc;
  }
}

// Transforms nl lines of length n held at a (line l at a + l * ls), ping-
// ponging with b; returns the buffer holding the result (natural order).
// `sign` -1: sum x_j e^{-2 pi i jk/n}, +1: e^{+...}; tw holds
// (cos, sin)(2 pi m / n), m < n; `rad` lists the stages (radix product n).
// Ends with __syncthreads.
__device__ float2* transform_lines(float2* a, float2* b, int nl, int ls, const Radices& rad, const float2* tw,
                                   float sign) {
  float2 *src = a, *dst = b;
  const int n = rad.n;
  for (int s = 0; s < 12; s++) {
    const int R = rad.st[s].r;
    if (R == 0) break;
    switch (R) {
      case 2: stage<2>(src, dst, nl, ls, n, rad.st[s], tw, sign); break;
      case 3: stage<3>(src, dst, nl, ls, n, rad.st[s], tw, sign); break;
      case 4: stage<4>(src, dst, nl, ls, n, rad.st[s], tw, sign); break;
      case 5: stage<5>(src, dst, nl, ls, n, rad.st[s], tw, sign); break;
      case 8: stage<8>(src, dst, nl, ls, n, rad.st[s], tw, sign); break;
      default: stage_generic(src, dst, nl, ls, n, rad, rad.st[s], tw, sign); break;
    }
    __syncthreads();
    float2* t = src;
    src = dst;
    dst = t;
  }
  return src;
}

__device__ __forceinline__ float direction(int log2n, bool inverse) {
  // powers of two: forward e^{-}, inverse e^{+}; otherwise swapped (see header)
  const bool fwd = (log2n >= 0) ? !inverse : inverse;
  return fwd ? -1.f : 1.f;
}

// Loads items 0..total-1 U at a time per thread (all U global loads issued
// before any shared-memory store, so each thread keeps U requests in flight).
template <int U, class Ld, class St>
__device__ __forceinline__ void batched(int total, Ld ld, St st) {
  using V = decltype(ld(0));
  for (int base = threadIdx.x; base < total; base += blockDim.x * U) {
    V v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = base + u * (int)blockDim.x;
      if (i < total) v[u] = ld(i);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = base + u * (int)blockDim.x;
      if (i < total) st(i, v[u]);
    }
  }
}

struct F4x2 {
  float4 a, b;
};

__device__ __forceinline__ bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }

__device__ __forceinline__ void load_tw(float2* dst, const float2* src, int n) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
}

// ------------------------------------------------------------------ rfft2
// Every CTA works on a full tile (lines past the plane's edge are zero-filled
// and never stored), so all index arithmetic uses plan-time divisors.

// grid (row-pair blocks of rp, c, b); lines = pairs of rows (a + i b), ls = w + 1
__global__ void __launch_bounds__(kThreads) k_rows_fwd(const FftParams p) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c = blockIdx.y, y0 = blockIdx.x * 2 * p.rp;
  const int W = p.w, ls = W + 1, R2 = 2 * p.rp;
  const int nrows = min(R2, p.h - y0);
  float2* tw = sm;
  float2* buf = tw + W;
  float2* tmp = buf + p.rp * ls;
  load_tw(tw, p.tw_w, W);
  const float* plane = p.feat + (((size_t)b * p.c + c) * p.h + y0) * W;
  if ((W & 3) == 0 && aligned16(p.feat)) {
    const int W4 = W >> 2;
    batched<4>(
        p.rp * W4,
        [&](int t) {
          const int l = t / W4, x = (t - l * W4) * 4;
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
          F4x2 v{z, z};
          if (2 * l < nrows) v.a = *reinterpret_cast<const float4*>(plane + (size_t)(2 * l) * W + x);
          if (2 * l + 1 < nrows) v.b = *reinterpret_cast<const float4*>(plane + (size_t)(2 * l + 1) * W + x);
          return v;
        },
        [&](int t, const F4x2& v) {
          const int l = t / W4, x = (t - l * W4) * 4;
          float2* d = buf + l * ls + x;
          d[0] = make_float2(v.a.x, v.b.x);
          d[1] = make_float2(v.a.y, v.b.y);
          d[2] = make_float2(v.a.z, v.b.z);
          d[3] = make_float2(v.a.w, v.b.w);
        });
  } else {
    batched<8>(
        p.rp * W,
        [&](int t) {
          const int l = (int)fdiv(t, p.fd_w), x = t - l * W;
          return make_float2(2 * l < nrows ? plane[(size_t)(2 * l) * W + x] : 0.f,
                             2 * l + 1 < nrows ? plane[(size_t)(2 * l + 1) * W + x] : 0.f);
        },
        [&](int t, float2 v) {
          const int l = (int)fdiv(t, p.fd_w);
          buf[l * ls + t - l * W] = v;
        });
  }
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, p.rp, ls, p.rad_w, tw, direction(p.log2w, false));
  // untangle the two real rows; T[b][c][kx][y], y fastest
  float2* T = p.tmp + ((size_t)b * p.c + c) * p.wh * p.h + y0;
  for (int t = threadIdx.x; t < p.wh * R2; t += blockDim.x) {
    const int kx = (int)fdiv(t, p.fd_rows), r = t - kx * R2, l = r >> 1;
    if (r >= nrows) continue;
    const float2 zk = L[l * ls + kx], zm = L[l * ls + (kx == 0 ? 0 : W - kx)];
    T[(size_t)kx * p.h + r] = (r & 1) ? make_float2(0.5f * (zk.y + zm.y), -0.5f * (zk.x - zm.x))
                                      : make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y - zm.y));
  }
}

// grid (kx blocks of kb, channel groups of cg, b); lines = (kx, channel)
// columns, channel fastest (conflict-free smem reads when storing channel-fastest)
__global__ void __launch_bounds__(kThreads) k_cols_fwd(const FftParams p) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c0 = blockIdx.y * p.cg, kx0 = blockIdx.x * p.kb;
  const int H = p.h, ls = H + 1, CG = p.cg, nl = CG * p.kb;
  const int ncg = min(CG, p.c - c0), nkb = min(p.kb, p.wh - kx0);
  float2* tw = sm;
  float2* buf = tw + H;
  float2* tmp = buf + nl * ls;
  load_tw(tw, p.tw_h, H);
  batched<8>(
      nl * H,
      [&](int t) {
        const int l = (int)fdiv(t, p.fd_h), y = t - l * H;
        const int kl = (int)fdiv(l, p.fd_cg), cl = l - kl * CG;
        return (cl < ncg && kl < nkb) ? p.tmp[(((size_t)b * p.c + c0 + cl) * p.wh + kx0 + kl) * H + y]
                                      : make_float2(0.f, 0.f);
      },
      [&](int t, float2 v) {
        const int l = (int)fdiv(t, p.fd_h);
        buf[l * ls + t - l * H] = v;
      });
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, p.rad_h, tw, direction(p.log2h, false));
  // spectrum [b][ky][kx][2c + part], channel fastest
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.spec);
  const int C2 = 2 * p.c;
  for (int t = threadIdx.x; t < nl * H; t += blockDim.x) {
    const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
    const int ky = (int)fdiv(r, p.fd_kb), kl = r - ky * p.kb;
    if (cl >= ncg || kl >= nkb) continue;
    const float2 v = L[(kl * CG + cl) * ls + ky];
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
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c0 = blockIdx.y * p.cg, kx0 = blockIdx.x * p.kb;
  const int H = p.h, ls = H + 1, CG = p.cg, nl = CG * p.kb;
  const int ncg = min(CG, p.c - c0), nkb = min(p.kb, p.wh - kx0);
  float2* tw = sm;
  float2* buf = tw + H;
  float2* tmp = buf + nl * ls;
  load_tw(tw, p.tw_h, H);
  const int C2 = 2 * p.c;
  batched<8>(
      nl * H,
      [&](int t) {
        const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
        const int ky = (int)fdiv(r, p.fd_kb), kl = r - ky * p.kb;
        float2 v = make_float2(0.f, 0.f);
        if (cl < ncg && kl < nkb)
          v = *reinterpret_cast<const float2*>(p.fu + (((size_t)b * H + ky) * p.wh + kx0 + kl) * C2 + 2 * (c0 + cl));
        return v;
      },
      [&](int t, float2 v) {
        const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
        const int ky = (int)fdiv(r, p.fd_kb), kl = r - ky * p.kb;
        buf[(kl * CG + cl) * ls + ky] = v;
      });
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, p.rad_h, tw, direction(p.log2h, true));
  // T[b][y][kx][c], channel fastest
  for (int t = threadIdx.x; t < nl * H; t += blockDim.x) {
    const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
    const int y = (int)fdiv(r, p.fd_kb), kl = r - y * p.kb;
    if (cl >= ncg || kl >= nkb) continue;
    p.tmp[(((size_t)b * H + y) * p.wh + kx0 + kl) * p.c + c0 + cl] = L[(kl * CG + cl) * ls + y];
  }
}

// grid (row-pair blocks of rpi, channel groups of cg, b); lines = (row pair, channel)
__global__ void __launch_bounds__(kThreads) k_rows_inv(const FftParams p) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float2 sm[];
  const int b = blockIdx.z, c0 = blockIdx.y * p.cg, y0 = blockIdx.x * 2 * p.rpi;
  const int W = p.w, ls = W + 1, fs = W + 1, CG = p.cg, nl = p.rpi * CG;
  const int ncg = min(CG, p.c - c0), nrows = min(2 * p.rpi, p.h - y0);
  float2* tw = sm;
  float2* buf = tw + W;
  float2* tmp = buf + nl * ls;
  load_tw(tw, p.tw_w, W);
  // Hermitian completion of each row's bins; line (pair, channel) = row a + i row b
  batched<4>(
      nl * W,
      [&](int t) {
        const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
        const int pr = (int)fdiv(r, p.fd_w), k = r - pr * W;
        const int ya = 2 * pr, yb = ya + 1;
        float2 a = make_float2(0.f, 0.f), bb = make_float2(0.f, 0.f);
        if (cl < ncg && ya < nrows) {
          const bool mirror = k >= p.wh;
          const int kk = mirror ? W - k : k;
          const float2* Ta = p.tmp + (((size_t)b * p.h + y0 + ya) * p.wh + kk) * p.c + c0 + cl;
          a = Ta[0];
          if (yb < nrows) bb = Ta[(size_t)p.wh * p.c];
          if (k == 0 || 2 * k == W) {
            a.y = 0.f;
            bb.y = 0.f;
          }
          if (mirror) {
            a.y = -a.y;
            bb.y = -bb.y;
          }
        }
        return make_float2(a.x - bb.y, a.y + bb.x);
      },
      [&](int t, float2 v) {
        const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
        const int pr = (int)fdiv(r, p.fd_w), k = r - pr * W;
        buf[(pr * CG + cl) * ls + k] = v;
      });
  __syncthreads();
  const float2* L = transform_lines(buf, tmp, nl, ls, p.rad_w, tw, direction(p.log2w, true));
  // feat rows of this tile, coalesced along x, into the buffer the result is not in
  float* fe = reinterpret_cast<float*>(L == buf ? tmp : buf);  // [row][channel][x]
  if ((W & 3) == 0 && aligned16(p.feat)) {
    const int W4 = W >> 2;
    batched<4>(
        2 * nl * W4,
        [&](int t) {
          const int r = t / W4, x = (t - r * W4) * 4;
          const int row = (int)fdiv(r, p.fd_cg), cl = r - row * CG;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (row < nrows && cl < ncg)
            v = *reinterpret_cast<const float4*>(p.feat + (((size_t)b * p.c + c0 + cl) * p.h + y0 + row) * W + x);
          return v;
        },
        [&](int t, const float4& v) {
          const int r = t / W4, x = (t - r * W4) * 4;
          float* d = fe + r * fs + x;  // r = row * CG + cl
          d[0] = v.x;
          d[1] = v.y;
          d[2] = v.z;
          d[3] = v.w;
        });
  } else {
    batched<8>(
        2 * nl * W,
        [&](int t) {
          const int r = (int)fdiv(t, p.fd_w), x = t - r * W;
          const int row = (int)fdiv(r, p.fd_cg), cl = r - row * CG;
          return (row < nrows && cl < ncg) ? p.feat[(((size_t)b * p.c + c0 + cl) * p.h + y0 + row) * W + x] : 0.f;
        },
        [&](int t, float v) {
          const int r = (int)fdiv(t, p.fd_w);
          fe[r * fs + t - r * W] = v;
        });
  }
  __syncthreads();
  // S [b][y][x][c] = feat + scale * row, channel fastest
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.s_out);
  for (int t = threadIdx.x; t < 2 * nl * W; t += blockDim.x) {
    const int r = (int)fdiv(t, p.fd_cg), cl = t - r * CG;
    const int row = (int)fdiv(r, p.fd_w), x = r - row * W;
    if (row >= nrows || cl >= ncg) continue;
    const float2 v = L[((row >> 1) * CG + cl) * ls + x];
    const float s = ((row & 1) ? v.y : v.x) * p.scale + fe[(row * CG + cl) * fs + x];
    const __nv_bfloat16 hs = __float2bfloat16_rn(s);
    const size_t o = (((size_t)b * p.h + y0 + row) * W + x) * p.c + c0 + cl;
    out[o] = hs;
    out[p.s_part + o] = __float2bfloat16_rn(s - __bfloat162float(hs));
  }
}

inline size_t tw_bytes(int n) { return sizeof(float2) * (size_t)n; }

}  // namespace

size_t fft_smem_bytes(const FftParams& p, int pass) {
  // twiddle table + two line buffers (the Stockham stages ping-pong)
  switch (pass) {
    case 0:  // rows_fwd
      return tw_bytes(p.w) + 2 * sizeof(float2) * (size_t)p.rp * (p.w + 1);
    case 1:  // cols_fwd / cols_inv
      return tw_bytes(p.h) + 2 * sizeof(float2) * (size_t)p.cg * p.kb * (p.h + 1);
    default:  // rows_inv (the feat rows reuse the free buffer)
      return tw_bytes(p.w) + 2 * sizeof(float2) * (size_t)p.rpi * p.cg * (p.w + 1);
  }
}

// Radices of one line length: eights (a final 8 x 2 becomes 4 x 4), a four or
// a two, then threes, fives and any other prime factors.
Radices fft_radices(int n) {
  Radices r{};
  int cnt = 0, ns = 1;
  const int len = n;
  r.n = n;
  r.len = make_fastdiv((unsigned)n);
  auto push = [&](int f) {
    if (cnt == 12) {  // more stages than a plan holds: reported as unsupported
      r.n = 0;
      return;
    }
    FftStage& s = r.st[cnt++];
    s.r = f;
    s.m = make_fastdiv((unsigned)(len / f));
    s.ns = make_fastdiv((unsigned)ns);
    s.rr = make_fastdiv((unsigned)f);
    s.nsr = make_fastdiv((unsigned)(ns * f));
    ns *= f;
  };
  int k = 0;
  while (n % 2 == 0) {
    n /= 2;
    k++;
  }
  while (k >= 3) {
    push(8);
    k -= 3;
  }
  if (k == 2) push(4);
  if (k == 1) {
    if (cnt > 0) {  // ... x 8 x 2 -> ... x 4 x 4
      ns /= 8;
      cnt--;
      push(4);
      push(4);
    } else {
      push(2);
    }
  }
  for (int f = 3; n > 1; f += 2)
    while (n % f == 0) {
      push(f);
      n /= f;
    }
  return r;
}

bool fft_tiles(FftParams& p, size_t max_smem) {
  constexpr int kElems = 4096;  // complex values per tile
  const int w = std::max(1, p.w), h = std::max(1, p.h), pairs = (h + 1) / 2;
  p.rad_h = fft_radices(h);
  p.rad_w = fft_radices(w);
  if (p.rad_h.n == 0 || p.rad_w.n == 0) return false;
  p.fd_w = make_fastdiv((unsigned)w);
  p.fd_h = make_fastdiv((unsigned)h);
  p.rp = std::max(1, std::min(kElems / w, pairs));
  for (p.cg = std::min(16, p.c); p.cg >= 1; p.cg /= 2) {
    p.kb = std::max(1, std::min(kElems / (p.cg * h), p.wh));
    p.rpi = std::max(1, std::min(kElems / (p.cg * w), pairs));
    if (fft_smem_bytes(p, 1) <= max_smem && fft_smem_bytes(p, 2) <= max_smem) break;
  }
  if (p.cg < 1) return false;
  p.fd_cg = make_fastdiv((unsigned)p.cg);
  p.fd_kb = make_fastdiv((unsigned)p.kb);
  p.fd_rows = make_fastdiv((unsigned)(2 * p.rp));
  return fft_smem_bytes(p, 0) <= max_smem;
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
  int e = launch_kernel(k_rows_fwd, g0, dim3(kThreads), fft_smem_bytes(p, 0), st, 1, p);
  if (e) return e;
  e = launch_kernel(k_cols_fwd, g1, dim3(kThreads), fft_smem_bytes(p, 1), st, 1, p);
  if (e) return e;
  return (int)cudaGetLastError();
}

int launch_irfft2(const FftParams& p, cudaStream_t st) {
  const dim3 g1((p.wh + p.kb - 1) / p.kb, (p.c + p.cg - 1) / p.cg, p.batch);
  const dim3 g2((p.h + 2 * p.rpi - 1) / (2 * p.rpi), (p.c + p.cg - 1) / p.cg, p.batch);
  int e = launch_kernel(k_cols_inv, g1, dim3(kThreads), fft_smem_bytes(p, 1), st, 1, p);
  if (e) return e;
  e = launch_kernel(k_rows_inv, g2, dim3(kThreads), fft_smem_bytes(p, 2), st, 1, p);
  if (e) return e;
  return (int)cudaGetLastError();
}

}  // namespace lama
