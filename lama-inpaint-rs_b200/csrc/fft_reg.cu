// Register-resident rfft2 / irfft2 for power-of-two planes up to 64 x 64.
//
// Same semantics as fft.cu (the reference's rfft2_ortho / irfft2_ortho,
// lama-rs/src/cpu.rs:769-837; power-of-two lengths use the standard transform
// directions there, cpu.rs:888-927), organised for throughput:
//   * one CTA = one image x 8 channels, 256 threads; thread t works on
//     channel t % 8, so a warp covers 8 channels x 4 lines and every global
//     access moves whole 16-64 byte channel groups;
//   * every 1-D transform lives in one thread's registers (fully unrolled
//     radix-2, twiddles from constant memory);
//   * rows: a real length-W row is one complex length-W/2 transform plus the
//     even/odd untangling (the half-length real-FFT identity);
//   * columns: after the row pass the DC and Nyquist columns are real, so
//     they share one complex transform, and each channel needs exactly W/2
//     column transforms; the inverse packs the Hermitian parts of those two
//     columns the same way (the row c2r ignores their imaginary parts);
//   * the plane sits in shared memory as [c][kx][y] with strides padded so
//     that both the row-thread and the column-thread access patterns are
//     bank-conflict free.
// Input feat is fp32 NCHW (written so by the conv1 epilogue); the spectrum
// and S are split bf16 NHWC operands of the following GEMMs.
#include <cstdint>

#include "fft.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace lama {

__constant__ float2 c_tw64[64];  // (cos, sin)(2 pi m / 64)

namespace {

constexpr int CG = 8;        // channels per CTA
constexpr int YS = 65;       // smem y stride (float2) of one column
constexpr int KS = 34;       // smem kx slots per channel (>= 33, stride = 4 words mod 32)

__host__ __device__ constexpr int ilog2(int n) { return n <= 1 ? 0 : 1 + ilog2(n >> 1); }
__host__ __device__ constexpr int brev(int i, int bits) {
  int r = 0;
  for (int b = 0; b < bits; b++) r |= ((i >> b) & 1) << (bits - 1 - b);
  return r;
}

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }

// e^{sign * 2 pi i m / n} for n | 64
template <int N, bool INV>
__device__ __forceinline__ float2 twid(int m) {
  float2 w = c_tw64[(m * (64 / N)) & 63];
  if (!INV) w.y = -w.y;
  return w;
}

// One radix-2 stage of span LEN, then the next.
template <int N, bool INV, int LEN>
__device__ __forceinline__ void fft_stages(float2 (&a)[N]) {
  if constexpr (LEN <= N) {
#pragma unroll
    for (int i = 0; i < N; i += LEN) {
#pragma unroll
      for (int k = 0; k < LEN / 2; k++) {
        const float2 u = a[i + k];
        float2 v = a[i + k + LEN / 2];
        if (k != 0) v = cmul(v, twid<LEN, INV>(k));
        a[i + k] = cadd(u, v);
        a[i + k + LEN / 2] = csub(u, v);
      }
    }
    fft_stages<N, INV, LEN * 2>(a);
  }
}

// Unnormalised in-register DFT of length N (power of two <= 64).
// INV = false: sum x_j e^{-2 pi i jk/N};  INV = true: e^{+...}.
template <int N, bool INV>
__device__ __forceinline__ void fft_reg(float2 (&a)[N]) {
  constexpr int B = ilog2(N);
#pragma unroll
  for (int i = 0; i < N; i++) {
    const int j = brev(i, B);
    if (i < j) {
      float2 t = a[i];
      a[i] = a[j];
      a[j] = t;
    }
  }
  fft_stages<N, INV, 2>(a);
}

struct Layout {
  float2* Z;  // [CG][KS][YS]
  __device__ __forceinline__ float2& at(int c, int kx, int y) const { return Z[(c * KS + kx) * YS + y]; }
};

// ------------------------------------------------------------------ rfft2
template <int H, int W>
__global__ void __launch_bounds__(256) k_rfft2_reg(const FftParams p) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int WH = W / 2 + 1, HALF = W / 2;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const Layout L{reinterpret_cast<float2*>(smem_raw)};
  const int t = threadIdx.x, c = t % CG, q = t / CG;
  const int b = blockIdx.y, cc = blockIdx.x * CG + c;
  const bool live = cc < p.c;

  // rows: x real, length W -> bins 0..W/2 via one complex length-W/2 transform
#pragma unroll 1
  for (int y = q; y < H; y += 32) {
    if (live) {
      const float4* row = reinterpret_cast<const float4*>(p.feat + (((size_t)b * p.c + cc) * H + y) * W);
      float2 z[HALF];
#pragma unroll
      for (int i = 0; i < W / 4; i++) {
        const float4 v = __ldg(row + i);
        z[2 * i] = make_float2(v.x, v.y);
        z[2 * i + 1] = make_float2(v.z, v.w);
      }
      fft_reg<HALF, false>(z);
#pragma unroll
      for (int k = 0; k <= HALF; k++) {
        const float2 zk = z[k % HALF], zm = conjf2(z[(HALF - k) % HALF]);
        const float2 e = make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y + zm.y));  // even-sample DFT
        const float2 d = make_float2(0.5f * (zk.x - zm.x), 0.5f * (zk.y - zm.y));
        const float2 o = make_float2(d.y, -d.x);                                    // odd-sample DFT = d / i
        L.at(c, k, y) = cadd(e, cmul(o, twid<W, false>(k)));
      }
    }
  }
  __syncthreads();

  // columns: slot 0 packs the (real) DC and Nyquist columns, slots 1..W/2-1 are kx
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.spec);
  const int C2 = 2 * p.c;
  if (live && q < HALF) {
    float2 a[H];
    if (q == 0) {
#pragma unroll
      for (int y = 0; y < H; y++) a[y] = make_float2(L.at(c, 0, y).x, L.at(c, HALF, y).x);
    } else {
#pragma unroll
      for (int y = 0; y < H; y++) a[y] = L.at(c, q, y);
    }
    fft_reg<H, false>(a);
    auto store = [&](int ky, int kx, float2 v) {
      uint32_t hi, lo;
      split_pair(v.x * p.scale, v.y * p.scale, hi, lo);
      const size_t off = (((size_t)b * H + ky) * WH + kx) * C2 + 2 * cc;
      *reinterpret_cast<uint32_t*>(out + off) = hi;
      *reinterpret_cast<uint32_t*>(out + p.spec_part + off) = lo;
    };
    if (q == 0) {
#pragma unroll
      for (int ky = 0; ky < H; ky++) {
        const float2 zk = a[ky], zm = conjf2(a[(H - ky) % H]);
        store(ky, 0, make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y + zm.y)));
        const float2 d = make_float2(0.5f * (zk.x - zm.x), 0.5f * (zk.y - zm.y));
        store(ky, HALF, make_float2(d.y, -d.x));
      }
    } else {
#pragma unroll
      for (int ky = 0; ky < H; ky++) store(ky, q, a[ky]);
    }
  }
}

// ------------------------------------------------------------------ irfft2 (+ feat)
template <int H, int W>
__global__ void __launch_bounds__(256) k_irfft2_reg(const FftParams p) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int WH = W / 2 + 1, HALF = W / 2;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const Layout L{reinterpret_cast<float2*>(smem_raw)};
  const int t = threadIdx.x, c = t % CG, q = t / CG;
  const int b = blockIdx.y, cc = blockIdx.x * CG + c;
  const bool live = cc < p.c;
  const int C2 = 2 * p.c;

  // columns (inverse): slot 0 transforms the Hermitian parts of the DC and
  // Nyquist columns together (only their real outputs are used)
  if (live && q < HALF) {
    float2 a[H];
    auto ld = [&](int ky, int kx) {
      const float2* s = reinterpret_cast<const float2*>(p.fu + (((size_t)b * H + ky) * WH + kx) * C2 + 2 * cc);
      return __ldg(s);
    };
    if (q == 0) {
#pragma unroll
      for (int k = 0; k <= H / 2; k++) {
        const int km = (H - k) % H;
        const float2 a0 = ld(k, 0), a0m = ld(km, 0), an = ld(k, HALF), anm = ld(km, HALF);
        // Hermitian parts h(k) = (v(k) + conj(v(-k))) / 2; z = h0 + i*hn
        const float2 h0 = make_float2(0.5f * (a0.x + a0m.x), 0.5f * (a0.y - a0m.y));
        const float2 hn = make_float2(0.5f * (an.x + anm.x), 0.5f * (an.y - anm.y));
        a[k] = make_float2(h0.x - hn.y, h0.y + hn.x);
        // h(-k) = conj(h(k))
        a[km] = make_float2(h0.x + hn.y, -h0.y + hn.x);
      }
    } else {
#pragma unroll
      for (int ky = 0; ky < H; ky++) a[ky] = ld(ky, q);
    }
    fft_reg<H, true>(a);
    if (q == 0) {
#pragma unroll
      for (int y = 0; y < H; y++) {
        L.at(c, 0, y) = make_float2(a[y].x, 0.f);
        L.at(c, HALF, y) = make_float2(a[y].y, 0.f);
      }
    } else {
#pragma unroll
      for (int y = 0; y < H; y++) L.at(c, q, y) = a[y];
    }
  }
  __syncthreads();

  // rows: Hermitian completion + real inverse via one complex length-W/2 transform
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.s_out);
#pragma unroll 1
  for (int y = q; y < H; y += 32) {
    if (!live) continue;
    float2 z[HALF];
#pragma unroll
    for (int k = 0; k < HALF; k++) {
      const float2 xk = L.at(c, k, y);
      const float2 xm = conjf2(L.at(c, HALF - k, y));
      const float2 e = cadd(xk, xm);                               // X[k] + X[k+W/2]
      const float2 o = cmul(csub(xk, xm), twid<W, true>(k));       // (X[k] - X[k+W/2]) e^{+2 pi i k/W}
      z[k] = make_float2(e.x - o.y, e.y + o.x);                    // e + i*o
    }
    fft_reg<HALF, true>(z);
    const float4* fr = reinterpret_cast<const float4*>(p.feat + (((size_t)b * p.c + cc) * H + y) * W);
    __nv_bfloat16* o = out + ((size_t)b * H + y) * W * p.c + cc;
#pragma unroll
    for (int i = 0; i < W / 4; i++) {
      const float4 f = __ldg(fr + i);
      const float v[4] = {z[2 * i].x * p.scale + f.x, z[2 * i].y * p.scale + f.y,
                          z[2 * i + 1].x * p.scale + f.z, z[2 * i + 1].y * p.scale + f.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
        const size_t off = (size_t)(4 * i + j) * p.c;
        o[off] = h;
        o[p.s_part + off] = __float2bfloat16_rn(v[j] - __bfloat162float(h));
      }
    }
  }
}

template <int H, int W>
int launch_pair(const FftParams& p, bool inverse, cudaStream_t st) {
  const size_t smem = (size_t)CG * KS * YS * sizeof(float2);
  dim3 grid((p.c + CG - 1) / CG, p.batch);
  if (inverse) return launch_kernel(k_irfft2_reg<H, W>, grid, dim3(256), smem, st, 1, p);
  return launch_kernel(k_rfft2_reg<H, W>, grid, dim3(256), smem, st, 1, p);
  return (int)cudaGetLastError();
}

template <int H, int W>
int prepare_pair() {
  const int smem = (int)((size_t)CG * KS * YS * sizeof(float2));
  cudaError_t e = cudaFuncSetAttribute(k_rfft2_reg<H, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  return (int)cudaFuncSetAttribute(k_irfft2_reg<H, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

// ------------------------------------------------------------------ rfft2, TMA-fed variant (64 x 64)
// Persistent CTAs, two per SM, walk items = (image, 4 channels).  The item's
// feat rows (4 x 64 rows of 256 bytes) arrive by TMA, 128-byte swizzled, in
// the first 64 KB of the CTA's plane buffer; every thread takes its row into
// registers, and after a barrier the row transforms overwrite the same bytes
// with the [c][kx][y] plane.  A CTA loads its next item once its column pass
// is done; the other CTA on the SM computes meanwhile, which hides the load.
//   rows: thread (c, y) = (t / 64, t % 64): the row as a 32-point complex
//     transform + untangling, into the plane [c][kx][y];
//   columns: thread (c, h, slot) = (t % 4, t / 4 % 2, t / 8): half h (outputs of
//     parity h, one DIF stage) of column `slot` (slot 0 = DC + i * Nyquist),
//     stored to the spectrum, 4 channels = 16 contiguous bytes per store.
constexpr int PF_CG = 4;
constexpr uint32_t PF_BOX = 256 * 128;    // one TMA box: 256 rows x 32 floats
constexpr uint32_t PF_BUF = 2 * PF_BOX;   // one item: x in [0, 32) and [32, 64)
constexpr int PF_KS = 34, PF_YS = 65;     // plane strides (float2)
constexpr size_t PF_PLANE = (size_t)PF_CG * PF_KS * PF_YS * sizeof(float2);
static_assert(PF_PLANE >= PF_BUF, "the TMA landing zone fits in the plane buffer");
constexpr size_t PF_SMEM = 1024 + PF_PLANE + 64;

__global__ void __launch_bounds__(256, 2) k_rfft2_pf(const __grid_constant__ FftPfParams q) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int H = 64, W = 64, WH = 33, HALF = 32;
  const FftParams& p = q.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float2* plane = reinterpret_cast<float2*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PF_PLANE);
  auto P = [&](int c, int kx, int y) -> float2& { return plane[(c * PF_KS + kx) * PF_YS + y]; };
  const int t = threadIdx.x;
  const int groups = p.c / PF_CG, items = p.batch * groups;
  auto issue = [&](int item) {
    const int b = item / groups, c0 = (item - b * groups) * PF_CG;
    const int row = (b * p.c + c0) * H;
    const uint32_t bar = smem_u32(full);
    mbar_arrive_expect_tx(bar, PF_BUF);
    tma_load_2d(smem_u32(smem), &q.feat_map, 0, row, bar);
    tma_load_2d(smem_u32(smem + PF_BOX), &q.feat_map, 32, row, bar);
  };
  if (t == 0) {
    mbar_init(smem_u32(full), 1);
    fence_mbar_init();
    tma_prefetch(&q.feat_map);
    if (blockIdx.x < items) issue(blockIdx.x);
  }
  __syncthreads();
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.spec);
  const int C2 = 2 * p.c;
  int k = 0;
  for (int item = blockIdx.x; item < items; item += gridDim.x, k++) {
    const bool ok = __syncthreads_and(mbar_wait(smem_u32(full), k & 1, p.err, 7));
    if (!ok) break;
    const int b = item / groups, c0 = (item - b * groups) * PF_CG;
    {
      const int c = t >> 6, y = t & 63, r = c * 64 + y;
      const uint8_t* rowb = smem + r * 128;
      float2 z[HALF];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const float4 v = *reinterpret_cast<const float4*>(rowb + (i >> 3) * PF_BOX + (((i & 7) ^ (r & 7)) << 4));
        z[2 * i] = make_float2(v.x, v.y);
        z[2 * i + 1] = make_float2(v.z, v.w);
      }
      __syncthreads();  // every row is in registers: the plane may overwrite the landing zone
      fft_reg<HALF, false>(z);
#pragma unroll
      for (int kx = 0; kx <= HALF; kx++) {
        const float2 zk = z[kx % HALF], zm = conjf2(z[(HALF - kx) % HALF]);
        const float2 e = make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y + zm.y));  // even-sample DFT
        const float2 d = make_float2(0.5f * (zk.x - zm.x), 0.5f * (zk.y - zm.y));
        const float2 o = make_float2(d.y, -d.x);                                    // odd-sample DFT = d / i
        P(c, kx, y) = cadd(e, cmul(o, twid<W, false>(kx)));
      }
    }
    __syncthreads();  // plane complete
    {
      const int c = t & 3, h = (t >> 2) & 1, slot = t >> 3;
      float2 u[HALF];
#pragma unroll
      for (int n = 0; n < HALF; n++) {
        float2 a, bb;
        if (slot == 0) {
          a = make_float2(P(c, 0, n).x, P(c, HALF, n).x);
          bb = make_float2(P(c, 0, n + HALF).x, P(c, HALF, n + HALF).x);
        } else {
          a = P(c, slot, n);
          bb = P(c, slot, n + HALF);
        }
        u[n] = h ? cmul(csub(a, bb), twid<H, false>(n)) : cadd(a, bb);
      }
      __syncthreads();  // the plane is read: the next item's rows may land in it
      if (t == 0 && item + gridDim.x < items) {
        fence_async_smem();
        issue(item + gridDim.x);
      }
      fft_reg<HALF, false>(u);  // u[k2] = X[2 k2 + h]
      const int cc = c0 + c;
      auto store = [&](int ky, int kx, float2 v) {
        uint32_t hi, lo;
        split_pair(v.x * p.scale, v.y * p.scale, hi, lo);
        const size_t off = (((size_t)b * H + ky) * WH + kx) * C2 + 2 * cc;
        *reinterpret_cast<uint32_t*>(out + off) = hi;
        *reinterpret_cast<uint32_t*>(out + p.spec_part + off) = lo;
      };
      if (slot == 0) {
#pragma unroll
        for (int k2 = 0; k2 < HALF; k2++) {
          // X[ky] of a + i b and X[-ky] (same parity, this thread)
          const float2 zk = u[k2];
          const float2 zm = conjf2(h ? u[HALF - 1 - k2] : u[(HALF - k2) % HALF]);
          const int ky = 2 * k2 + h;
          store(ky, 0, make_float2(0.5f * (zk.x + zm.x), 0.5f * (zk.y + zm.y)));
          const float2 d = make_float2(0.5f * (zk.x - zm.x), 0.5f * (zk.y - zm.y));
          store(ky, HALF, make_float2(d.y, -d.x));
        }
      } else {
#pragma unroll
        for (int k2 = 0; k2 < HALF; k2++) store(2 * k2 + h, slot, u[k2]);
      }
    }
  }
}

// ------------------------------------------------------------------ irfft2 by row parity (64 x 64)
// One CTA = one image x CG channels x one parity h of the output rows: the
// column pass computes only the outputs y = 2m + h of every inverse column
// transform (one decimation-in-frequency stage, then 32 points in
// registers), so the half plane [CG][kx][32] fits in shared memory.
//   CG = 16, 256 threads (batches): the row pass stores S with 16 channels =
//     32 contiguous bytes per pixel and part; each thread runs three column
//     and two row transforms;
//   CG = 4, 128 threads (small batches, where 16-channel CTAs would leave most
//     SMs idle): four times the CTAs, one column and one row transform per
//     thread, 8-byte runs of S.
constexpr int PAR_KS = 34, PAR_YS = 33;
template <int CG>
constexpr size_t par_smem() { return (size_t)CG * PAR_KS * PAR_YS * sizeof(float2); }

template <int CG, int NT>
__global__ void __launch_bounds__(NT, 1) k_irfft2_par(const FftParams p) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr int H = 64, W = 64, WH = 33, HALF = 32;
  constexpr int STEP = NT / CG;  // column slots (and output rows) per pass over the CTA's threads
  extern __shared__ __align__(16) float2 zp[];
  auto P = [&](int c, int kx, int m) -> float2& { return zp[(c * PAR_KS + kx) * PAR_YS + m]; };
  const int t = threadIdx.x, h = blockIdx.z, b = blockIdx.y, c0 = blockIdx.x * CG;
  const int c = t % CG, cc = c0 + c;
  const int C2 = 2 * p.c;
  auto ld = [&](int ky, int kx) {
    return __ldg(reinterpret_cast<const float2*>(p.fu + (((size_t)b * H + ky) * WH + kx) * C2 + 2 * cc));
  };
  // Hermitian parts of the DC and Nyquist columns, h(k) = (v(k) + conj(v(-k))) / 2,
  // packed as z = h0 + i * hn
  auto packed = [&](int ky) {
    const int km = (H - ky) % H;
    const float2 a0 = ld(ky, 0), a0m = ld(km, 0), an = ld(ky, HALF), anm = ld(km, HALF);
    const float2 h0 = make_float2(0.5f * (a0.x + a0m.x), 0.5f * (a0.y - a0m.y));
    const float2 hn = make_float2(0.5f * (an.x + anm.x), 0.5f * (an.y - anm.y));
    return make_float2(h0.x - hn.y, h0.y + hn.x);
  };
#pragma unroll 1
  for (int slot = t / CG; slot < HALF; slot += STEP) {
    float2 u[HALF];
    if (slot == 0) {
#pragma unroll
      for (int n = 0; n < HALF; n++) {
        const float2 a = packed(n), bb = packed(n + HALF);
        u[n] = h ? cmul(csub(a, bb), twid<H, true>(n)) : cadd(a, bb);
      }
    } else {
#pragma unroll
      for (int n = 0; n < HALF; n++) {
        const float2 a = ld(n, slot), bb = ld(n + HALF, slot);
        u[n] = h ? cmul(csub(a, bb), twid<H, true>(n)) : cadd(a, bb);
      }
    }
    fft_reg<HALF, true>(u);  // u[m] = y[2m + h]
    if (slot == 0) {
#pragma unroll
      for (int m = 0; m < HALF; m++) {
        P(c, 0, m) = make_float2(u[m].x, 0.f);
        P(c, HALF, m) = make_float2(u[m].y, 0.f);
      }
    } else {
#pragma unroll
      for (int m = 0; m < HALF; m++) P(c, slot, m) = u[m];
    }
  }
  __syncthreads();
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.s_out);
#pragma unroll 1
  for (int m = t / CG; m < HALF; m += STEP) {
    const int y = 2 * m + h;
    float2 z[HALF];
#pragma unroll
    for (int kx = 0; kx < HALF; kx++) {
      const float2 xk = P(c, kx, m);
      const float2 xm = conjf2(P(c, HALF - kx, m));
      const float2 e = cadd(xk, xm);                           // X[k] + X[k+W/2]
      const float2 o = cmul(csub(xk, xm), twid<W, true>(kx));  // (X[k] - X[k+W/2]) e^{+2 pi i k/W}
      z[kx] = make_float2(e.x - o.y, e.y + o.x);               // e + i*o
    }
    fft_reg<HALF, true>(z);
    const float4* fr = reinterpret_cast<const float4*>(p.feat + (((size_t)b * p.c + cc) * H + y) * W);
    __nv_bfloat16* o = out + ((size_t)b * H + y) * W * p.c + cc;
#pragma unroll
    for (int i = 0; i < W / 4; i++) {
      const float4 f = __ldg(fr + i);
      const float v[4] = {z[2 * i].x * p.scale + f.x, z[2 * i].y * p.scale + f.y,
                          z[2 * i + 1].x * p.scale + f.z, z[2 * i + 1].y * p.scale + f.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const __nv_bfloat16 hv = __float2bfloat16_rn(v[j]);
        const size_t off = (size_t)(4 * i + j) * p.c;
        o[off] = hv;
        o[p.s_part + off] = __float2bfloat16_rn(v[j] - __bfloat162float(hv));
      }
    }
  }
}

template <int H>
int dispatch_w(const FftParams& p, bool inv, cudaStream_t st) {
  switch (p.w) {
    case 8: return launch_pair<H, 8>(p, inv, st);
    case 16: return launch_pair<H, 16>(p, inv, st);
    case 32: return launch_pair<H, 32>(p, inv, st);
    case 64: return launch_pair<H, 64>(p, inv, st);
  }
  return -1;
}

template <int H>
int prepare_w() {
  int e;
  if ((e = prepare_pair<H, 8>())) return e;
  if ((e = prepare_pair<H, 16>())) return e;
  if ((e = prepare_pair<H, 32>())) return e;
  return prepare_pair<H, 64>();
}

}  // namespace

bool fft_pf_supported(int c, int h, int w) { return h == 64 && w == 64 && c % PF_CG == 0; }

int fft_pf_prepare() {
  cudaError_t e = cudaFuncSetAttribute(k_rfft2_pf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM);
  if (e != cudaSuccess) return (int)e;
  e = cudaFuncSetAttribute(k_irfft2_par<16, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)par_smem<16>());
  if (e != cudaSuccess) return (int)e;
  return (int)cudaFuncSetAttribute(k_irfft2_par<4, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)par_smem<4>());
}

bool irfft2_par_narrow(int c, int batch, int sms) { return c % 4 == 0 && batch * (c / 16) * 2 < sms; }

int launch_irfft2_par(const FftParams& p, int sms, cudaStream_t st) {
  if (irfft2_par_narrow(p.c, p.batch, sms))
    return launch_kernel(k_irfft2_par<4, 128>, dim3(p.c / 4, p.batch, 2), dim3(128), par_smem<4>(), st, 1, p);
  return launch_kernel(k_irfft2_par<16, 256>, dim3(p.c / 16, p.batch, 2), dim3(256), par_smem<16>(), st, 1, p);
}

int launch_rfft2_pf(const FftPfParams& q, int grid, cudaStream_t st) {
  return launch_kernel(k_rfft2_pf, dim3(grid), dim3(256), PF_SMEM, st, 1, q);
}


bool fft_reg_supported(int h, int w) {
  auto ok = [](int n) { return n == 8 || n == 16 || n == 32 || n == 64; };
  return ok(h) && ok(w);
}

int fft_reg_prepare() {
  float2 tw[64];
  for (int m = 0; m < 64; m++) {
    const double a = 2.0 * 3.14159265358979323846 * (double)m / 64.0;
    tw[m] = make_float2((float)cos(a), (float)sin(a));
  }
  cudaError_t e = cudaMemcpyToSymbol(c_tw64, tw, sizeof(tw));
  if (e != cudaSuccess) return (int)e;
  int r;
  if ((r = prepare_w<8>())) return r;
  if ((r = prepare_w<16>())) return r;
  if ((r = prepare_w<32>())) return r;
  return prepare_w<64>();
}

int launch_fft_reg(const FftParams& p, bool inverse, cudaStream_t st) {
  switch (p.h) {
    case 8: return dispatch_w<8>(p, inverse, st);
    case 16: return dispatch_w<16>(p, inverse, st);
    case 32: return dispatch_w<32>(p, inverse, st);
    case 64: return dispatch_w<64>(p, inverse, st);
  }
  return -1;
}

}  // namespace lama
