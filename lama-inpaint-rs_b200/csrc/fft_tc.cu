// Tensor-core rfft2 of 64 x 64 planes (tcgen05).
//
// The same transform as the other rfft2 kernels (the reference's rfft2_ortho,
// lama-rs/src/cpu.rs:769-800, standard directions for power-of-two sides,
// cpu.rs:888-927), written as two small real GEMMs per item of (image, 4
// channels), each run as three BF16 MMAs of split operands (hi*hi + hi*lo +
// lo*hi, FP32 accumulation in TMEM), like the convolutions:
//   rows:    R[(c,y)][n] = sum_x feat[c][y][x] Wr[n][x] with the real-input
//            row packed into N = 64: n = 0 Re R[0] (weight 1), n = 1 Re R[32]
//            ((-1)^x), n = 2 kx, 2 kx + 1 Re, Im R[kx] (cos, -sin),
//            kx = 1..31 (Im R[0] = Im R[32] = 0 for real rows); one MMA tile =
//            2 channels x 64 rows (M = 128), K = 64 (x);
//   columns: X[(ky,r)][(kx,c)] = sum_(y,r') Fc[(ky,r)][(y,r')] R[(c,y)][(kx,r')],
//            Fc = [[cos, sin], [-sin, cos]](2 pi ky y / 64) / 64 (the ortho
//            scale, exact) with re/im interleaved in M and K; M = 128,
//            N = 33 kx x 4 channels = 132 -> 144, K = 128.
// Input and output keep the layouts of the other spectral kernels: feat fp32
// NCHW, the spectrum split bf16 [2][B][64][33][2C].
// Persistent CTAs (one per SM, 216 KB of shared memory, 512 TMEM columns)
// walk items; warp roles:
//   warp 8 (one thread): TMA loads of feat and the MMAs;
//   warps 0-3: split each landed half item (2 channels, fp32) in place into
//     the row GEMM's bf16 hi/lo A operand, then move the row GEMM's result
//     from TMEM into the column GEMM's B operand (split, transposed);
//   warps 4-7: the column GEMM's result -> split spectrum, one 16-byte run (4
//     channels x re/im) per bin and part.
// Measured: the item period is set by those 16-byte spectrum stores (2112 per
// item and part, one 128-byte line each); twice the epilogue warps made each
// epilogue slower, not the item shorter.
// Every wait is bounded (error codes 20-28 in the device status word).
#include <cmath>
#include <cstdint>
#include <cstring>

#include "fft.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace lama {
namespace {

constexpr int TC_CG = 4;                  // channels per item
constexpr uint32_t TC_BOX = 16384;        // one TMA box: 128 rows x 32 floats
constexpr uint32_t TC_HALF = 2 * TC_BOX;  // half an item: 2 channels x 64 rows x 64 floats
constexpr int TC_N1 = 64;                 // row GEMM N
constexpr int TC_N2 = 144;                // column GEMM N (132 used)
constexpr uint32_t TC_WR = TC_N1 * 128;   // one part of Wr: 64 rows x 64 bf16
constexpr uint32_t TC_FCB = 128 * 128;    // one (K block, part) of Fc: 128 rows x 64 bf16
constexpr uint32_t TC_B2B = TC_N2 * 128;  // one (K block, part) of the column GEMM's B
constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_WR = OFF_A + 2 * TC_HALF;
constexpr uint32_t OFF_FC = OFF_WR + 2 * TC_WR;
constexpr uint32_t OFF_B2 = OFF_FC + 4 * TC_FCB;
constexpr uint32_t OFF_BAR = OFF_B2 + 4 * TC_B2B;
constexpr uint32_t TC_TAB = OFF_B2 - OFF_WR;  // Wr and Fc, copied as one block
constexpr size_t TC_SMEM = 1024 + OFF_BAR + 128;
constexpr uint32_t TC_TMEM = 512;
constexpr uint32_t TC_D2 = 256;  // TMEM column of the column GEMM's accumulator
static_assert(TC_SMEM <= 232448, "fits one SM's shared memory");
static_assert(OFF_WR % 1024 == 0 && OFF_FC % 1024 == 0 && OFF_B2 % 1024 == 0 && TC_WR % 1024 == 0 &&
                  TC_B2B % 1024 == 0,
              "swizzle atoms stay 1024-byte aligned");

// barriers
enum { B_LOAD = 0, B_A1 = 2, B_M1 = 4, B_B2 = 6, B_M2 = 7, B_D2E = 8, B_TAB = 9, B_COUNT = 10 };

// Byte offset of 16-byte chunk `chunk` of row `row` in a K-major operand with
// 128-byte rows and the 128-byte swizzle (rows of 64 bf16 or 32 floats).
__host__ __device__ constexpr uint32_t sw128(uint32_t row, uint32_t chunk) {
  return row * 128 + (((chunk ^ (row & 7)) & 7) << 4);
}

__global__ void __launch_bounds__(288, 1) k_rfft2_tc(const __grid_constant__ FftTcParams q) {
  pdl_launch_dependents();
  const FftParams& p = q.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = p.c / TC_CG, items = p.batch * groups;

  if (threadIdx.x == 0) {
    for (int i = 0; i < B_COUNT; i++) mbar_init(bar(i), 1);
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(tmem_slot), TC_TMEM);
    tmem_relinquish();
  }
  if (warp >= 4 && warp < 8) {
    // rows 132..143 of the column GEMM's B blocks are padding: zero them once
    for (int i = threadIdx.x - 128; i < 4 * 12 * 8; i += 128) {
      const int blk = i / 96, rem = i % 96;
      *reinterpret_cast<uint4*>(smem + OFF_B2 + blk * TC_B2B + 132 * 128 + rem * 16) = make_uint4(0, 0, 0, 0);
    }
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();

  if (warp == 8) {
    if (lane == 0) {
      tma_prefetch(&q.map);
      mbar_arrive_expect_tx(bar(B_TAB), TC_TAB);
      bulk_load(s0 + OFF_WR, q.tab, TC_TAB, bar(B_TAB));
      auto issue = [&](int item, int h) {
        const int b = item / groups, c0 = (item - b * groups) * TC_CG + 2 * h;
        const int row = (b * p.c + c0) * 64;
        mbar_arrive_expect_tx(bar(B_LOAD + h), TC_HALF);
        tma_load_2d(s0 + OFF_A + h * TC_HALF, &q.map, 0, row, bar(B_LOAD + h));
        tma_load_2d(s0 + OFF_A + h * TC_HALF + TC_BOX, &q.map, 32, row, bar(B_LOAD + h));
      };
      int last_load = -1, last_m1 = -1, last_m2 = -1;  // item counts of the last copies / commits issued
      if ((int)blockIdx.x < items) {
        issue(blockIdx.x, 0);
        issue(blockIdx.x, 1);
        last_load = 0;
      }
      constexpr uint32_t ID1 = idesc_bf16_f32(TC_N1), ID2 = idesc_bf16_f32(TC_N2);
      bool ok = mbar_wait(bar(B_TAB), 0, p.err, 20);
      int k = 0;
      for (int item = blockIdx.x; ok && item < items; item += gridDim.x, k++) {
        const uint32_t ph = k & 1;
        // row GEMM, one half item (2 channels) at a time, once it is split
        for (int h = 0; h < 2; h++) {
          if (!(ok = mbar_wait(bar(B_A1 + h), ph, p.err, 21))) break;
          tc_fence_after();
          const uint32_t a = s0 + OFF_A + h * TC_HALF, w = s0 + OFF_WR, d = tmem + h * TC_N1;
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint64_t ahi = smem_desc(a + kk * 32, 1024u, 2u), alo = smem_desc(a + TC_BOX + kk * 32, 1024u, 2u);
            const uint64_t bhi = smem_desc(w + kk * 32, 1024u, 2u), blo = smem_desc(w + TC_WR + kk * 32, 1024u, 2u);
            mma_bf16(d, alo, bhi, ID1, kk > 0 ? 1u : 0u);
            mma_bf16(d, ahi, blo, ID1, 1u);
            mma_bf16(d, ahi, bhi, ID1, 1u);
          }
          mma_commit(bar(B_M1 + h));
          last_m1 = k;
        }
        if (!ok) break;
        // the next item's halves land where this item's A operand was read
        const int next = item + gridDim.x;
        if (next < items) {
          for (int h = 0; h < 2; h++) {
            if (!(ok = mbar_wait(bar(B_M1 + h), ph, p.err, 22))) break;
            issue(next, h);
            last_load = k + 1;
          }
          if (!ok) break;
        }
        // column GEMM once its B operand is staged and the previous result is read
        if (!(ok = mbar_wait(bar(B_B2), ph, p.err, 23))) break;
        if (k > 0 && !(ok = mbar_wait(bar(B_D2E), ph ^ 1u, p.err, 24))) break;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; kb++)
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint32_t a = s0 + OFF_FC + kb * 2 * TC_FCB + kk * 32, b = s0 + OFF_B2 + kb * 2 * TC_B2B + kk * 32;
            const uint64_t ahi = smem_desc(a, 1024u, 2u), alo = smem_desc(a + TC_FCB, 1024u, 2u);
            const uint64_t bhi = smem_desc(b, 1024u, 2u), blo = smem_desc(b + TC_B2B, 1024u, 2u);
            mma_bf16(tmem + TC_D2, alo, bhi, ID2, (kb | kk) ? 1u : 0u);
            mma_bf16(tmem + TC_D2, ahi, blo, ID2, 1u);
            mma_bf16(tmem + TC_D2, ahi, bhi, ID2, 1u);
          }
        mma_commit(bar(B_M2));
        last_m2 = k;
      }
      // everything this thread issued has finished before the CTA tears down
      // (already so unless a wait above ran out)
      if (last_load >= 0)
        for (int h = 0; h < 2; h++) mbar_wait_drain(bar(B_LOAD + h), last_load & 1);
      if (last_m1 >= 0)
        for (int h = 0; h < 2; h++) mbar_wait_drain(bar(B_M1 + h), last_m1 & 1);
      if (last_m2 >= 0) mbar_wait_drain(bar(B_M2), last_m2 & 1);
    }
  } else if (warp < 4) {
    const int t = threadIdx.x;  // row (channel t / 64, y = t % 64) of a half item
    int k = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x, k++) {
      const uint32_t ph = k & 1;
      bool ok = true;
      for (int h = 0; h < 2; h++) {
        if (!(ok = named_sync_and(1, 128, mbar_wait(bar(B_LOAD + h), ph, p.err, 25)))) break;
        // fp32 row t (x in [0,32) in box 0, [32,64) in box 1) -> hi over box 0's
        // row t, lo over box 1's row t (the row is in registers before the stores)
        uint8_t* base = smem + OFF_A + h * TC_HALF;
        float4 v[16];
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = *reinterpret_cast<const float4*>(base + (j >> 3) * TC_BOX + sw128(t, j & 7));
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const float4 a = v[2 * c], b = v[2 * c + 1];
          uint4 hi, lo;
          split_pair(a.x, a.y, hi.x, lo.x);
          split_pair(a.z, a.w, hi.y, lo.y);
          split_pair(b.x, b.y, hi.z, lo.z);
          split_pair(b.z, b.w, hi.w, lo.w);
          *reinterpret_cast<uint4*>(base + sw128(t, c)) = hi;
          *reinterpret_cast<uint4*>(base + TC_BOX + sw128(t, c)) = lo;
        }
        fence_async_smem();
        named_sync(1, 128);
        if (t == 0) mbar_arrive(bar(B_A1 + h));
      }
      if (!ok) break;
      // row GEMM result (both halves) -> the column GEMM's B operand, once the
      // previous column GEMM has read it
      ok = mbar_wait(bar(B_M1 + 1), ph, p.err, 26);
      if (ok && k > 0) ok = mbar_wait(bar(B_M2), ph ^ 1u, p.err, 27);
      if (!named_sync_and(1, 128, ok)) break;
      tc_fence_after();
      // TMEM lane 32 * warp + lane = (channel 2h + warp / 2, y = 32 (warp & 1) + lane);
      // B row 4 kx + channel holds K = (y, re/im): this thread's word is
      // (Re R[y][kx], Im R[y][kx]) at K offset 2y of block y / 32
      uint8_t* bhi = smem + OFF_B2 + (warp & 1) * 2 * TC_B2B;
      uint8_t* blo = bhi + TC_B2B;
      auto put = [&](int row, float re, float im) {
        uint32_t hi, lo;
        split_pair(re, im, hi, lo);
        const uint32_t off = sw128(row, lane >> 2) + ((lane & 3) << 2);
        *reinterpret_cast<uint32_t*>(bhi + off) = hi;
        *reinterpret_cast<uint32_t*>(blo + off) = lo;
      };
#pragma unroll 1
      for (int h = 0; h < 2; h++) {
        const int c = 2 * h + (warp >> 1);
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + h * TC_N1;
        float v[64];
        tmem_ld32(ta, v);
        tmem_wait_ld();
        tmem_ld32(ta + 32, v + 32);
        tmem_wait_ld();
        put(c, v[0], 0.f);           // kx = 0
        put(4 * 32 + c, v[1], 0.f);  // kx = 32
#pragma unroll
        for (int kx = 1; kx < 32; kx++) put(4 * kx + c, v[2 * kx], v[2 * kx + 1]);
      }
      tc_fence_before();
      fence_async_smem();
      named_sync(1, 128);
      if (t == 0) mbar_arrive(bar(B_B2));
    }
  } else {
    // TMEM lane 32 * (warp - 4) + lane = 2 ky + r of the column GEMM's result;
    // column 4 kx + c.  The (re, im) lane pair forms each bin's two 16-byte
    // runs: the re lane stores the hi part, the im lane the lo part.
    const int qw = warp - 4, L = 32 * qw + lane, ky = L >> 1, r = L & 1;
    const int C2 = 2 * p.c;
    int k = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x, k++) {
      if (!named_sync_and(2, 128, mbar_wait(bar(B_M2), k & 1, p.err, 28))) break;
      tc_fence_after();
      const int b = item / groups, c0 = (item - b * groups) * TC_CG;
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.spec) + (size_t)(b * 64 + ky) * 33 * C2 + 2 * c0 +
                           (r ? p.spec_part : 0);
      const uint32_t ta = tmem + ((uint32_t)(qw * 32) << 16) + TC_D2;
#pragma unroll 1
      for (int j = 0; j < 9; j++) {
        float v[16];
        tmem_ld16(ta + 16 * j, v);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int kx = 4 * j + u;
          if (kx > 32) break;
          uint32_t h01, l01, h23, l23;
          split_pair(v[4 * u], v[4 * u + 1], h01, l01);
          split_pair(v[4 * u + 2], v[4 * u + 3], h23, l23);
          const uint32_t g01 = __shfl_xor_sync(0xffffffffu, r ? h01 : l01, 1);
          const uint32_t g23 = __shfl_xor_sync(0xffffffffu, r ? h23 : l23, 1);
          const uint32_t re01 = r ? g01 : h01, im01 = r ? l01 : g01;
          const uint32_t re23 = r ? g23 : h23, im23 = r ? l23 : g23;
          uint4 o;
          o.x = __byte_perm(re01, im01, 0x5410);
          o.y = __byte_perm(re01, im01, 0x7632);
          o.z = __byte_perm(re23, im23, 0x5410);
          o.w = __byte_perm(re23, im23, 0x7632);
          *reinterpret_cast<uint4*>(dst + (size_t)kx * C2) = o;
        }
      }
      tc_fence_before();
      named_sync(2, 128);
      if (threadIdx.x == 128) mbar_arrive(bar(B_D2E));
    }
  }
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, TC_TMEM);
  }
}

uint16_t bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float bf16_float(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

}  // namespace

bool fft_tc_supported(int c, int h, int w) { return h == 64 && w == 64 && c % TC_CG == 0; }

size_t fft_tc_table_bytes() { return TC_TAB; }

// Wr (hi part, lo part) then Fc ([K block][part]), each laid out exactly as
// the kernel's shared-memory operand (K-major, 128-byte rows, 128-byte swizzle
// relative to a 1024-byte aligned base).  cos / sin of 2 pi a / 64 in double,
// exact at the multiples of pi / 2; split x = hi + lo, hi = bf16(x),
// lo = bf16(x - hi).
void fft_tc_table(uint8_t* out) {
  memset(out, 0, TC_TAB);
  auto cs = [](int a, double& c, double& s) {
    a &= 63;
    const double t = 2.0 * M_PI * (double)a / 64.0;
    c = (a == 16 || a == 48) ? 0.0 : std::cos(t);
    s = (a == 0 || a == 32) ? 0.0 : std::sin(t);
  };
  auto put = [&](uint32_t part0, uint32_t part1, int row, int k, double x) {
    const uint16_t hi = bf16_rne((float)x);
    const uint16_t lo = bf16_rne((float)(x - (double)bf16_float(hi)));
    const uint32_t off = sw128(row, k >> 3) + (k & 7) * 2;
    memcpy(out + part0 + off, &hi, 2);
    memcpy(out + part1 + off, &lo, 2);
  };
  // Wr[n][x]: the packed real row (DC, Nyquist, then Re / Im of kx = 1..31)
  for (int x = 0; x < 64; x++) {
    put(0, TC_WR, 0, x, 1.0);
    put(0, TC_WR, 1, x, (x & 1) ? -1.0 : 1.0);
    for (int kx = 1; kx < 32; kx++) {
      double c, s;
      cs(kx * x, c, s);
      put(0, TC_WR, 2 * kx, x, c);
      put(0, TC_WR, 2 * kx + 1, x, -s);
    }
  }
  // Fc / 64 (the ortho scale): Re X = cos Re R + sin Im R, Im X = -sin Re R + cos Im R
  const uint32_t fc = OFF_FC - OFF_WR;
  for (int ky = 0; ky < 64; ky++)
    for (int y = 0; y < 64; y++) {
      double c, s;
      cs(ky * y, c, s);
      c /= 64.0;
      s /= 64.0;
      const int kb = y / 32, k = 2 * (y % 32);
      const uint32_t p0 = fc + kb * 2 * TC_FCB, p1 = p0 + TC_FCB;
      put(p0, p1, 2 * ky, k, c);
      put(p0, p1, 2 * ky, k + 1, s);
      put(p0, p1, 2 * ky + 1, k, -s);
      put(p0, p1, 2 * ky + 1, k + 1, c);
    }
}

int fft_tc_prepare() {
  return (int)cudaFuncSetAttribute(k_rfft2_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
}

int launch_rfft2_tc(const FftTcParams& q, int grid, cudaStream_t st) {
  return launch_kernel(k_rfft2_tc, dim3(grid), dim3(288), TC_SMEM, st, 1, q);
}

}  // namespace lama
