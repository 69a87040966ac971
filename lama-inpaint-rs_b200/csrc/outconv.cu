// OutConv 7x7 64 -> 3 + bias + sigmoid (model.34 / model.35 of big-lama;
// lama-rs/src/cuda.rs:1683-1691 k_conv7x7 + lg_sigmoid, cpu.rs:540-552) with
// every input row read once.
//
// The tensor core computes, for one padded input row r and 128 input columns
// of a strip, all 147 tap products P[px][n], n = ky*21 + kx*3 + co (N = 160,
// K = the 64 input channels, three BF16 MMAs of split operands).  Output
// pixel (y, x) of channel co is the sum over (ky, kx) of P of input row
// y + ky at column x + kx.  TMEM lane = input column: the 128 rows of A are
// four groups of 32 input columns that start 26 columns apart, so lane l < 26
// of a warp finds the inputs x .. x + 6 of its output column x in its own
// warp and takes P[x + kx][*] from the lane kx places up (warp shuffles).
// The kx sums go into a ring of seven output-row accumulators in registers;
// output row r - 6 is complete after input row r and is stored (sigmoid,
// fp32 NCHW).
//
// Work units are (image, strip of 104 output columns, segment of 16..64
// output rows, read with 6 extra input rows).  Warp 0 issues the TMA loads
// (four 32 x 64 boxes per row and part, weights once),
// warp 1 the MMAs into a double-buffered TMEM accumulator, warp 2 owns TMEM,
// warps 4..11 are the epilogue: warps 4+q (part 0, ky 0..3) and 8+q (part 1,
// ky 4..6) read TMEM lanes 32q.. and keep their own rings; part 1 hands its
// sums of a completed row to part 0 (through a buffer per row parity, one
// named barrier per row), which adds the bias and stores.
#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "outconv.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace lama {
namespace {

constexpr int OC_N = 160;                    // 147 products, padded to a multiple of 16
constexpr int OC_NST = 5;                    // A stages
constexpr uint32_t OC_A = 128 * 64 * 2;      // one part of one input-row tile
constexpr uint32_t OC_STAGE = 2 * OC_A;      // hi + lo
constexpr uint32_t OC_WPART = OC_N * 64 * 2;  // one part of the weights
// [2][128][3]: part 1's sums of ky 4..6 for a completed row, by row parity
constexpr uint32_t OC_X_OFF = OC_NST * OC_STAGE + 2 * OC_WPART;
constexpr uint32_t OC_BAR_OFF = OC_X_OFF + 2 * 128 * 3 * 4;
constexpr size_t OC_SMEM = 1024 + OC_BAR_OFF + 256;
constexpr int OC_QCOLS = 26;                 // output columns of a warp (32 input columns)
constexpr int OC_STRIP = 4 * OC_QCOLS, OC_SEG_MAX = 64;

__global__ void __launch_bounds__(384, 1) k_outconv_ring(const __grid_constant__ OutConvParams q) {
  pdl_launch_dependents();
  pdl_wait();
  constexpr uint32_t IDESC = idesc_bf16_f32(OC_N);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* X = reinterpret_cast<float*>(smem + OC_X_OFF);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OC_BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * OC_NST + 5);
  const uint32_t smem0 = smem_u32(smem);
  const uint32_t wbase = smem0 + OC_NST * OC_STAGE;
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + OC_NST + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * OC_NST + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * OC_NST + 2 + a); };
  const uint32_t wbar = smem_u32(bars + 2 * OC_NST + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = q.batch * q.strips * q.segs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < OC_NST; s++) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 256);
    }
    mbar_init(wbar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&q.amap);
    tma_prefetch(&q.wmap);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // input rows of a unit (padded coordinates start at the segment's first output row)
  auto decode = [&](int u, int& b, int& x0, int& y0, int& nout) {
    const int per_b = q.strips * q.segs;
    b = u / per_b;
    const int r = u - b * per_b, s = r / q.segs, g = r - s * q.segs;
    x0 = s * OC_STRIP;
    y0 = g * q.seg;
    nout = min(q.seg, q.h - y0);
  };

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(wbar, 2 * OC_WPART);
      tma_load_3d(wbase, &q.wmap, 0, 0, 0, wbar);
      tma_load_3d(wbase + OC_WPART, &q.wmap, 0, 0, 1, wbar);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int b, x0, y0, nout;
        decode(u, b, x0, y0, nout);
        for (int rr = 0; rr < nout + 6; rr++) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, q.err, 11)) { ok = false; break; }
          mbar_arrive_expect_tx(full_bar(stage), OC_STAGE);
          const uint32_t sa = smem0 + stage * OC_STAGE;
#pragma unroll
          for (int part = 0; part < 2; part++)
#pragma unroll
            for (int g = 0; g < 4; g++)  // A rows 32g.. = input columns x0 + 26g ..
              tma_load_5d(sa + part * OC_A + g * 4096, &q.amap, 0, x0 + g * OC_QCOLS, y0 + rr, b, part,
                          full_bar(stage));
          if (++stage == OC_NST) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(wbar, 0, q.err, 12);
      tc_fence_after();
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int b, x0, y0, nout;
        decode(u, b, x0, y0, nout);
        for (int rr = 0; rr < nout + 6 && ok; rr++, it++) {
          const int acc = it & 1;
          if (!mbar_wait(tempty_bar(acc), ((it >> 1) & 1) ^ 1, q.err, 13)) { ok = false; break; }
          if (!mbar_wait(full_bar(stage), phase, q.err, 14)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem0 + stage * OC_STAGE;
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * OC_N);
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const uint64_t a_hi = smem_desc(sa + k * 32, 1024u, 2u);
            const uint64_t a_lo = smem_desc(sa + OC_A + k * 32, 1024u, 2u);
            const uint64_t b_hi = smem_desc(wbase + k * 32, 1024u, 2u);
            const uint64_t b_lo = smem_desc(wbase + OC_WPART + k * 32, 1024u, 2u);
            mma_bf16(d_tmem, a_lo, b_hi, IDESC, k != 0 ? 1u : 0u);
            mma_bf16(d_tmem, a_hi, b_lo, IDESC, 1u);
            mma_bf16(d_tmem, a_hi, b_hi, IDESC, 1u);
          }
          mma_commit(empty_bar(stage));
          mma_commit(tfull_bar(acc));
          if (++stage == OC_NST) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp >= 4) {
    const int quarter = (warp - 4) & 3, part = (warp - 4) >> 2;
    const int px = quarter * 32 + lane;        // TMEM lane
    const int ox = quarter * OC_QCOLS + lane;  // strip column: input column of the lane, output column if lane < 26
    const float bias0 = __ldg(q.bias), bias1 = __ldg(q.bias + 1), bias2 = __ldg(q.bias + 2);
    // Every epilogue thread passes the same named barriers the same number of
    // times, also after a bounded wait has run out (then it only takes part
    // in the barriers), so no thread can be left waiting on one.
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int b, x0, y0, nout;
      decode(u, b, x0, y0, nout);
      const int nin = nout + 6;
      const bool col = lane < OC_QCOLS && x0 + ox < q.w;
      float* ob = q.out + (size_t)b * 3 * q.h * q.w + (size_t)y0 * q.w + x0 + ox;
      float acc[7][3];
#pragma unroll
      for (int s = 0; s < 7; s++) acc[s][0] = acc[s][1] = acc[s][2] = 0.f;
      for (int base = 0; base < nin; base += 7) {
#pragma unroll
        for (int i = 0; i < 7; i++) {
          const int rr = base + i;
          if (rr >= nin) break;
          const int a = it & 1;
          // u8 path: this row's source bytes are loaded before the accumulator
          // wait, so their latency is hidden by it (used after the row's sums)
          uint32_t src = 0;  // mask byte << 24
          bool src_in = false;
          if (part == 0 && col && rr >= 6 && (q.win || q.dst)) {
            const int y = y0 + rr - 6, x = x0 + ox;
            if (q.win) {
              const WinDesc& d = *q.win;
              const int gy = d.wy0 + y, gx = d.wx0 + x;
              src_in = y < q.ih && x < q.iw && gx >= d.sx0 && gx < d.sx1 && gy >= d.sy0 && gy < d.sy1;
              if (src_in) src = (uint32_t)__ldg(d.mask + (size_t)gy * d.fw + gx) << 24;
            } else {
              src_in = y < q.ih && x < q.iw;
              if (src_in) src = (uint32_t)__ldg(q.mask + ((size_t)b * q.ih + y) * q.iw + x) << 24;
            }
          }
          if (ok) ok = mbar_wait(tfull_bar(a), (it >> 1) & 1, q.err, 15);
          ok = __all_sync(0xffffffffu, ok);  // warp-uniform: the shuffles below take every lane
          it++;
          tc_fence_after();
          // part 0: columns 0..95 (ky 0..3 = n 0..83); part 1: columns 64..159
          // (ky 4..6 = n 84..146 at v[20..82])
          float v[96];
          if (ok) {
            const uint32_t trow = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * OC_N + part * 64);
            tmem_ld32(trow, v);
            tmem_ld32(trow + 32, v + 32);
            tmem_ld32(trow + 64, v + 64);
            tmem_wait_ld();
          }
          tc_fence_before();
          if (ok) mbar_arrive(tempty_bar(a));
          if (ok) {
            // input row rr feeds output rows rr - ky (ring slot (i - ky) mod 7)
            auto tap_sums = [&](auto part_c) {
              constexpr int P1 = decltype(part_c)::value;
              constexpr int KY0 = P1 ? 4 : 0, KY1 = P1 ? 7 : 4, VOFF = P1 ? 64 : 0;
#pragma unroll
              for (int ky = KY0; ky < KY1; ky++) {
                const int yy = rr - ky;
                const bool live = yy >= 0 && yy < nout;
                float t[3];
#pragma unroll
                for (int co = 0; co < 3; co++) {
                  t[co] = v[ky * 21 + co - VOFF];
#pragma unroll
                  for (int kx = 1; kx < 7; kx++) {
                    const int n = ky * 21 + kx * 3 + co;
                    t[co] += __shfl_down_sync(0xffffffffu, v[n - VOFF], kx);
                  }
                }
                if (live) {
                  float* s = acc[(i - ky + 7) % 7];
                  s[0] += t[0];
                  s[1] += t[1];
                  s[2] += t[2];
                }
              }
            };
            if (part == 0) tap_sums(std::integral_constant<int, 0>{});
            else tap_sums(std::integral_constant<int, 1>{});
            if (part == 1 && rr >= 6) {  // hand the completed row's ky 4..6 sums to part 0
              float* s = acc[(i + 1) % 7];
              if (col) {
                float* xs = X + a * 384 + px * 3;
                xs[0] = s[0];
                xs[1] = s[1];
                xs[2] = s[2];
              }
              s[0] = s[1] = s[2] = 0.f;
            }
          }
          // X[a] written above is read below; X[a] is written again two rows
          // later, after every part-0 thread has passed the next barrier
          asm volatile("bar.sync 1, 256;" ::: "memory");
          // output row rr - 6 is complete
          if (ok && part == 0 && rr >= 6) {
            float* s = acc[(i + 1) % 7];
            if (col) {
              const int yd = rr - 6;
              const float* xs = X + a * 384 + px * 3;
              const float z[3] = {s[0] + xs[0] + bias0, s[1] + xs[1] + bias1, s[2] + xs[2] + bias2};
              if (q.win) {
                const int y = y0 + yd, x = x0 + ox;
                const WinDesc& d = *q.win;
                const int gy = d.wy0 + y, gx = d.wx0 + x;
                if (src_in && (src >> 24) != 0) {
                  uint8_t* o = d.img + ((size_t)gy * d.fw + gx) * 3;
#pragma unroll
                  for (int co = 0; co < 3; co++) {
                    const float v = fminf(fmaxf(1.0f / (1.0f + expf(-z[co])), 0.0f), 1.0f) * 255.0f;
                    o[co] = (uint8_t)(int)(v + 0.5f);
                  }
                }
              } else if (q.dst) {
                const int y = y0 + yd, x = x0 + ox;
                if (src_in && (src >> 24) != 0) {  // unmasked bytes were copied from the source
                  const size_t pix = ((size_t)b * q.ih + y) * q.iw + x;
                  uint8_t* d = q.dst + pix * 3;
                  {
#pragma unroll
                    for (int co = 0; co < 3; co++) {
                      const float v = fminf(fmaxf(1.0f / (1.0f + expf(-z[co])), 0.0f), 1.0f) * 255.0f;
                      d[co] = (uint8_t)(int)(v + 0.5f);
                    }
                  }
                }
              } else {
#pragma unroll
                for (int co = 0; co < 3; co++)
                  ob[(size_t)co * q.h * q.w + (size_t)yd * q.w] = 1.0f / (1.0f + expf(-z[co]));
              }
            }
            s[0] = s[1] = s[2] = 0.f;
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

int outconv_prepare() {
  return (int)cudaFuncSetAttribute(k_outconv_ring, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)OC_SMEM);
}

void outconv_units(OutConvParams& q, int sms) {
  q.strips = (q.w + OC_STRIP - 1) / OC_STRIP;
  // A unit of s output rows reads s + 6 input rows; an SM runs
  // ceil(units / sms) units one after another.  Pick the segment length in
  // [16, 64] with the fewest input rows per SM (ties: the longer segment).
  long long best = -1;
  for (int s = OC_SEG_MAX; s >= 16; s--) {
    const long long units = (long long)q.batch * q.strips * ((q.h + s - 1) / s);
    const long long cost = (units + sms - 1) / sms * (std::min(s, q.h) + 6);
    if (best < 0 || cost < best) {
      best = cost;
      q.seg = s;
    }
  }
  q.segs = (q.h + q.seg - 1) / q.seg;
}

int launch_outconv(const OutConvParams& q, int sms, cudaStream_t st) {
  const int units = q.batch * q.strips * q.segs;
  return launch_kernel(k_outconv_ring, dim3(units < sms ? units : sms), dim3(384), OC_SMEM, st, 1, q);
}

}  // namespace lama
