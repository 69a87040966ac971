// OutConv 7x7 64 -> 3 + bias + sigmoid (model.34 / model.35 of big-lama;
// lama-rs/src/cuda.rs:1683-1691 k_conv7x7 + lg_sigmoid, cpu.rs:540-552) with
// every input row read once.
//
// The tensor core computes, for one padded input row r and 128 input columns
// of a strip, all 147 tap products P[px][n], n = ky*21 + kx*3 + co (N = 160,
// K = the 64 input channels, three BF16 MMAs of split operands).  Output
// pixel (y, x) of channel co is the sum over (ky, kx) of P of input row
// y + ky at column x + kx: the epilogue stages P in shared memory, each
// thread (one output column) sums the seven kx products per (ky, co) and adds
// them into a ring of seven output-row accumulators in registers; output row
// r - 6 is complete after input row r and is stored (sigmoid, fp32 NCHW).
//
// Work units are (image, strip of 122 output columns = 128 input columns,
// segment of up to 64 output rows, read with 6 extra input rows; shorter
// segments when a batch has too few units for the SMs).  Warp 0 issues the
// TMA loads (one 128 x 64 box per row and part, weights once), warp 1 the
// MMAs into a double-buffered TMEM accumulator, warp 2 owns TMEM, warps 4..11
// are the epilogue: warps 4+q and 8+q drain TMEM lanes 32q.. (input columns)
// in two column halves; then thread (column, part) sums ky 0..3 (part 0) or
// 4..6 (part 1) into its ring, and part 0 adds part 1's sums when a row is
// complete.
#include <algorithm>
#include <cstdint>

#include "outconv.cuh"
#include "ptx.cuh"

namespace lama {
namespace {

constexpr int OC_N = 160;                    // 147 products, padded to a multiple of 16
constexpr int OC_NST = 3;                    // A stages
constexpr uint32_t OC_A = 128 * 64 * 2;      // one part of one input-row tile
constexpr uint32_t OC_STAGE = 2 * OC_A;      // hi + lo
constexpr uint32_t OC_WPART = OC_N * 64 * 2;  // one part of the weights
constexpr int OC_PLD = 161;                  // P row stride (floats)
constexpr uint32_t OC_P_OFF = OC_NST * OC_STAGE + 2 * OC_WPART;
constexpr uint32_t OC_X_OFF = OC_P_OFF + 128 * OC_PLD * 4;  // [128][3] partial sums of ky 4..6
constexpr uint32_t OC_BAR_OFF = OC_X_OFF + 128 * 3 * 4;
constexpr size_t OC_SMEM = 1024 + OC_BAR_OFF + 256;
constexpr int OC_STRIP = 122, OC_SEG_MAX = 64;

__global__ void __launch_bounds__(384, 1) k_outconv_ring(const __grid_constant__ OutConvParams q) {
  constexpr uint32_t IDESC = idesc_bf16_f32(OC_N);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* P = reinterpret_cast<float*>(smem + OC_P_OFF);
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
          tma_load_5d(sa, &q.amap, 0, x0, y0 + rr, b, 0, full_bar(stage));
          tma_load_5d(sa + OC_A, &q.amap, 0, x0, y0 + rr, b, 1, full_bar(stage));
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
    const int quarter = (warp - 4) & 3, half = (warp - 4) >> 2;
    const int tp = threadIdx.x - 128;
    const int px = tp & 127, part = tp >> 7;    // reduction role: input column, ky group
    const int lp = quarter * 32 + lane;         // TMEM lane = input column of the drain role
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
      const bool col = px < OC_STRIP && x0 + px < q.w;
      float* ob = q.out + (size_t)b * 3 * q.h * q.w + (size_t)y0 * q.w + x0 + px;
      float acc[7][3];
#pragma unroll
      for (int s = 0; s < 7; s++) acc[s][0] = acc[s][1] = acc[s][2] = 0.f;
      for (int base = 0; base < nin; base += 7) {
#pragma unroll
        for (int i = 0; i < 7; i++) {
          const int rr = base + i;
          if (rr >= nin) break;
          const int a = it & 1;
          if (ok) ok = mbar_wait(tfull_bar(a), (it >> 1) & 1, q.err, 15);
          it++;
          tc_fence_after();
          if (ok) {
            // drain: columns [80 * half, 80 * half + 80) of TMEM lane lp into P
            const uint32_t trow = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * OC_N + half * 80);
            float* prow = P + lp * OC_PLD + half * 80;
            float v[32];
            tmem_ld32(trow, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j++) prow[j] = v[j];
            tmem_ld32(trow + 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j++) prow[32 + j] = v[j];
            tmem_ld16(trow + 64, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j++) prow[64 + j] = v[j];
          }
          tc_fence_before();
          if (ok) mbar_arrive(tempty_bar(a));
          asm volatile("bar.sync 1, 256;" ::: "memory");
          if (ok && col) {
            // input row rr feeds output rows rr - ky (ring slot (i - ky) mod 7)
#pragma unroll
            for (int ky = 0; ky < 7; ky++) {
              if ((ky < 4) != (part == 0)) continue;
              const int yy = rr - ky;
              if (yy < 0 || yy >= nout) continue;
              float t0 = 0.f, t1 = 0.f, t2 = 0.f;
#pragma unroll
              for (int kx = 0; kx < 7; kx++) {
                const float* pp = P + (px + kx) * OC_PLD + ky * 21 + kx * 3;
                t0 += pp[0];
                t1 += pp[1];
                t2 += pp[2];
              }
              float* s = acc[(i - ky + 7) % 7];
              s[0] += t0;
              s[1] += t1;
              s[2] += t2;
            }
            if (part == 1 && rr >= 6) {  // hand the completed row's ky 4..6 sums to part 0
              float* s = acc[(i + 1) % 7];
              X[px * 3] = s[0];
              X[px * 3 + 1] = s[1];
              X[px * 3 + 2] = s[2];
              s[0] = s[1] = s[2] = 0.f;
            }
          }
          asm volatile("bar.sync 1, 256;" ::: "memory");
          // output row rr - 6 is complete
          if (ok && col && part == 0 && rr >= 6) {
            float* s = acc[(i + 1) % 7];
            const int yd = rr - 6;
            const float z[3] = {s[0] + X[px * 3] + bias0, s[1] + X[px * 3 + 1] + bias1, s[2] + X[px * 3 + 2] + bias2};
#pragma unroll
            for (int co = 0; co < 3; co++) ob[(size_t)co * q.h * q.w + (size_t)yd * q.w] = 1.0f / (1.0f + expf(-z[co]));
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
  k_outconv_ring<<<units < sms ? units : sms, 384, OC_SMEM, st>>>(q);
  return (int)cudaGetLastError();
}

}  // namespace lama
