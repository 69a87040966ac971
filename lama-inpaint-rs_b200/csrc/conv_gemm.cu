// Implicit-GEMM convolution on the sm_100a tensor core (tcgen05 + TMEM + TMA).
//
// Replaces the reference's im2col + FP32 SIMT SGEMM pair (lama-rs/cuda/lama.cu
// k_im2col :20-48 and k_sgemm_slab :363-456, launched from
// lama-rs/src/cuda.rs:973-1139) and every elementwise pass that follows a
// convolution there (k_bias_plane, k_bn_relu, k_bn_relu_add, lg_add_inplace,
// lg_sigmoid, k_reflect_pad, k_convt_put, lg_copy for Concat): those become
// the epilogue and the output addressing of this one kernel.
//
// Arithmetic: the reference is FP32.  Operands are carried as split bf16
// pairs (x = hi + lo) and each K step issues three BF16 MMAs into one FP32
// TMEM accumulator - hi*hi + hi*lo + lo*hi - which reproduces an FP32 dot
// product to ~2^-16 relative (the dropped lo*lo term and the 16-bit operand
// rounding) at the BF16 tensor-core rate.
//
// Structure: persistent CTAs (one per SM), 384 threads:
//   warp 0      TMA producer (one elected thread), STAGES-deep smem ring
//   warp 1      MMA issuer (one thread): 4 K-steps x 3 MMAs per 64-wide K block
//   warp 2      TMEM allocator
//   warps 4..11 epilogue (two warps per TMEM lane quarter, splitting the
//               columns): tcgen05.ld 32 columns at a time, fused BN/bias,
//               ReLU, residual, sigmoid, split-bf16 or fp32 store, reflect halo
// TMEM holds two BN-column accumulators so the epilogue of one tile overlaps
// the main loop of the next.
#include <algorithm>
#include <type_traits>
#include <cstdio>

#include "gemm.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace lama {

namespace {

constexpr uint32_t A_PART = 128 * 64 * 2;  // one 128 x 64 bf16 operand tile

__host__ __device__ constexpr int stages_for(int bn) {
  // (2 * A_PART + 2 * bn * 128) bytes per stage, within ~200 KB
  return bn <= 16 ? 5 : bn <= 64 ? 4 : bn <= 128 ? 3 : 2;
}
// Swapped tiles transpose through 32 x 33 fp32 staging tiles (one per
// epilogue warp).
constexpr int SHIFT_LD = 33;
// Tile widths whose split outputs can leave through TMA stores: each of the
// 8 epilogue warps stages 32 pixels x 32 channels (hi and lo, 2 KB each) at
// STAGING_OFF past the pipeline stages.
__host__ __device__ constexpr bool tma_store_bn(int bn) { return bn == 64 || bn == 128 || bn == 192; }
constexpr uint32_t STAGING_OFF = 1024;
constexpr uint32_t STAGING_WARP = 4096;
__host__ __device__ constexpr uint32_t extra_smem(int bn) {
  return bn == 256 ? 8u * 32u * SHIFT_LD * 4u : tma_store_bn(bn) ? STAGING_OFF - 256u + 8u * STAGING_WARP : 0u;
}
__host__ __device__ constexpr uint32_t stage_bytes(int bn) { return 2 * A_PART + 2u * (uint32_t)bn * 128u; }
// TMEM accumulator buffers: four for tiles up to 128 columns wide, so the
// epilogue (whose TMA stores share the TMA unit with the operand loads) may
// fall up to three tiles behind the MMAs; two for wider tiles.
__host__ __device__ constexpr int tmem_bufs_for(int bn) { return bn <= 128 ? 4 : 2; }
__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  const int c = tmem_bufs_for(bn) * bn;
  return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512;
}

struct TileInfo {
  int cls, nt, b, i0, j0;
  bool dummy;      // CTA-pair tile past the class's last M tile (loads zeros, stores nothing)
  int kb0, kb1;    // K units of this tile (K blocks, or row-union iterations; a part of the class's K with split-K)
  int part;        // split-K part of this tile
  int split_tile;  // split-K: workspace slice of part 0 of this CTA's output tile (slices part 0..ksplit-1 follow)
};

// Tile t of the launch.  With CTA pairs (p.pair) t counts pair tiles: the
// pair's two CTAs take M tiles 2m and 2m + 1 (rank) of the same N tile.
__device__ __forceinline__ TileInfo decode_tile(const GemmParams& p, int t, int rank = 0) {
  TileInfo ti;
  int c = 0;
  while (c + 1 < p.nclass && t >= p.cls[c + 1].tile0) c++;
  const GemmClass& C = p.cls[c];
  int lt = t - C.tile0;
  ti.cls = c;
  const int part = C.part0 + lt % C.nparts;  // split-K parts of one output tile are consecutive tiles
  lt /= C.nparts;
  ti.kb0 = C.kcut[part];
  ti.kb1 = C.kcut[part + 1];
  ti.part = part;
  ti.nt = lt % C.ntiles_n;
  int mt = lt / C.ntiles_n;
  if (p.pair) mt = 2 * mt + rank;
  ti.split_tile = C.ws_tile0 + (mt * C.ntiles_n + ti.nt) * C.ksplit;
  ti.dummy = mt >= p.m_tiles;
  int per_img = p.tiles_y * p.tiles_x;
  ti.b = mt / per_img;
  int r = mt - ti.b * per_img;
  ti.i0 = (r / p.tiles_x) * p.bh;
  ti.j0 = (r % p.tiles_x) * p.bw;
  return ti;
}

// The k-th tile of a CTA (pair) slot: from the launch's static schedule when
// it has one (p.sched: the host's longest-first assignment of tiles of
// unequal K), else round robin over the slots.  -1 past the slot's last tile.
__device__ __forceinline__ int tile_of(const GemmParams& p, int slot, int k, int nslots) {
  if (p.sched) {
    const int a = __ldg(p.sched_off + slot) + k;
    return a < __ldg(p.sched_off + slot + 1) ? __ldg(p.sched + a) : -1;
  }
  const int t = slot + k * nslots;
  return t < p.total_tiles ? t : -1;
}

__device__ __forceinline__ int reflect_idx(int i, int n) {
  if (n == 1) return 0;
  int period = 2 * (n - 1);
  int m = i % period;
  if (m < 0) m += period;
  return m >= n ? period - m : m;
}

// Padded positions whose value is interior coordinate q: q itself plus any
// halo cells that reflect onto it.  Returns the count (<= 1 + 2*halo).
__device__ __forceinline__ int halo_targets(int q, int n, int halo, int reflect, int* out) {
  int cnt = 0;
  out[cnt++] = q + halo;
  // only interior positions within `halo` of an edge are reflected into the halo
  if (reflect && halo > 0 && (q <= halo || q >= n - 1 - halo)) {
    for (int p = 0; p < halo; p++)
      if (reflect_idx(p - halo, n) == q) out[cnt++] = p;
    for (int p = n + halo; p < n + 2 * halo; p++)
      if (reflect_idx(p - halo, n) == q) out[cnt++] = p;
  }
  return cnt;
}

template <int CH>
__device__ __forceinline__ void store_split(const GemmParams& p, int b, int oy, int ox, int n, const float* v) {
  int ty[7], tx[7];
  int ny = halo_targets(oy, p.out_h, p.out_halo, p.out_reflect, ty);
  int nx = halo_targets(ox, p.out_w, p.out_halo, p.out_reflect, tx);
  uint32_t hi[CH / 2], lo[CH / 2];
#pragma unroll
  for (int k = 0; k < CH / 2; k++) split_pair(v[2 * k], v[2 * k + 1], hi[k], lo[k]);
  const int hp = p.out_h + 2 * p.out_halo, wp = p.out_w + 2 * p.out_halo;
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(p.out);
  for (int a = 0; a < ny; a++)
    for (int c = 0; c < nx; c++) {
      long long off = (((long long)b * hp + ty[a]) * wp + tx[c]) * p.out_c + n;
      uint4* dh = reinterpret_cast<uint4*>(base + off);
      uint4* dl = reinterpret_cast<uint4*>(base + p.out_part + off);
#pragma unroll
      for (int k = 0; k < CH / 8; k++) {
        dh[k] = make_uint4(hi[4 * k], hi[4 * k + 1], hi[4 * k + 2], hi[4 * k + 3]);
        dl[k] = make_uint4(lo[4 * k], lo[4 * k + 1], lo[4 * k + 2], lo[4 * k + 3]);
      }
    }
}

// Residual and sigmoid of CH channels starting at absolute channel n of one
// output pixel.
template <int CH>
__device__ __forceinline__ void finish_channels(const GemmParams& p, int b, int oy, int ox, int n, float* v) {
  if (p.skip) {
    const int hp = p.out_h + 2 * p.out_halo, wp = p.out_w + 2 * p.out_halo;
    long long off = (((long long)b * hp + oy + p.out_halo) * wp + ox + p.out_halo) * p.out_c + n;
    const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(p.skip);
    const uint4* sh = reinterpret_cast<const uint4*>(sb + off);
    const uint4* sl = reinterpret_cast<const uint4*>(sb + p.out_part + off);
#pragma unroll
    for (int k = 0; k < CH / 8; k++) {
      uint4 h = sh[k], l = sl[k];
      float2 f0 = join_pair(h.x, l.x), f1 = join_pair(h.y, l.y), f2 = join_pair(h.z, l.z), f3 = join_pair(h.w, l.w);
      v[8 * k + 0] += f0.x; v[8 * k + 1] += f0.y;
      v[8 * k + 2] += f1.x; v[8 * k + 3] += f1.y;
      v[8 * k + 4] += f2.x; v[8 * k + 5] += f2.y;
      v[8 * k + 6] += f3.x; v[8 * k + 7] += f3.y;
    }
  }
  if (p.sigmoid) {
#pragma unroll
    for (int k = 0; k < CH; k++) {
      float e = expf(-v[k]);
      v[k] = 1.0f / (1.0f + e);
    }
  }
}

// Residual, sigmoid and the store of CH channels [C.n0, C.n0 + CH) of one
// output pixel whose values already carry the per-channel affine and ReLU.
template <int CH>
__device__ __forceinline__ void store_channels(const GemmParams& p, const GemmClass& C, int b, int oy, int ox,
                                               float* v, int nloc = 0) {
  const int n = C.n0 + nloc;
  finish_channels<CH>(p, b, oy, ox, n, v);
  if (p.out_kind == OUT_SPLIT) {
    store_split<CH>(p, b, oy, ox, n, v);
  } else if (p.out_kind == OUT_F32_NHWC) {
    const int hp = p.out_h + 2 * p.out_halo, wp = p.out_w + 2 * p.out_halo;
    long long off = (((long long)b * hp + oy + p.out_halo) * wp + ox + p.out_halo) * p.out_c + n;
    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + off);
#pragma unroll
    for (int k = 0; k < CH / 4; k++) d[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  } else {
    float* o = reinterpret_cast<float*>(p.out);
#pragma unroll
    for (int k = 0; k < CH; k++)
      if (nloc + k < C.nvalid)
        o[(((long long)b * p.out_c + n + k) * p.out_h + oy) * p.out_w + ox] = v[k];
  }
}

// The reflected halo copies of one output pixel (every target but the
// interior one), split bf16.
__device__ __forceinline__ void store_split_halo(const GemmParams& p, int b, int oy, int ox, int n,
                                                 const uint32_t* hi, const uint32_t* lo) {
  int ty[7], tx[7];
  const int ny = halo_targets(oy, p.out_h, p.out_halo, p.out_reflect, ty);
  const int nx = halo_targets(ox, p.out_w, p.out_halo, p.out_reflect, tx);
  if (ny == 1 && nx == 1) return;
  const int hp = p.out_h + 2 * p.out_halo, wp = p.out_w + 2 * p.out_halo;
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(p.out);
  for (int a = 0; a < ny; a++)
    for (int c = 0; c < nx; c++) {
      if (a == 0 && c == 0) continue;
      long long off = (((long long)b * hp + ty[a]) * wp + tx[c]) * p.out_c + n;
      uint4* dh = reinterpret_cast<uint4*>(base + off);
      uint4* dl = reinterpret_cast<uint4*>(base + p.out_part + off);
#pragma unroll
      for (int k = 0; k < 4; k++) {
        dh[k] = make_uint4(hi[4 * k], hi[4 * k + 1], hi[4 * k + 2], hi[4 * k + 3]);
        dl[k] = make_uint4(lo[4 * k], lo[4 * k + 1], lo[4 * k + 2], lo[4 * k + 3]);
      }
    }
}

// fp32 store of one warp's 32 pixels x 32 channels through the TMA unit
// (ostore 2: NCHW, the staging tile is [channel][pixel]; ostore 3: NHWC,
// [pixel][channel] with the 128-byte swizzle).
__device__ __forceinline__ void store_f32_tma(const GemmParams& p, const void* omap, uint8_t* stage, int lane, int b,
                                              int n, int box_x, int box_y, const float* v) {
  if (lane == 0) bulk_wait_read0();
  __syncwarp();
  if (p.ostore == 2) {
    float* st = reinterpret_cast<float*>(stage);
#pragma unroll
    for (int k = 0; k < 32; k++) st[k * 32 + lane] = v[k];
  } else {
    uint4* st = reinterpret_cast<uint4*>(stage + lane * 128);
#pragma unroll
    for (int k = 0; k < 8; k++) st[k ^ (lane & 7)] = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                                                 __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (p.ostore == 2) tma_store_4d(omap, smem_u32(stage), box_x, box_y, n, b);
    else tma_store_4d(omap, smem_u32(stage), n, box_x, box_y, b);
    bulk_commit();
  }
}

// Split store of one warp's 32 pixels x 32 channels through the TMA unit: the
// lane's pixel row goes to the warp's staging tile (64-byte swizzle, the
// layout omap's box expects), one lane issues the hi and lo box stores, and
// border lanes add their reflected halo copies with ordinary stores.  The
// previous chunk's stores must have read the staging tile first.
__device__ __forceinline__ void store_split_tma(const GemmParams& p, const void* omap, uint8_t* stage, int lane,
                                                bool valid, int b, int oy, int ox, int n, int box_x, int box_y,
                                                const float* v) {
  uint32_t hi[16], lo[16];
#pragma unroll
  for (int k = 0; k < 16; k++) split_pair(v[2 * k], v[2 * k + 1], hi[k], lo[k]);
  if (lane == 0) bulk_wait_read0();
  __syncwarp();
  const int sw = (lane >> 1) & 3;
  uint4* sh = reinterpret_cast<uint4*>(stage + lane * 64);
  uint4* sl = reinterpret_cast<uint4*>(stage + 2048 + lane * 64);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    sh[k ^ sw] = make_uint4(hi[4 * k], hi[4 * k + 1], hi[4 * k + 2], hi[4 * k + 3]);
    sl[k ^ sw] = make_uint4(lo[4 * k], lo[4 * k + 1], lo[4 * k + 2], lo[4 * k + 3]);
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_5d(omap, smem_u32(stage), n, box_x, box_y, b, 0);
    tma_store_5d(omap, smem_u32(stage + 2048), n, box_x, box_y, b, 1);
    bulk_commit();
  }
  if (valid && p.out_halo && p.out_reflect) store_split_halo(p, b, oy, ox, n, hi, lo);
}

// Per-channel affine (folded BN / bias) and ReLU of CH channels starting at
// class-relative channel nloc.  Whole chunks inside the class read the scale
// and shift with 16-byte loads where both are 16-byte aligned (every lane
// reads the same address, so each load is one broadcast).
template <int CH>
__device__ __forceinline__ void affine_relu(const GemmParams& p, const GemmClass& C, int nloc, float* v) {
  const int n = C.n0 + nloc;
  if (CH % 4 == 0 && nloc + CH <= C.nvalid &&
      ((reinterpret_cast<uintptr_t>(p.scale + n) | reinterpret_cast<uintptr_t>(p.shift + n)) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(p.scale + n);
    const float4* t4 = reinterpret_cast<const float4*>(p.shift + n);
#pragma unroll
    for (int q = 0; q < CH / 4; q++) {
      const float4 s = __ldg(s4 + q), t = __ldg(t4 + q);
      const float sv[4] = {s.x, s.y, s.z, s.w}, tv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        float x = v[4 * q + e] * sv[e];
        x = x + tv[e];
        if (p.relu) x = x > 0.f ? x : 0.f;
        v[4 * q + e] = x;
      }
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < CH; k++) {
    int nn = n + k;
    float s = 1.f, t = 0.f;
    if (nloc + k < C.nvalid) {
      s = __ldg(p.scale + nn);
      t = __ldg(p.shift + nn);
    }
    float x = v[k] * s;
    x = x + t;
    if (p.relu) x = x > 0.f ? x : 0.f;
    v[k] = x;
  }
}

template <int CH>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, const GemmClass& C, int b, int oy, int ox,
                                               int nloc, float* v) {
  affine_relu<CH>(p, C, nloc, v);
  store_channels<CH>(p, C, b, oy, ox, v, nloc);
}

// Swapped-tile epilogue: TMEM lane m holds output channel n0 + nt*128 + m for
// the tile's BN pixels.  Each warp owns 32 channels; per 32-pixel chunk it
// applies the per-channel affine + ReLU, transposes the 32 x 32 block through
// its own shared-memory tile, and then every lane owns one pixel and stores the
// warp's 32 channels as 16-byte vectors (with residual, split and halo), the
// same store path as the pixel-major epilogue.
template <int BN>
__device__ __forceinline__ void epilogue_swapped(const GemmParams& p, const GemmClass& C, const TileInfo& ti, int m,
                                                 uint32_t trow, float* tbuf, int half) {
  const int lane = m & 31;
  const int wch = ti.nt * 128 + (m & ~31);  // class-relative first channel of this warp
  const int nloc = wch + lane;
  const bool chv = nloc < C.nvalid;
  const int n = C.n0 + nloc;
  const float sc = chv ? __ldg(p.scale + n) : 0.f;
  const float sh = chv ? __ldg(p.shift + n) : 0.f;
#pragma unroll 1
  for (int ch = half; ch < BN / 32; ch += 2) {
    float v[32];
    tmem_ld32(trow + ch * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int q = 0; q < 32; q++) {
      float x = v[q] * sc;
      x = x + sh;
      if (p.relu) x = x > 0.f ? x : 0.f;
      tbuf[q * SHIFT_LD + lane] = x;  // [pixel][channel]
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 32; k++) v[k] = tbuf[lane * SHIFT_LD + k];
    __syncwarp();
    const int pix = ch * 32 + lane;
    const int i = ti.i0 + pix / p.bw, j = ti.j0 + pix % p.bw;
    if (i < p.mh && j < p.mw && wch < C.nvalid) {
      const int oy = i * C.oy_mul + C.oy_add, ox = j * C.ox_mul + C.ox_add;
      GemmClass Cn = C;  // affine already applied: run the store path with identity scale/shift
      Cn.n0 = C.n0 + wch;
      store_channels<32>(p, Cn, ti.b, oy, ox, v);
    }
  }
}

// SWAP = false: M = 128 pixels (A = activations), N = BN output channels (B = weights).
// SWAP = true:  M = 128 output channels (A = weights), N = BN pixels (B = activations);
//               more MACs per staged byte when the output has >= 128 channels
//               (BN = 256: 65 MAC/B instead of 48 at BN = 128).  The epilogue then
//               holds one output channel per thread and walks the tile's pixels.
//
// PAIR: a cluster of two CTAs computes 256 x BN tiles with cta_group::2 MMAs.
// Each CTA stages its own 128 A rows and BN/2 B rows (so a stage carries a
// quarter less than a single-CTA 128 x BN stage for the same MMA work, and the
// pipeline gets one more stage); the even CTA's barriers count both CTAs' TMA
// bytes and both epilogues' releases, its MMA warp issues for the pair, and
// commits arrive on both CTAs' barriers.  Each CTA's epilogue drains its own
// TMEM (its 128 pixels).
template <int BN, bool SWAP, bool PAIR = false>
__global__ void __launch_bounds__(384, 1) k_conv_gemm(const __grid_constant__ GemmParams p) {
  constexpr int BROWS = PAIR ? BN / 2 : BN;  // B rows staged by this CTA
  constexpr int STAGES = stages_for(BROWS);
  constexpr uint32_t B_PART = (uint32_t)BROWS * 128u;
  constexpr uint32_t STAGE = stage_bytes(BROWS);
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr int NACC = tmem_bufs_for(BN);
  constexpr int CH = BN < 32 ? BN : 32;
  constexpr uint32_t IDESC = idesc_bf16_f32(BN, PAIR ? 256 : 128);
  static_assert(!(PAIR && SWAP), "CTA pairs use pixel-major tiles");
  static_assert((2 * STAGES + 2 * NACC) * 8 + 12 <= 256, "barriers and TMEM slot fit the 256-byte block");

  extern __shared__ uint8_t smem_raw[];
  pdl_launch_dependents();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * NACC);
  // split-K verdict of the current tile (2 * tile sequence + last) and the
  // count of epilogue warps that have added their partial sums
  volatile int* split_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* split_cnt = reinterpret_cast<int*>(tmem_slot + 2);
  float* shift_buf = reinterpret_cast<float*>(smem + STAGES * STAGE + 256);
  const uint32_t smem0 = smem_u32(smem);
  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + NACC + a); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = PAIR ? (int)cluster_ctarank() : 0;
  const int slot = PAIR ? blockIdx.x / 2 : blockIdx.x;  // this CTA's (pair's) slot in the launch's schedule
  const int tstep = PAIR ? gridDim.x / 2 : gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    *split_flag = -2;
    *split_cnt = 0;
    for (int a = 0; a < NACC; a++) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), PAIR ? 16 : 256);  // pairs: one release per epilogue warp of both CTAs
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < p.nclass; i++) tma_prefetch(&p.bmap[i]);
    if (p.ostore)
      for (int i = 0; i < p.nclass; i++) tma_prefetch(&p.omap[i]);
    for (int i = 0; i < GEMM_MAX_AMAPS; i++) tma_prefetch(&p.amap[i]);
  }
  if (warp == 2) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // set-up done: from here on the previous kernel's outputs are read (and
  // buffers it reads are written), so wait for it to complete
  pdl_wait();
  // epilogue release of an accumulator buffer (pairs: on the even CTA's barrier)
  auto release = [&](int a) {
    tc_fence_before();
    if constexpr (PAIR) {
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(tempty_bar(a), 0));
    } else {
      mbar_arrive(tempty_bar(a));
    }
  };

  // Row-union stages: two normal stages each, A box (up to 6 rows x 32 pixels
  // of 64 channels, or 7 rows of 32 channels; both parts) at 0, the group's
  // weight K blocks (both parts each) from U_A.  With 32-channel boxes a K
  // block holds two taps (tap parity = which half of its 128-byte row).
  constexpr uint32_t U_A = 6u * 32u * 128u * 2u;
  constexpr int USTAGES = STAGES / 2;
  static_assert(SWAP || BROWS != 64 || (STAGES % 2 == 0 && U_A + 3u * 2u * B_PART <= 2u * STAGE),
                "row-union stages fit two normal stages");

  if (warp == 0 && p.uni) {
    // ---------------------------------------------------------- producer (row union)
    if constexpr (!SWAP && BROWS == 64) {
      if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int k = 0, t; ok && (t = tile_of(p, slot, k, tstep)) >= 0; k++) {
          const TileInfo ti = decode_tile(p, t, rank);
          const GemmClass& C = p.cls[ti.cls];
          const int wrow = ti.nt * BN + rank * BROWS;
          int u = 0;  // union iteration (group, block) in class order; this part runs [kb0, kb1)
          for (int g = 0; g < C.ngroup && ok && u < ti.kb1; g++) {
            const GemmGroup& G = C.grp[g];
            const GemmSeg& S = C.seg[G.seg];
            const int tsh = p.cb == 32 ? 1 : 0;                          // log2(taps per K block)
            const uint32_t bytes = (uint32_t)p.urows[S.amap] * (uint32_t)p.bw * (uint32_t)p.cb * 4u +
                                   (uint32_t)(G.ndy >> tsh) * 2u * B_PART;
            for (int blk = 0; blk < S.nblk && u < ti.kb1; blk++, u++) {
              if (u < ti.kb0) continue;
              if (!mbar_wait(empty_bar(stage), phase ^ 1, p.err, 1)) { ok = false; break; }
              const uint32_t fb = PAIR ? mapa_shared(full_bar(stage), 0) : full_bar(stage);
              if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), PAIR ? 2 * bytes : bytes);
              const uint32_t sa = smem0 + (uint32_t)stage * 2u * STAGE;
              const int cx = S.c0 + blk * p.cb, x = ti.j0 + G.dx, y = ti.i0 + G.dy0;
              if constexpr (PAIR) tma_load_5d_pair(sa, &p.amap_u[S.amap], cx, x, y, ti.b, 0, fb);
              else tma_load_5d(sa, &p.amap_u[S.amap], cx, x, y, ti.b, 0, fb);
              for (int j = 0; j < (G.ndy >> tsh); j++) {
                const int kb = (S.sub0 + G.tap[j << tsh] * S.nblk + blk) >> tsh;
                const uint32_t dst = sa + U_A + (uint32_t)j * 2u * B_PART;
                if constexpr (PAIR) tma_load_3d_pair(dst, &p.bmap[ti.cls], kb * 64, wrow, 0, fb);
                else tma_load_3d(dst, &p.bmap[ti.cls], kb * 64, wrow, 0, fb);
              }
              if (++stage == USTAGES) { stage = 0; phase ^= 1; }
            }
          }
        }
      }
    }
  } else if (warp == 1 && p.uni) {
    // ---------------------------------------------------------- MMA issuer (row union)
    if constexpr (!SWAP && BROWS == 64) {
      if (lane == 0 && rank == 0) {
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        bool ok = true;
        for (int t; ok && (t = tile_of(p, slot, it, tstep)) >= 0; it++) {
          const TileInfo ti = decode_tile(p, t, rank);
          const GemmClass& C = p.cls[ti.cls];
          const int acc = it % NACC;
          if (!mbar_wait(tempty_bar(acc), ((it / NACC) & 1) ^ 1, p.err, 2)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          uint32_t accum = 0;
          int u = 0;  // as in the producer
          for (int g = 0; g < C.ngroup && ok && u < ti.kb1; g++) {
            const GemmGroup& G = C.grp[g];
            const GemmSeg& S = C.seg[G.seg];
            const bool sw64 = p.cb == 32;
            const uint32_t rowb = (uint32_t)p.bw * (uint32_t)p.cb * 2u;     // one pixel row of the box
            const uint32_t apart = (uint32_t)p.urows[S.amap] * rowb;        // hi part of the box
            for (int blk = 0; blk < S.nblk && u < ti.kb1; blk++, u++) {
              if (u < ti.kb0) continue;
              if (!mbar_wait(full_bar(stage), phase, p.err, 3)) { ok = false; break; }
              tc_fence_after();
              const uint32_t sa = smem0 + (uint32_t)stage * 2u * STAGE;
              // the K steps of one tap: 64-channel rows (128-byte swizzle) or
              // 32-channel rows (64-byte swizzle), unrolled per case
              auto tap_mmas = [&](auto kst, auto ndy) {
                constexpr int KS = decltype(kst)::value, NDY = decltype(ndy)::value;
                constexpr uint32_t SBO = KS == 4 ? 1024u : 512u, LAYOUT = KS == 4 ? 2u : 4u;
                constexpr int TPK = KS == 4 ? 1 : 2;  // taps per K block
                // descriptors of the stage's first A row and first B block; the
                // others differ only in the start-address field (bytes / 16,
                // shared-memory addresses stay below 2^18 so it never carries)
                const uint64_t a0 = smem_desc(sa, SBO, LAYOUT), b0 = smem_desc(sa + U_A, 1024u, 2u);
                const uint64_t dap = apart >> 4;
#pragma unroll
                for (int j = 0; j < NDY; j++) {
                  const uint64_t aj = a0 + (((uint32_t)j * rowb) >> 4);
                  const uint64_t bj = b0 + (((uint32_t)(j / TPK) * 2u * B_PART + (uint32_t)(j % TPK) * 64u) >> 4);
#pragma unroll
                  for (int k = 0; k < KS; k++) {
                    const uint64_t a_hi = aj + 2u * k;
                    const uint64_t a_lo = a_hi + dap;
                    const uint64_t b_hi = bj + 2u * k;
                    const uint64_t b_lo = b_hi + (B_PART >> 4);
                    if constexpr (PAIR) {
                      mma_bf16_pair(d_tmem, a_lo, b_hi, IDESC, accum);
                      mma_bf16_pair(d_tmem, a_hi, b_lo, IDESC, 1u);
                      mma_bf16_pair(d_tmem, a_hi, b_hi, IDESC, 1u);
                    } else {
                      mma_bf16(d_tmem, a_lo, b_hi, IDESC, accum);
                      mma_bf16(d_tmem, a_hi, b_lo, IDESC, 1u);
                      mma_bf16(d_tmem, a_hi, b_hi, IDESC, 1u);
                    }
                    accum = 1u;
                  }
                }
              };
              // the group's taps as a compile-time count (whole loops unrolled)
              auto by_ndy = [&](auto kst) {
                switch (G.ndy) {
                  case 1: tap_mmas(kst, std::integral_constant<int, 1>{}); break;
                  case 2: tap_mmas(kst, std::integral_constant<int, 2>{}); break;
                  case 3: tap_mmas(kst, std::integral_constant<int, 3>{}); break;
                  default: tap_mmas(kst, std::integral_constant<int, 4>{}); break;
                }
              };
              if (sw64) by_ndy(std::integral_constant<int, 2>{});
              else by_ndy(std::integral_constant<int, 4>{});
              if constexpr (PAIR) mma_commit_pair(empty_bar(stage), 3);
              else mma_commit(empty_bar(stage));
              if (++stage == USTAGES) { stage = 0; phase ^= 1; }
            }
          }
          if (ok) {
            if constexpr (PAIR) mma_commit_pair(tfull_bar(acc), 3);
            else mma_commit(tfull_bar(acc));
          }
        }
      }
    }
  } else if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const int subs_per_kb = 64 / p.cb;
      const uint32_t sub_bytes = (uint32_t)p.cb * (SWAP ? BN : 128u) * 2u;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int k = 0, t; ok && (t = tile_of(p, slot, k, tstep)) >= 0; k++) {
        const TileInfo ti = decode_tile(p, t, rank);
        const GemmClass& C = p.cls[ti.cls];
        int seg = 0;
        for (int kb = ti.kb0; kb < ti.kb1; kb++) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, p.err, 1)) { ok = false; break; }
          const uint32_t fb = PAIR ? mapa_shared(full_bar(stage), 0) : full_bar(stage);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), PAIR ? 2 * STAGE : STAGE);
          const uint32_t sa = smem0 + (uint32_t)stage * STAGE;
          // activation sub-boxes: the A operand, or the B operand when swapped
          const uint32_t act = SWAP ? sa + 2 * A_PART : sa;
          for (int u = 0; u < subs_per_kb; u++) {
            const int sub = kb * subs_per_kb + u;
            while (seg + 1 < C.nseg && sub >= C.seg[seg + 1].sub0) seg++;
            const GemmSeg& S = C.seg[seg];
            const int r = sub - S.sub0;
            const int tap = r / S.nblk, blk = r - tap * S.nblk;
            const int cx = S.c0 + blk * p.cb;
            const int x = ti.j0 * S.stride + S.dx[tap];
            const int y = ti.i0 * S.stride + S.dy[tap];
            // one copy brings the hi and the lo sub-box (the map's boxes span both parts)
            if constexpr (PAIR) tma_load_5d_pair(act + u * 2 * sub_bytes, &p.amap[S.amap], cx, x, y, ti.b, 0, fb);
            else tma_load_5d(act + u * 2 * sub_bytes, &p.amap[S.amap], cx, x, y, ti.b, 0, fb);
          }
          // weights: the B operand (BN rows), or the A operand (128 rows) when swapped
          const uint32_t wdst = SWAP ? sa : sa + 2 * A_PART;
          const int wrow = SWAP ? ti.nt * 128 : ti.nt * BN + rank * BROWS;
          if constexpr (PAIR) tma_load_3d_pair(wdst, &p.bmap[ti.cls], kb * 64, wrow, 0, fb);
          else tma_load_3d(wdst, &p.bmap[ti.cls], kb * 64, wrow, 0, fb);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      const bool sw64 = !SWAP && (p.cb == 32);  // swapped A is the 128B-swizzled weight tile
      const uint32_t a_sbo = sw64 ? 512u : 1024u;
      const uint32_t a_layout = sw64 ? 4u : 2u;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t; ok && (t = tile_of(p, slot, it, tstep)) >= 0; it++) {
        const TileInfo ti = decode_tile(p, t, rank);
        const int acc = it % NACC;
        if (!mbar_wait(tempty_bar(acc), ((it / NACC) & 1) ^ 1, p.err, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = ti.kb0; kb < ti.kb1; kb++) {
          if (!mbar_wait(full_bar(stage), phase, p.err, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem0 + (uint32_t)stage * STAGE;
          const uint32_t sb = sa + 2 * A_PART;
          // as in the row-union loop: only the start-address fields differ
          const uint64_t a0 = smem_desc(sa, a_sbo, a_layout), b0 = smem_desc(sb, 1024u, 2u);
          const uint64_t dal = (sw64 ? 8192u : A_PART) >> 4;
#pragma unroll
          for (int k = 0; k < 4; k++) {
            // 64-byte swizzle (32-channel sub-boxes): [sub][part][128 px][32 ch];
            // 128-byte swizzle: [part][128 px][64 ch]
            const uint32_t aoff = sw64 ? (uint32_t)((k >> 1) * 16384 + (k & 1) * 32) : (uint32_t)(k * 32);
            const uint64_t a_hi = a0 + (aoff >> 4);
            const uint64_t a_lo = a_hi + dal;
            const uint64_t b_hi = b0 + 2u * k;
            const uint64_t b_lo = b_hi + (B_PART >> 4);
            if constexpr (PAIR) {
              mma_bf16_pair(d_tmem, a_lo, b_hi, IDESC, (kb != ti.kb0 || k != 0) ? 1u : 0u);
              mma_bf16_pair(d_tmem, a_hi, b_lo, IDESC, 1u);
              mma_bf16_pair(d_tmem, a_hi, b_hi, IDESC, 1u);
            } else {
              mma_bf16(d_tmem, a_lo, b_hi, IDESC, (kb != ti.kb0 || k != 0) ? 1u : 0u);
              mma_bf16(d_tmem, a_hi, b_lo, IDESC, 1u);
              mma_bf16(d_tmem, a_hi, b_hi, IDESC, 1u);
            }
          }
          if constexpr (PAIR) mma_commit_pair(empty_bar(stage), 3);
          else mma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (ok) {
          if constexpr (PAIR) mma_commit_pair(tfull_bar(acc), 3);
          else mma_commit(tfull_bar(acc));
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------- epilogue
    // 8 warps: warp 4+q and 8+q share TMEM lanes 32q..32q+31 and split the columns
    const int ew = warp - 4;
    const int quarter = ew & 3, half = ew >> 2;
    const int m = quarter * 32 + lane;
    int it = 0;
    for (int t; (t = tile_of(p, slot, it, tstep)) >= 0; it++) {
      const TileInfo ti = decode_tile(p, t, rank);
      const GemmClass& C = p.cls[ti.cls];
      const int acc = it % NACC;
      if constexpr (!SWAP) {
        // While the MMAs run: the scale / shift lines of this warp's chunks
        // into L1 and the residual of its pixel into L2.
        const int pi = ti.i0 + m / p.bw, pj = ti.j0 + m % p.bw;
        const bool pv = pi < p.mh && pj < p.mw && !ti.dummy;
        const int hp = p.out_h + 2 * p.out_halo, wp = p.out_w + 2 * p.out_halo;
        const long long poff =
            (((long long)ti.b * hp + pi * C.oy_mul + C.oy_add + p.out_halo) * wp + pj * C.ox_mul + C.ox_add +
             p.out_halo) * p.out_c + C.n0;
        for (int ch = half; ch < BN / 32; ch += 2) {
          const int nloc = ti.nt * BN + ch * 32;
          if (nloc >= C.nvalid) break;
          if (lane == 0) prefetch_l1(p.scale + C.n0 + nloc);
          if (lane == 1) prefetch_l1(p.shift + C.n0 + nloc);
          if (p.skip && pv) {
            const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(p.skip) + poff + nloc;
            prefetch_l2(sb);
            prefetch_l2(sb + p.out_part);
          }
        }
      }
      if (!mbar_wait(tfull_bar(acc), (it / NACC) & 1, p.err, 4)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (SWAP) {
        epilogue_swapped<BN>(p, C, ti, m, trow, shift_buf + ew * 32 * SHIFT_LD, half);
        release(acc);
        continue;
      }
      const int i = ti.i0 + m / p.bw, j = ti.j0 + m % p.bw;
      const bool valid = (i < p.mh) && (j < p.mw) && !ti.dummy;
      const int oy = i * C.oy_mul + C.oy_add, ox = j * C.ox_mul + C.ox_add;
      // split-K: every part stores its raw sums in its own workspace slice; the
      // CTA whose part arrives last finishes the tile from the sum of the
      // slices in part order (deterministic), the others are done
      const bool split = (CH == 32 && !SWAP) && C.ksplit > 1;
      const float* wsp = nullptr;
      if constexpr (CH == 32 && !SWAP) {
        if (split) {
          wsp = p.ws + (size_t)ti.split_tile * (BN * 128) + m;  // slice [n][m] of part 0
          float* mine = p.ws + (size_t)(ti.split_tile + ti.part) * (BN * 128) + m;
#pragma unroll 1
          for (int ch = half; ch < BN / 32; ch += 2) {
            float v[32];
            tmem_ld32(trow + ch * 32, v);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; k++) __stcg(mine + (ch * 32 + k) * 128, v[k]);
          }
          release(acc);
          __threadfence();
          __syncwarp();
          // the eighth epilogue warp to get here counts this CTA's part in and
          // publishes (tile sequence, last?) for the others, which wait for it
          // with a bounded spin
          int last = 0;
          if (lane == 0) {
            if (atomicAdd(split_cnt, 1) == 7) {
              *split_cnt = 0;
              // the other seven warps' slices (each fenced before its count)
              // are ordered before this part's arrival at the tile counter
              __threadfence();
              last = atomicAdd(p.cnt + ti.split_tile, 1) == C.ksplit - 1;
              if (last) p.cnt[ti.split_tile] = 0;
              __threadfence_block();
              *split_flag = 2 * it + last;
            } else {
              const long long t0 = clock64();
              int f;
              while (((f = *split_flag) >> 1) != it) {
                if (clock64() - t0 > LAMA_WAIT_CYCLES) {
                  atomicCAS(p.err, 0, 5);
                  f = 2 * it;
                  break;
                }
              }
              last = f & 1;
            }
          }
          last = __shfl_sync(0xffffffffu, last, 0);
          if (!last) continue;
          __threadfence();
        }
      }
      // the 32 values of chunk ch: from TMEM, or (split-K fix-up) from the workspace
      auto chunk32 = [&](int ch, float* v) {
        if (split) {
#pragma unroll
          for (int k = 0; k < 32; k++) v[k] = __ldcg(wsp + (ch * 32 + k) * 128);
          // two slices' loads in flight at a time; the sum stays in part order
#pragma unroll 1
          for (int q = 1; q < C.ksplit; q += 2) {
            const float* sa = wsp + (size_t)q * (BN * 128) + ch * 32 * 128;
            const float* sb = sa + (BN * 128);
            const bool two = q + 1 < C.ksplit;
            float a[32], b[32];
#pragma unroll
            for (int k = 0; k < 32; k++) a[k] = __ldcg(sa + k * 128);
#pragma unroll
            for (int k = 0; k < 32; k++) b[k] = two ? __ldcg(sb + k * 128) : 0.f;
#pragma unroll
            for (int k = 0; k < 32; k++) v[k] += a[k];
            if (two) {
#pragma unroll
              for (int k = 0; k < 32; k++) v[k] += b[k];
            }
          }
        } else {
          tmem_ld32(trow + ch * 32, v);
          tmem_wait_ld();
        }
      };
      if constexpr (tma_store_bn(BN)) {
        if (p.ostore) {
          // box origin: the warp's first pixel (32 consecutive M rows)
          const int m0 = quarter * 32;
          const int box_x = ti.j0 + m0 % p.bw, box_y = ti.i0 + m0 / p.bw;  // M-space (class grid)
          const void* omap = &p.omap[ti.cls];
          uint8_t* stage = smem + STAGES * STAGE + STAGING_OFF + ew * STAGING_WARP;
#pragma unroll 1
          for (int ch = half; ch < BN / 32; ch += 2) {
            float v[32];
            chunk32(ch, v);
            const int nloc = ti.nt * BN + ch * 32;
            if (nloc >= C.nvalid) continue;
            affine_relu<32>(p, C, nloc, v);
            if (valid) finish_channels<32>(p, ti.b, oy, ox, C.n0 + nloc, v);
            if (p.ostore == 1) store_split_tma(p, omap, stage, lane, valid, ti.b, oy, ox, C.n0 + nloc, box_x, box_y, v);
            else store_f32_tma(p, omap, stage, lane, ti.b, C.n0 + nloc, box_x, box_y, v);
          }
          if (!split) release(acc);
          continue;
        }
      }
#pragma unroll 1
      for (int ch = half; ch < BN / CH; ch += 2) {
        float v[CH];
        if constexpr (CH == 32) {
          chunk32(ch, v);
        } else {
          tmem_ld16(trow + ch * CH, v);
          tmem_wait_ld();
        }
        const int nloc = ti.nt * BN + ch * CH;
        if (valid && nloc < C.nvalid) epilogue_chunk<CH>(p, C, ti.b, oy, ox, nloc, v);
      }
      if (!split) release(acc);
    }
    if constexpr (tma_store_bn(BN)) {
      if (p.ostore && lane == 0) bulk_wait0();
    }
  }

  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's remote arrives and MMAs are done
  if (warp == 2) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int BN, bool SWAP = false, bool PAIR = false>
constexpr size_t smem_for() {
  constexpr int brows = PAIR ? BN / 2 : BN;
  return (size_t)stages_for(brows) * stage_bytes(brows) + 1024 + 256 + extra_smem(BN);
}

template <int BN, bool SWAP = false, bool PAIR = false>
int prepare_bn() {
  return (int)cudaFuncSetAttribute(k_conv_gemm<BN, SWAP, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem_for<BN, SWAP, PAIR>());
}

template <int BN, bool SWAP = false, bool PAIR = false>
int launch_bn(const GemmParams& p, int grid, cudaStream_t stream) {
  return launch_kernel(k_conv_gemm<BN, SWAP, PAIR>, dim3(grid), dim3(384), smem_for<BN, SWAP, PAIR>(), stream,
                       PAIR ? 2 : 1, p);
}

}  // namespace

size_t conv_gemm_smem_bytes(int bn) { return (size_t)stages_for(bn) * stage_bytes(bn) + 1024 + 256 + extra_smem(bn); }
bool conv_gemm_pair_bn(int bn) { return bn == 128 || bn == 192; }

namespace {
template <int BN>
int pair_clusters_for() {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(384);
  cfg.dynamicSmemBytes = smem_for<BN, false, true>();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k_conv_gemm<BN, false, true>, &cfg) != cudaSuccess) return 0;
  return n;
}
}  // namespace

// Clusters of the pair kernels that fit on the current device at once (the
// smaller of the tile widths' counts).
int conv_gemm_pair_clusters() { return std::min(pair_clusters_for<128>(), pair_clusters_for<192>()); }

int conv_gemm_prepare() {
  int e = 0;
  if ((e = prepare_bn<16>())) return e;
  if ((e = prepare_bn<32>())) return e;
  if ((e = prepare_bn<64>())) return e;
  if ((e = prepare_bn<128>())) return e;
  if ((e = prepare_bn<192>())) return e;
  if ((e = prepare_bn<256, true>())) return e;
  if ((e = prepare_bn<128, false, true>())) return e;
  if ((e = prepare_bn<192, false, true>())) return e;
  return prepare_bn<256>();
}

int launch_conv_gemm(const GemmParams& p, int bn, int grid, cudaStream_t stream) {
  if (p.swap) return bn == 256 ? launch_bn<256, true>(p, grid, stream) : -1;
  if (p.pair) return bn == 128 ? launch_bn<128, false, true>(p, grid, stream)
                    : bn == 192 ? launch_bn<192, false, true>(p, grid, stream) : -1;
  switch (bn) {
    case 16: return launch_bn<16>(p, grid, stream);
    case 32: return launch_bn<32>(p, grid, stream);
    case 64: return launch_bn<64>(p, grid, stream);
    case 128: return launch_bn<128>(p, grid, stream);
    case 192: return launch_bn<192>(p, grid, stream);
    case 256: return launch_bn<256>(p, grid, stream);
    default: return -1;
  }
}

}  // namespace lama
