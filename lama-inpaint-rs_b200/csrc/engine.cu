// The B200 big-lama engine: weights, per-shape plans, CUDA graphs, C ABI.
//
// Host side of the drop-in boundary declared in include/lama_b200.h.  It
// replaces the reference's CUDA host engine (lama-rs/src/cuda.rs): module
// bring-up (:225-275), the size-bucketed allocator (:91-184), the weight arena
// and BN-fold staging (:330-387, :595-830), the device step tree (:903-962)
// and the launch loop (:1542-1691).  Design differences, B200-first:
//   * weights are repacked once at open into the operand layout of the
//     tensor-core kernel: per launch and per tile class a [2][N][K] split-bf16
//     matrix, with K-concatenated l2l|g2l and l2g|conv2 and the four
//     ConvTranspose phase matrices (cuda.rs:566-577 tap table);
//   * BatchNorm (cpu.rs:45-64) and conv biases fold into a per-channel
//     scale/shift applied in the GEMM epilogue;
//   * every activation buffer of a (batch, h, w) shape is allocated once (a
//     "plan"); the whole pass is captured into one CUDA graph and replayed;
//   * activations are NHWC split-bf16 with reflect halos written by the
//     producing epilogue, so ReflectPad, Concat and the residual adds cost no
//     launches.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "fft.cuh"
#include "gemm.cuh"
#include "lama_b200.h"
#include "launch.cuh"
#include "outconv.cuh"
#include "pointwise.cuh"
#include "ptx.cuh"
#include "weights.h"

using namespace lama;

namespace {

// ------------------------------------------------------------------ errors
struct EngineError {
  int code;
  std::string msg;
};

#define CK(x)                                                                                   \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) throw EngineError{LAMA_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)}; \
  } while (0)

#define CKL(x)                                                                                  \
  do {                                                                                          \
    int e_ = (x);                                                                               \
    if (e_ != 0)                                                                                \
      throw EngineError{LAMA_ECUDA, std::string(#x) + ": " + cudaGetErrorString((cudaError_t)e_)}; \
  } while (0)

// ------------------------------------------------------------------ host bf16
uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// ------------------------------------------------------------------ device memory
// A dry DevMem (capacity estimates) hands out distinct placeholder addresses
// that are never dereferenced and only counts the bytes.
struct DevMem {
  std::vector<void*> ptrs;
  size_t total = 0;
  bool dry = false;
  uintptr_t dry_next = (uintptr_t)1 << 40;
  void* alloc(size_t bytes, bool zero = true) {
    if (dry) {
      void* q = (void*)dry_next;
      dry_next += (std::max<size_t>(bytes, 256) + 255) / 256 * 256;
      total += bytes;
      return q;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 256));
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw EngineError{LAMA_ENOMEM, "cudaMalloc(" + std::to_string(bytes) + " bytes): " + cudaGetErrorString(e)};
    }
    if (zero) CK(cudaMemset(p, 0, std::max<size_t>(bytes, 256)));
    ptrs.push_back(p);
    total += bytes;
    return p;
  }
  void free_all() {
    for (void* p : ptrs) cudaFree(p);
    ptrs.clear();
    total = 0;
  }
  ~DevMem() { free_all(); }
};

// ------------------------------------------------------------------ tensor maps
// Resolved once per process.  A function-local static is initialised once even
// when engines on several devices are opened from several threads at a time
// (and is tried again on the next call if resolving it threw).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p)
      throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled is not available from the driver"};
    return (PFN_cuTensorMapEncodeTiled_v12000)p;
  }();
  return fn;
}

// Set while a plan is built dry (capacity estimates): tensor maps are left
// zero instead of being encoded, so no driver call is made.
thread_local bool t_dry_build = false;

CUresult encode_tiled(CUtensorMap* m, CUtensorMapDataType type, cuuint32_t rank, void* base, const cuuint64_t* dims,
                      const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr,
                      CUtensorMapInterleave il, CUtensorMapSwizzle sw, CUtensorMapL2promotion l2,
                      CUtensorMapFloatOOBfill oob) {
  if (t_dry_build) {
    memset(m, 0, sizeof(*m));
    return CUDA_SUCCESS;
  }
  return encode_fn()(m, type, rank, base, dims, strides, box, estr, il, sw, l2, oob);
}

// A split-bf16 NHWC activation: [2][B][H+2halo][W+2halo][C].
struct Act {
  void* p = nullptr;
  int B = 0, H = 0, W = 0, C = 0, halo = 0;
  long long part() const { return (long long)B * (H + 2 * halo) * (W + 2 * halo) * C; }
  size_t bytes() const { return (size_t)part() * 2 * 2; }
};

// Boxes of cb channels x (bw x bh) pixels; parts = 2 fetches the hi and lo
// planes in one copy (the lo box lands right after the hi box).
CUtensorMap act_map(const Act& a, int cb, int bw, int bh, int stride, bool interior, int parts = 1) {
  CUtensorMap m;
  const int hp = a.H + 2 * a.halo, wp = a.W + 2 * a.halo;
  char* base = (char*)a.p;
  cuuint64_t dims[5];
  if (interior) {
    base += (((size_t)a.halo * wp + a.halo) * a.C) * 2;
    dims[1] = (cuuint64_t)a.W;
    dims[2] = (cuuint64_t)a.H;
  } else {
    dims[1] = (cuuint64_t)wp;
    dims[2] = (cuuint64_t)hp;
  }
  dims[0] = (cuuint64_t)a.C;
  dims[3] = (cuuint64_t)a.B;
  dims[4] = 2;
  cuuint64_t strides[4] = {(cuuint64_t)a.C * 2, (cuuint64_t)wp * a.C * 2, (cuuint64_t)hp * wp * a.C * 2,
                           (cuuint64_t)a.part() * 2};
  cuuint32_t box[5] = {(cuuint32_t)cb, (cuuint32_t)(bw * stride), (cuuint32_t)(bh * stride), 1, (cuuint32_t)parts};
  cuuint32_t estr[5] = {1, (cuuint32_t)stride, (cuuint32_t)stride, 1, 1};
  CUresult r = encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           cb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled (activation) failed: " + std::to_string((int)r)};
  return m;
}

// Split output pixels (y, x) = (i * mul_y + add_y, j * mul_x + add_x) of one
// tile class as a dense (C, j, i, B, part) grid starting at the class's first
// interior pixel; boxes clip at the interior's far edges, so they never touch
// the trailing halo (written by reflection).
CUtensorMap out_map(void* p, long long part, int B, int C, int H, int W, int halo, int bw, int mul_y, int add_y,
                    int mul_x, int add_x) {
  CUtensorMap m;
  const int hp = H + 2 * halo, wp = W + 2 * halo;
  char* base = (char*)p + (((size_t)(add_y + halo) * wp + add_x + halo) * C) * 2;
  cuuint64_t dims[5] = {(cuuint64_t)C, (cuuint64_t)((W - add_x + mul_x - 1) / mul_x),
                        (cuuint64_t)((H - add_y + mul_y - 1) / mul_y), (cuuint64_t)B, 2};
  cuuint64_t strides[4] = {(cuuint64_t)C * 2 * mul_x, (cuuint64_t)wp * C * 2 * mul_y, (cuuint64_t)hp * wp * C * 2,
                           (cuuint64_t)part * 2};
  const int bx = std::min(bw, 32);
  cuuint32_t box[5] = {32, (cuuint32_t)bx, (cuuint32_t)(32 / bx), 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled (output) failed: " + std::to_string((int)r)};
  return m;
}

// fp32 output, NCHW (W, H, C, B) or NHWC (C, W, H, B), boxes of 32 channels x
// 32 pixels (min(bw, 32) wide).
CUtensorMap out_map_f32(void* p, bool nchw, int B, int C, int H, int W, int bw) {
  CUtensorMap m;
  const int bx = std::min(bw, 32);
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4];
  if (nchw) {
    dims[0] = (cuuint64_t)W; dims[1] = (cuuint64_t)H; dims[2] = (cuuint64_t)C; dims[3] = (cuuint64_t)B;
    strides[0] = (cuuint64_t)W * 4; strides[1] = (cuuint64_t)H * W * 4; strides[2] = (cuuint64_t)C * H * W * 4;
    box[0] = (cuuint32_t)bx; box[1] = (cuuint32_t)(32 / bx); box[2] = 32; box[3] = 1;
  } else {
    dims[0] = (cuuint64_t)C; dims[1] = (cuuint64_t)W; dims[2] = (cuuint64_t)H; dims[3] = (cuuint64_t)B;
    strides[0] = (cuuint64_t)C * 4; strides[1] = (cuuint64_t)W * C * 4; strides[2] = (cuuint64_t)H * W * C * 4;
    box[0] = 32; box[1] = (cuuint32_t)bx; box[2] = (cuuint32_t)(32 / bx); box[3] = 1;
  }
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           nchw ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::string d = " dims";
    for (int i = 0; i < 4; i++) d += " " + std::to_string((unsigned long long)dims[i]);
    d += " strides";
    for (int i = 0; i < 3; i++) d += " " + std::to_string((unsigned long long)strides[i]);
    d += " box";
    for (int i = 0; i < 4; i++) d += " " + std::to_string((unsigned)box[i]);
    throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled (fp32 output) failed: " + std::to_string((int)r) + d};
  }
  return m;
}

// ------------------------------------------------------------------ weights
struct WClass {
  int n = 0, npad = 0, k = 0;
  void* w = nullptr;            // [2][npad][k] bf16 on the device
  std::vector<uint16_t> host;   // staged until the device exists
};

struct GemmW {
  std::vector<WClass> cls;
  float* scale = nullptr;
  float* shift = nullptr;
  std::vector<float> hscale, hshift;
  int nout = 0;
};

// Boxes of 64 K x bn rows; parts = 2 as for act_map.
CUtensorMap w_map(const WClass& c, int bn, int parts = 1) {
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)c.k, (cuuint64_t)c.npad, 2};
  cuuint64_t strides[2] = {(cuuint64_t)c.k * 2, (cuuint64_t)c.npad * c.k * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)bn, (cuuint32_t)parts};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, c.w, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled (weights) failed: " + std::to_string((int)r)};
  return m;
}

struct FfcW {
  GemmW conv1, fu, out;
};

struct Weights {
  GemmW m1, m2, m3, m4;
  std::vector<FfcW> ffc;  // 36: block 0 conv1, block 0 conv2, ...
  GemmW ct[3];
  GemmW outc;
};

struct Loader {
  const WeightFile& wf;
  std::vector<float> get(const std::string& name, const std::vector<int64_t>& shape) {
    std::vector<float> v;
    std::string err;
    if (!wf.f32(name, shape, v, err)) throw EngineError{LAMA_EWEIGHTS, err};
    return v;
  }
  // cpu.rs:45-64 (`Bn::load`): s = w / sqrt(var + 1e-5), t = b - mean * s, in f32.
  void bn(const std::string& p, int c, std::vector<float>& s, std::vector<float>& t) {
    auto w = get(p + ".weight", {c}), b = get(p + ".bias", {c});
    auto mean = get(p + ".running_mean", {c}), var = get(p + ".running_var", {c});
    for (int i = 0; i < c; i++) {
      float sd = std::sqrt(var[i] + 1e-5f);
      float sc = w[i] / sd;
      float ms = mean[i] * sc;
      s.push_back(sc);
      t.push_back(b[i] - ms);
    }
  }
  // One class: fp32 [n][k] -> split bf16 [2][npad][k] on the device.
  WClass upload(const std::vector<float>& m, int n, int k) {
    WClass c;
    c.n = n;
    c.k = k;
    c.npad = (n + 15) / 16 * 16;
    std::vector<uint16_t> h((size_t)2 * c.npad * k, 0);
    for (int i = 0; i < n; i++)
      for (int j = 0; j < k; j++) {
        float v = m[(size_t)i * k + j];
        uint16_t hi = f2bf(v);
        uint16_t lo = f2bf(v - bf2f(hi));
        h[(size_t)i * k + j] = hi;
        h[(size_t)c.npad * k + (size_t)i * k + j] = lo;
      }
    c.host = std::move(h);
    return c;
  }
  void affine(GemmW& g, const std::vector<float>& s, const std::vector<float>& t) {
    g.nout = (int)s.size();
    g.hscale = s;
    g.hshift = t;
  }
};

// Copy every staged weight matrix and affine vector into one device arena.
void upload_gemm(GemmW& g, char*& cur) {
  for (WClass& c : g.cls) {
    c.w = cur;
    CK(cudaMemcpy(c.w, c.host.data(), c.host.size() * 2, cudaMemcpyHostToDevice));
    cur += (c.host.size() * 2 + 255) / 256 * 256;
    c.host.clear();
    c.host.shrink_to_fit();
  }
  g.scale = (float*)cur;
  CK(cudaMemcpy(g.scale, g.hscale.data(), g.hscale.size() * 4, cudaMemcpyHostToDevice));
  cur += (g.hscale.size() * 4 + 255) / 256 * 256;
  g.shift = (float*)cur;
  CK(cudaMemcpy(g.shift, g.hshift.data(), g.hshift.size() * 4, cudaMemcpyHostToDevice));
  cur += (g.hshift.size() * 4 + 255) / 256 * 256;
}

size_t gemm_bytes(const GemmW& g) {
  size_t b = 0;
  for (const WClass& c : g.cls) b += (c.host.size() * 2 + 255) / 256 * 256;
  return b + 2 * ((g.hscale.size() * 4 + 255) / 256 * 256);
}

template <class F>
void for_each_gemm(Weights& W, F&& f) {
  f(W.m1); f(W.m2); f(W.m3); f(W.m4);
  for (FfcW& x : W.ffc) { f(x.conv1); f(x.fu); f(x.out); }
  for (GemmW& g : W.ct) f(g);
  f(W.outc);
}

void upload_weights(Weights& W, DevMem& mem) {
  size_t total = 0;
  for_each_gemm(W, [&](GemmW& g) { total += gemm_bytes(g); });
  char* cur = (char*)mem.alloc(total, false);
  for_each_gemm(W, [&](GemmW& g) { upload_gemm(g, cur); });
}

// K order of a kxk conv segment: tap-major (ky, kx), then input channel.
void put_conv(std::vector<float>& m, int ktot, int kofs, const std::vector<float>& w, int cout, int cin, int kk,
              int row0 = 0) {
  for (int n = 0; n < cout; n++)
    for (int t = 0; t < kk * kk; t++)
      for (int c = 0; c < cin; c++)
        m[(size_t)(row0 + n) * ktot + kofs + t * cin + c] = w[((size_t)n * cin + c) * kk * kk + t];
}

// Reads, checks (names and shapes, as the reference's loaders do:
// cpu.rs:561-616, cuda.rs:832-962) and repacks every tensor on the host.
void load_weights(const WeightFile& wf, Weights& W) {
  Loader L{wf};
  std::vector<float> s, t;
  // model.1: 7x7 4->64 valid.  K = 8 row taps x 32, channel = kx*4 + c (28 used).
  {
    auto w = L.get("model.1.ffc.convl2l.weight", {64, 4, 7, 7});
    std::vector<float> m((size_t)64 * 256, 0.f);
    for (int n = 0; n < 64; n++)
      for (int ky = 0; ky < 7; ky++)
        for (int kx = 0; kx < 7; kx++)
          for (int c = 0; c < 4; c++) m[(size_t)n * 256 + ky * 32 + kx * 4 + c] = w[((n * 4 + c) * 7 + ky) * 7 + kx];
    W.m1.cls.push_back(L.upload(m, 64, 256));
    s.clear(); t.clear();
    L.bn("model.1.bn_l", 64, s, t);
    L.affine(W.m1, s, t);
  }
  // model.2, model.3: 3x3 stride-2 reflect
  const int enc[2][3] = {{2, 64, 128}, {3, 128, 256}};
  GemmW* encw[2] = {&W.m2, &W.m3};
  for (int e = 0; e < 2; e++) {
    const int idx = enc[e][0], cin = enc[e][1], cout = enc[e][2];
    auto w = L.get("model." + std::to_string(idx) + ".ffc.convl2l.weight", {cout, cin, 3, 3});
    std::vector<float> m((size_t)cout * 9 * cin, 0.f);
    put_conv(m, 9 * cin, 0, w, cout, cin, 3);
    encw[e]->cls.push_back(L.upload(m, cout, 9 * cin));
    s.clear(); t.clear();
    L.bn("model." + std::to_string(idx) + ".bn_l", cout, s, t);
    L.affine(*encw[e], s, t);
  }
  // model.4: 256 -> 128 local (l2l) + 384 global (l2g)
  {
    auto l2l = L.get("model.4.ffc.convl2l.weight", {128, 256, 3, 3});
    auto l2g = L.get("model.4.ffc.convl2g.weight", {384, 256, 3, 3});
    std::vector<float> m((size_t)512 * 2304, 0.f);
    put_conv(m, 2304, 0, l2l, 128, 256, 3, 0);
    put_conv(m, 2304, 0, l2g, 384, 256, 3, 128);
    W.m4.cls.push_back(L.upload(m, 512, 2304));
    s.clear(); t.clear();
    L.bn("model.4.bn_l", 128, s, t);
    L.bn("model.4.bn_g", 384, s, t);
    L.affine(W.m4, s, t);
  }
  // 18 resblocks x 2 FFC layers
  for (int blk = 5; blk <= 22; blk++)
    for (int sub = 1; sub <= 2; sub++) {
      const std::string part = "model." + std::to_string(blk) + ".conv" + std::to_string(sub);
      const std::string p = part + ".ffc";
      FfcW f;
      auto c1 = L.get(p + ".convg2g.conv1.0.weight", {192, 384, 1, 1});
      f.conv1.cls.push_back(L.upload(c1, 192, 384));
      s.clear(); t.clear();
      L.bn(p + ".convg2g.conv1.1", 192, s, t);
      L.affine(f.conv1, s, t);
      auto fu = L.get(p + ".convg2g.fu.conv_layer.weight", {384, 384, 1, 1});
      f.fu.cls.push_back(L.upload(fu, 384, 384));
      s.clear(); t.clear();
      L.bn(p + ".convg2g.fu.bn", 384, s, t);
      L.affine(f.fu, s, t);
      // local class: 3x3 over all 512 channels = [l2l | g2l]
      auto l2l = L.get(p + ".convl2l.weight", {128, 128, 3, 3});
      auto g2l = L.get(p + ".convg2l.weight", {128, 384, 3, 3});
      std::vector<float> ml((size_t)128 * 4608, 0.f);
      for (int n = 0; n < 128; n++)
        for (int tp = 0; tp < 9; tp++) {
          for (int c = 0; c < 128; c++) ml[(size_t)n * 4608 + tp * 512 + c] = l2l[((size_t)n * 128 + c) * 9 + tp];
          for (int c = 0; c < 384; c++)
            ml[(size_t)n * 4608 + tp * 512 + 128 + c] = g2l[((size_t)n * 384 + c) * 9 + tp];
        }
      f.out.cls.push_back(L.upload(ml, 128, 4608));
      // global class: 3x3 over the 128 local channels (l2g), then 1x1 over S (conv2)
      auto l2g = L.get(p + ".convl2g.weight", {384, 128, 3, 3});
      auto cv2 = L.get(p + ".convg2g.conv2.weight", {384, 192, 1, 1});
      std::vector<float> mg((size_t)384 * 1344, 0.f);
      put_conv(mg, 1344, 0, l2g, 384, 128, 3);
      for (int n = 0; n < 384; n++)
        for (int c = 0; c < 192; c++) mg[(size_t)n * 1344 + 1152 + c] = cv2[(size_t)n * 192 + c];
      f.out.cls.push_back(L.upload(mg, 384, 1344));
      s.clear(); t.clear();
      L.bn(part + ".bn_l", 128, s, t);
      L.bn(part + ".bn_g", 384, s, t);
      L.affine(f.out, s, t);
      W.ffc.push_back(std::move(f));
    }
  // ConvTranspose2d k3 s2 p1 op1 as four output phases; weight [cin][cout][3][3].
  // Phase (py, px) taps: (ky, kx, dy, dx) with input pixel (i + dy, j + dx).
  static const int taps[4][4][4] = {
      {{1, 1, 0, 0}},
      {{1, 0, 0, 1}, {1, 2, 0, 0}},
      {{0, 1, 1, 0}, {2, 1, 0, 0}},
      {{0, 0, 1, 1}, {0, 2, 1, 0}, {2, 0, 0, 1}, {2, 2, 0, 0}}};
  static const int ntaps[4] = {1, 2, 2, 4};
  const int ups[3][4] = {{24, 25, 512, 256}, {27, 28, 256, 128}, {30, 31, 128, 64}};
  for (int u = 0; u < 3; u++) {
    const int idx = ups[u][0], bnx = ups[u][1], cin = ups[u][2], cout = ups[u][3];
    auto w = L.get("model." + std::to_string(idx) + ".weight", {cin, cout, 3, 3});
    auto bias = L.get("model." + std::to_string(idx) + ".bias", {cout});
    for (int ph = 0; ph < 4; ph++) {
      const int k = ntaps[ph] * cin;
      std::vector<float> m((size_t)cout * k, 0.f);
      for (int n = 0; n < cout; n++)
        for (int ti = 0; ti < ntaps[ph]; ti++) {
          const int ky = taps[ph][ti][0], kx = taps[ph][ti][1];
          for (int c = 0; c < cin; c++) m[(size_t)n * k + ti * cin + c] = w[(((size_t)c * cout + n) * 3 + ky) * 3 + kx];
        }
      W.ct[u].cls.push_back(L.upload(m, cout, k));
    }
    s.clear(); t.clear();
    L.bn("model." + std::to_string(bnx), cout, s, t);
    // (acc + bias) * s + t  ->  acc * s + (bias * s + t)
    for (int n = 0; n < cout; n++) t[n] = bias[n] * s[n] + t[n];
    L.affine(W.ct[u], s, t);
  }
  // OutConv 7x7 64 -> 3 with bias, over the reflect-padded input, for the
  // row-ring kernel (outconv.cu): n = ky*21 + kx*3 + co (147 of 160), K = c.
  {
    auto w = L.get("model.34.weight", {3, 64, 7, 7});
    auto bias = L.get("model.34.bias", {3});
    std::vector<float> m2((size_t)160 * 64, 0.f);
    for (int ky = 0; ky < 7; ky++)
      for (int kx = 0; kx < 7; kx++)
        for (int co = 0; co < 3; co++)
          for (int c = 0; c < 64; c++)
            m2[(size_t)(ky * 21 + kx * 3 + co) * 64 + c] = w[(((size_t)co * 64 + c) * 7 + ky) * 7 + kx];
    W.outc.cls.push_back(L.upload(m2, 160, 64));
    std::vector<float> one(32, 1.f), sh(32, 0.f);
    for (int n = 0; n < 3; n++) sh[n] = bias[n];
    L.affine(W.outc, one, sh);
  }
}

// The shapes (not the values) of every packed weight class, as load_weights
// builds them: what a dry plan build needs to estimate a pass's memory
// without a checkpoint or a GPU.
void weight_shapes(Weights& W) {
  auto cls = [](int n, int k) {
    WClass c;
    c.n = n;
    c.k = k;
    c.npad = (n + 15) / 16 * 16;
    return c;
  };
  W.m1.cls = {cls(64, 256)};
  W.m2.cls = {cls(128, 576)};
  W.m3.cls = {cls(256, 1152)};
  W.m4.cls = {cls(512, 2304)};
  W.ffc.assign(36, FfcW());
  for (FfcW& f : W.ffc) {
    f.conv1.cls = {cls(192, 384)};
    f.fu.cls = {cls(384, 384)};
    f.out.cls = {cls(128, 4608), cls(384, 1344)};
  }
  const int ntaps[4] = {1, 2, 2, 4}, cins[3] = {512, 256, 128};
  for (int u = 0; u < 3; u++) {
    W.ct[u].cls.clear();
    for (int ph = 0; ph < 4; ph++) W.ct[u].cls.push_back(cls(cins[u] / 2, ntaps[ph] * cins[u]));
  }
  W.outc.cls = {cls(160, 64)};
}

// The loaded checkpoint's packed classes have the shapes weight_shapes gives.
void check_weight_shapes(Weights& loaded) {
  Weights ref;
  weight_shapes(ref);
  std::vector<std::pair<int, int>> a, b;
  for_each_gemm(loaded, [&](GemmW& g) { for (auto& c : g.cls) a.push_back({c.n, c.k}); });
  for_each_gemm(ref, [&](GemmW& g) { for (auto& c : g.cls) b.push_back({c.n, c.k}); });
  if (a != b) throw EngineError{LAMA_EUNSUPPORTED, "packed weight shapes differ from the capacity model"};
}

// ------------------------------------------------------------------ ops
enum OpKind { OP_GEMM, OP_RFFT, OP_IRFFT, OP_RFFT_REG, OP_IRFFT_REG, OP_RFFT_PF, OP_RFFT_TC, OP_IRFFT_PAR, OP_OUTCONV, OP_UNFOLD_F32, OP_UNFOLD_U8, OP_TO_SPLIT, OP_TO_NCHW, OP_COPY };

struct Op {
  OpKind kind;
  std::string name;
  int bn = 0, grid = 0;
  std::unique_ptr<GemmParams> g;
  std::unique_ptr<FftPfParams> fpf;
  std::unique_ptr<FftTcParams> ftc;
  const void* csrc = nullptr;  // OP_COPY: device-to-device copy
  void* cdst = nullptr;
  size_t cbytes = 0;
  std::unique_ptr<OutConvParams> oc;
  FftParams f{};
  UnfoldParams u{};
  ConvertParams cv{};
  double flops = 0, bytes = 0;
  // split-K: workspace floats and tile counters this GEMM needs; ops of one
  // lane run one after another, so they share the plan's workspace of that
  // lane (the finisher of a tile resets its counter)
  size_t ws_floats = 0;
  int ws_counters = 0;
  // Graph lanes: lane 1 ops run on a second stream concurrently with lane 0;
  // `waits` are earlier ops of the other lane this op must follow (within a
  // lane, program order).  Eager runs (profiling, debug) issue every op on
  // one stream in plan order, which respects the same dependencies.
  int lane = 0;
  std::vector<int> waits;
  bool pdl = false;  // programmatic dependent launch (small passes)
  // output tensor, for the diagnostics entry points: split bf16 or fp32,
  // dims = (B, rows, cols, channels) of the stored layout (halo included;
  // NCHW outputs report (B, C, H, W)).
  void* out_ptr = nullptr;
  int out_split = 0;
  long long out_part = 0;
  int dims[4] = {0, 0, 0, 0};
};

}  // namespace
namespace lama {
thread_local bool t_pdl_launch = false;
}
namespace {

int launch_op_kind(const Op& op, cudaStream_t st);

// A plan's launch; with op.pdl the kernel may start while the previous one on
// its stream finishes (programmatic dependent launch, launch.cuh).
int launch_op(const Op& op, cudaStream_t st) {
  t_pdl_launch = op.pdl;
  const int r = launch_op_kind(op, st);
  t_pdl_launch = false;
  return r;
}

int launch_op_kind(const Op& op, cudaStream_t st) {
  switch (op.kind) {
    case OP_GEMM: return launch_conv_gemm(*op.g, op.bn, op.grid, st);
    case OP_RFFT: return launch_rfft2(op.f, st);
    case OP_IRFFT: return launch_irfft2(op.f, st);
    case OP_RFFT_REG: return launch_fft_reg(op.f, false, st);
    case OP_IRFFT_REG: return launch_fft_reg(op.f, true, st);
    case OP_RFFT_PF: return launch_rfft2_pf(*op.fpf, op.grid, st);
    case OP_RFFT_TC: return launch_rfft2_tc(*op.ftc, op.grid, st);
    case OP_IRFFT_PAR: return launch_irfft2_par(op.f, op.grid, st);
    case OP_OUTCONV: return launch_outconv(*op.oc, op.grid, st);
    case OP_UNFOLD_F32: return launch_unfold_f32(op.u, st);
    case OP_UNFOLD_U8: return launch_unfold_u8(op.u, st);
    case OP_TO_SPLIT: return launch_nchw_to_split(op.cv, st);
    case OP_TO_NCHW: return launch_split_to_nchw(op.cv, st);
    case OP_COPY: return (int)cudaMemcpyAsync(op.cdst, op.csrc, op.cbytes, cudaMemcpyDeviceToDevice, st);
  }
  return -1;
}

struct SegSpec {
  int amap, c0, nch, stride;
  std::vector<std::pair<int, int>> taps;  // (dy, dx)
};
struct ClassSpec {
  int wc, n0, nvalid;
  int oy_mul = 1, oy_add = 0, ox_mul = 1, ox_add = 0;
  std::vector<SegSpec> segs;
};

ClassSpec one_seg(int wc, int n0, int nvalid, SegSpec seg) {
  ClassSpec c{wc, n0, nvalid};
  c.segs.push_back(std::move(seg));
  return c;
}
struct AmapSpec {
  Act act;
  int stride;
  bool interior;
};
struct OutSpec {
  int kind;
  void* p;
  long long part;
  int c, h, w, halo, reflect;
  const void* skip;
};

// Tile of `px` pixels (bh x bw) over an mh x mw grid, least padding waste;
// TMA boxes cap each side at 256 / stride.
void choose_tile(int mh, int mw, int& bh, int& bw, int px = 128, int stride = 1) {
  long long best = -1;
  for (int cand = px; cand >= 8; cand >>= 1) {
    const int ch = px / cand;
    if (cand * stride > 256 || ch * stride > 256) continue;
    const long long cost = (long long)((mh + ch - 1) / ch) * ch * ((mw + cand - 1) / cand) * cand;
    if (best < 0 || cost < best) {
      best = cost;
      bw = cand;
      bh = ch;
    }
  }
}

}  // namespace

// ------------------------------------------------------------------ engine
constexpr int kDefaultChainSms = 40;
// convT2 and convT3 run the four phase tiles of each pixel tile on one CTA
// in a row, so the input rows they share are read from HBM once (measured at
// 64 images: convT3 4.35 -> 3.93 ms, convT2 1.84 -> 1.81; convT1, whose input
// is small enough to stay in L2, 1.44 -> 1.54, so it keeps class order)
constexpr bool kConvTClassGroups = true;

struct Plan {
  int kind = 0;  // 0 f32 forward, 1 u8 inpaint, 2 resblocks, 3 one --sections pass (window)
  int B = 0, H = 0, W = 0, h = 0, w = 0, nblocks = 0;
  DevMem mem;
  float* in_f32 = nullptr;
  float* out = nullptr;
  uint8_t *rgb = nullptr, *mask = nullptr, *out_rgb = nullptr;
  WinDesc* win = nullptr;  // kind 3: the pass's window, read by the kernels at run time
  float *l_in = nullptr, *g_in = nullptr, *l_out = nullptr, *g_out = nullptr;
  std::vector<Op> ops;
  cudaGraphExec_t exec = nullptr;
  ~Plan() {
    if (exec) cudaGraphExecDestroy(exec);
  }
};

struct lama_engine {
  int device = 0;
  int sms = 148;
  std::string gpu_name = "the GPU";
  cudaStream_t stream = nullptr;
  cudaStream_t side_stream = nullptr;  // the second graph lane's stream during capture
  std::string err;
  DevMem wmem;
  Weights W;
  int* d_err = nullptr;
  int tiling = LAMA_TILING_AUTO;
  int spectral = LAMA_SPECTRAL_AUTO;
  int pair_clusters = 0;  // co-resident CTA-pair clusters (0: no pair tiles)
  int chain_sms = kDefaultChainSms;  // SMs of the spectral graph lane at small batches (0: one lane)
  std::map<std::tuple<int, int, int, int, int, int, int>, std::unique_ptr<Plan>> plans;
  // lama_inpaint_u8_stream: copy stream and double-buffered staging
  cudaStream_t copy_stream = nullptr;
  DevMem pipe_mem;
  size_t pipe_bytes = 0;  // bytes of one staging set (rgb + mask + out)
  uint8_t* pipe_buf[2] = {nullptr, nullptr};
  cudaEvent_t ev_in[2] = {nullptr, nullptr}, ev_done[2] = {nullptr, nullptr};
  // --sections: the device-resident working image, mask and pass windows
  DevMem sec_mem;
  uint8_t* sec_img = nullptr;
  uint8_t* sec_mask = nullptr;
  WinDesc* sec_desc = nullptr;
  size_t sec_px = 0, sec_n = 0;
};

namespace {

constexpr size_t kFftSmem = 160 * 1024;  // dynamic shared memory cap of the two-pass spectral kernels

struct Builder {
  lama_engine& e;
  Plan& pl;

  void build_ops();  // every launch of the plan's pass, in order

  // SMs of the spectral lane for an FFC stack of B images of h x w latents,
  // or 0 for one lane: small launches (fewer 128 x 128 output tiles of the
  // FFC GEMM than SMs) whose latent suits the row-union CTA-pair tiles.
  int lanes_for(int B, int h, int w) const {
    if (e.chain_sms <= 0 || e.tiling != LAMA_TILING_AUTO || e.pair_clusters <= 0) return 0;
    if (w % 32 || h % 4) return 0;
    // measured: two lanes win at one 512x512 image (3.75 vs 3.91 ms) and lose
    // at two (5.9 vs 5.1 ms), where the GEMM alone nearly fills the GPU
    const long long outs = (long long)B * ((h * w + 127) / 128) * 4;
    if (outs >= e.sms) return 0;
    return std::min(e.chain_sms, e.sms / 2);
  }

  // The register-resident spectral kernels are the faster choice wherever
  // they apply (measured at batch 1 and 32 on 64x64 planes).
  bool use_reg_fft() const { return e.spectral != LAMA_SPECTRAL_TWO_PASS; }

  Act act(int B, int H, int W, int C, int halo) {
    Act a;
    a.B = B; a.H = H; a.W = W; a.C = C; a.halo = halo;
    a.p = pl.mem.alloc(a.bytes());
    return a;
  }

  int choose_bn(const std::vector<int>& ns, int m_tiles) {
    if (ns.size() == 1 && ns[0] < 16) return 16;
    const int cands[4] = {256, 192, 128, 64};
    int fallback = 0;
    for (int bn : cands) {
      bool ok = true;
      long long tiles = 0;
      for (int n : ns) {
        if (n % bn) ok = false;
        tiles += (long long)m_tiles * (n / std::max(bn, 1));
      }
      if (!ok) continue;
      fallback = bn;
      if (tiles >= e.sms) return bn;
    }
    return fallback;
  }

  // One GEMM launch (pushed to the plan).  max_sms caps the SMs it runs on
  // (0 = all; graph lanes share the GPU); tail_class >= 0 runs that class's
  // last K segment as its own split-K part in a second launch pushed right
  // after the first (tail_flops of the algorithmic FLOPs), which finishes the
  // class's tiles from the first launch's partial sums.
  void gemm(const std::string& name, const GemmW& Wt, const std::vector<AmapSpec>& amaps,
            const std::vector<ClassSpec>& classes, int cb, int B, int mh, int mw, const OutSpec& o, int relu,
            int sigmoid, double flops, int max_sms = 0, int tail_class = -1, double tail_flops = 0,
            bool class_groups = false) {
    const int sms = max_sms > 0 ? std::min(max_sms, e.sms) : e.sms;
    const int clusters = std::min(e.pair_clusters, sms / 2);
    Op op;
    op.kind = OP_GEMM;
    op.name = name;
    op.flops = flops;
    op.g.reset(new GemmParams());
    GemmParams& p = *op.g;
    memset(&p, 0, sizeof(p));
    int max_stride = 1;
    for (auto& a : amaps) max_stride = std::max(max_stride, a.stride);
    // Swapped tiles (M = 128 output channels, N = 256 pixels) stage more MACs per
    // byte and apply when every class has a multiple of 128 channels.  Measured:
    // since split outputs leave through TMA stores (pixel-major tiles only),
    // pixel-major tiles beat swapped ones for the FFC layers at batch 1 and 32
    // and for the FourierUnit conv, so only LAMA_TILING_SWAPPED selects them.
    bool swap = e.tiling == LAMA_TILING_SWAPPED && cb == 64 &&
                (o.kind == OUT_SPLIT || o.kind == OUT_F32_NHWC);
    for (auto& c : classes) swap = swap && c.nvalid % 128 == 0;
    int bh = 1, bw = 128;
    if (swap) {
      choose_tile(mh, mw, bh, bw, 256, max_stride);
    }
    if (!swap) {
      bh = 1;
      bw = 128;
      choose_tile(mh, mw, bh, bw, 128, max_stride);
    }
    p.swap = swap ? 1 : 0;
    p.cb = cb;
    p.batch = B;
    p.mh = mh;
    p.mw = mw;
    p.bh = bh;
    p.bw = bw;
    p.tiles_y = (mh + bh - 1) / bh;
    p.tiles_x = (mw + bw - 1) / bw;
    p.m_tiles = B * p.tiles_y * p.tiles_x;
    std::vector<int> ns;
    for (auto& c : classes) ns.push_back(c.nvalid);
    // Small launches (under two 128 x 128 output tiles per SM, e.g. the FFC
    // layers of a batch-1 pass) whose taps allow the row union run as CTA
    // pairs of 256 x 128 tiles with the union and split K: each SM then stages
    // a quarter of the operand bytes per MMA that 128 x 64 tiles with per-tap
    // boxes need, which is what bounds such launches (L2 -> SM traffic).
    bool small_union = false;
    if (!swap && e.tiling == LAMA_TILING_AUTO && cb == 64 && e.pair_clusters > 0 && mw % 32 == 0 && mh % 4 == 0) {
      long long outs = 0;
      bool ok = true, taps = false;
      for (auto& c : classes) {
        ok = ok && c.nvalid % 128 == 0;
        outs += (long long)p.m_tiles * (c.nvalid / 128);
        for (auto& sg : c.segs) {
          ok = ok && sg.stride == 1;
          taps = taps || sg.taps.size() > 1;
        }
      }
      small_union = ok && taps && outs < 2LL * e.sms;
    }
    const int bn = swap ? 256 : small_union ? 128 : choose_bn(ns, p.m_tiles);
    if (!bn) throw EngineError{LAMA_EUNSUPPORTED, name + ": no tile width divides the output channels"};
    op.bn = bn;
    // CTA pairs (256 x BN tiles over two SMs) where the kernel has them and
    // there are enough tiles for every SM (or split K fills it, above)
    const bool pair = !swap && conv_gemm_pair_bn(bn) && e.pair_clusters > 0 &&
                      (e.tiling == LAMA_TILING_PAIRED || small_union ||
                       (e.tiling == LAMA_TILING_AUTO && p.m_tiles >= 2 * e.sms));
    p.pair = pair ? 1 : 0;
    // Row union: 3x3-style taps that share dx read the row windows of one box
    // of bh + 2 rows per 64-channel block instead of one box per tap.  Tiles
    // of 4 x 32 pixels; the kernel's union stages exist for 64 B rows per CTA
    // (BN = 64 single CTAs, BN = 128 pairs); split-K launches keep per-tap boxes.
    std::vector<std::vector<GemmGroup>> groups(classes.size());
    // 32-channel boxes (model.1): two taps per K block, so groups are whole K
    // blocks (2 or 4 consecutive taps of one-block segments)
    bool uni = !swap && (cb == 64 || cb == 32) && (pair ? bn == 128 : bn == 64) && mw % 32 == 0 && mh % 4 == 0;
    const int maxrun = cb == 64 ? 3 : 4;
    bool multi = false;
    for (size_t ci = 0; ci < classes.size() && uni; ci++) {
      int sub_base = 0;  // first cb-channel sub-box of the segment in the class's K order
      for (size_t si = 0; si < classes[ci].segs.size() && uni; si++) {
        const SegSpec& ss = classes[ci].segs[si];
        if (ss.stride != 1 || (cb == 32 && ss.nch != 32)) { uni = false; break; }
        std::vector<int> done(ss.taps.size(), 0);
        for (size_t t0 = 0; t0 < ss.taps.size(); t0 += done[t0] ? 1 : 0) {
          if (done[t0]) continue;
          // the run of taps with this dx and dy = dy0, dy0 + 1, dy0 + 2
          GemmGroup g{};
          g.seg = (int8_t)si;
          g.dx = (int8_t)ss.taps[t0].second;
          g.dy0 = (int8_t)ss.taps[t0].first;
          for (size_t t = 0; t < ss.taps.size(); t++)  // start at the smallest dy left in this column
            if (!done[t] && ss.taps[t].second == g.dx) g.dy0 = (int8_t)std::min<int>(g.dy0, ss.taps[t].first);
          g.ndy = 0;
          for (int d = 0; d < maxrun; d++) {
            int found = -1;
            for (size_t t = 0; t < ss.taps.size(); t++)
              if (!done[t] && ss.taps[t].second == g.dx && ss.taps[t].first == g.dy0 + d) found = (int)t;
            if (found < 0) break;
            done[found] = 1;
            g.tap[g.ndy++] = (int8_t)found;
          }
          if (cb == 32) {  // whole K blocks: an even run of consecutive tap indices starting a block
            bool whole = g.ndy % 2 == 0 && (sub_base + g.tap[0]) % 2 == 0;
            for (int j = 1; j < g.ndy; j++) whole = whole && g.tap[j] == g.tap[0] + j;
            if (!whole) { uni = false; break; }
          }
          multi = multi || g.ndy > 1;
          groups[ci].push_back(g);
        }
        sub_base += (ss.nch / cb) * (int)ss.taps.size();
      }
      if (groups[ci].size() > (size_t)GEMM_MAX_GROUPS) uni = false;
    }
    uni = uni && multi;
    if (uni) {
      bh = 4;
      bw = 32;
      p.bh = bh;
      p.bw = bw;
      p.tiles_y = (mh + bh - 1) / bh;
      p.tiles_x = (mw + bw - 1) / bw;
      p.m_tiles = B * p.tiles_y * p.tiles_x;
    }
    for (size_t i = 0; i < amaps.size(); i++)
      p.amap[i] = act_map(amaps[i].act, cb, bw, bh, amaps[i].stride, amaps[i].interior, 2);
    for (size_t i = amaps.size(); i < (size_t)GEMM_MAX_AMAPS; i++) p.amap[i] = p.amap[0];
    p.nclass = (int)classes.size();
    int tile0 = 0;
    for (size_t ci = 0; ci < classes.size(); ci++) {
      const ClassSpec& cs = classes[ci];
      GemmClass& C = p.cls[ci];
      const WClass& wc = Wt.cls[cs.wc];
      p.bmap[ci] = w_map(wc, swap ? 128 : pair ? bn / 2 : bn, 2);
      C.n0 = cs.n0;
      C.nvalid = cs.nvalid;
      C.ntiles_n = swap ? cs.nvalid / 128 : (cs.nvalid + bn - 1) / bn;
      C.oy_mul = cs.oy_mul; C.oy_add = cs.oy_add; C.ox_mul = cs.ox_mul; C.ox_add = cs.ox_add;
      C.nseg = (int)cs.segs.size();
      int sub = 0;
      for (size_t si = 0; si < cs.segs.size(); si++) {
        const SegSpec& ss = cs.segs[si];
        GemmSeg& S = C.seg[si];
        S.amap = ss.amap;
        S.c0 = ss.c0;
        S.nblk = ss.nch / cb;
        S.ntaps = (int)ss.taps.size();
        S.stride = ss.stride;
        S.sub0 = sub;
        for (size_t t = 0; t < ss.taps.size(); t++) {
          S.dy[t] = (int8_t)ss.taps[t].first;
          S.dx[t] = (int8_t)ss.taps[t].second;
        }
        sub += S.nblk * S.ntaps;
      }
      if ((sub * cb) % 64) throw EngineError{LAMA_EUNSUPPORTED, name + ": K is not a multiple of 64"};
      C.nkb = sub * cb / 64;
      if (C.nkb * 64 != wc.k)
        throw EngineError{LAMA_EUNSUPPORTED, name + ": K mismatch between plan and packed weights"};
    }
    // Row-union groups of every class (kernel mode p.uni).
    if (uni) {
      p.uni = 1;
      int span[GEMM_MAX_AMAPS] = {1, 1, 1};
      for (size_t ci = 0; ci < classes.size(); ci++) {
        GemmClass& C = p.cls[ci];
        C.ngroup = (int)groups[ci].size();
        for (int g = 0; g < C.ngroup; g++) {
          C.grp[g] = groups[ci][g];
          const int a = C.seg[C.grp[g].seg].amap;
          span[a] = std::max(span[a], (int)C.grp[g].ndy);
        }
      }
      for (size_t i = 0; i < amaps.size(); i++) {
        p.urows[i] = bh + span[i] - 1;
        p.amap_u[i] = act_map(amaps[i].act, cb, bw, p.urows[i], 1, amaps[i].interior, 2);
      }
    }
    // K units of each class and their weight in 64-wide K blocks: K blocks,
    // or (row union) one unit per group and channel block, in group order.
    std::vector<std::vector<int>> unit_kb(classes.size());
    for (size_t ci = 0; ci < classes.size(); ci++) {
      const GemmClass& C = p.cls[ci];
      if (uni) {
        for (int g = 0; g < C.ngroup; g++)
          for (int blk = 0; blk < C.seg[C.grp[g].seg].nblk; blk++)
            unit_kb[ci].push_back(cb == 32 ? C.grp[g].ndy / 2 : C.grp[g].ndy);
      } else {
        unit_kb[ci].assign(C.nkb, 1);
      }
    }
    // Split-K for launches too small to fill the GPU (batch-1 passes): K parts
    // of at most ~the per-SM (per-pair) share of all K blocks, finished
    // in-kernel by the last part (32-column chunks).  Parts are cut at unit
    // boundaries with balanced K blocks.
    // (from the SM count alone, so that the plan's memory does not depend on
    // how many clusters the device co-schedules)
    const int slots = pair ? sms / 2 : sms;
    const long long mt_sched = pair ? (p.m_tiles + 1) / 2 : p.m_tiles;  // output tiles per N tile as scheduled
    long long kbs = 0;
    for (size_t ci = 0; ci < classes.size(); ci++) kbs += mt_sched * p.cls[ci].ntiles_n * p.cls[ci].nkb;
    const int share = pair ? (int)std::max<long long>(12, (kbs + 2 * slots - 1) / (2 * slots))
                           : (int)std::max<long long>(12, (kbs + slots - 1) / slots);
    const bool can_split = !swap && bn >= 32;
    if (tail_class >= 0 && (!can_split || tail_class >= (int)classes.size() || classes[tail_class].segs.size() < 2))
      throw EngineError{LAMA_EUNSUPPORTED, name + ": a separate tail launch needs a splittable class of two segments"};
    int ws_tiles = 0;
    for (size_t ci = 0; ci < classes.size(); ci++) {
      GemmClass& C = p.cls[ci];
      const std::vector<int>& uk = unit_kb[ci];
      const bool tail = (int)ci == tail_class;
      // units [0, nhead) are split into parts; a tail class's last segment
      // (units [nhead, nunits)) is one more part of its own
      const int nunits = (int)uk.size();
      int nhead = nunits;
      if (tail) {
        nhead = 0;
        const int last = C.nseg - 1;
        if (uni) {
          for (int g = 0; g < C.ngroup; g++)
            if (C.grp[g].seg != last) nhead += C.seg[C.grp[g].seg].nblk;
        } else {
          nhead = C.seg[last].sub0 * cb / 64;
        }
      }
      int kb_head = 0;
      for (int u = 0; u < nhead; u++) kb_head += uk[u];
      int nsplit = can_split ? std::min(GEMM_MAX_KSPLIT - (tail ? 1 : 0), std::max(1, (kb_head + share - 1) / share)) : 1;
      nsplit = std::min(nsplit, nhead);
      // cut q ends at the first unit boundary with >= (q + 1) / nsplit of the head's K blocks
      C.kcut[0] = 0;
      int u = 0, acc = 0;
      for (int q = 0; q < nsplit; q++) {
        const long long goal = (long long)kb_head * (q + 1) / nsplit;
        while (u < nhead && (acc < goal || u <= C.kcut[q]) && nhead - u > nsplit - 1 - q) acc += uk[u++];
        C.kcut[q + 1] = (int16_t)u;
      }
      C.kcut[nsplit] = (int16_t)nhead;
      C.ksplit = nsplit;
      if (tail) C.kcut[++C.ksplit] = (int16_t)nunits;
      C.part0 = 0;
      C.nparts = tail ? C.ksplit - 1 : C.ksplit;
      C.ws_tile0 = ws_tiles;
      // one slice per part and per CTA-sized output tile (pairs: per CTA of the pair)
      if (C.ksplit > 1) ws_tiles += (int)(pair ? 2 * mt_sched : p.m_tiles) * C.ntiles_n * C.ksplit;
      C.tile0 = tile0;
      tile0 += (int)mt_sched * C.ntiles_n * C.nparts;
    }
    if (ws_tiles) {  // pointers are set once the plan's shared workspace exists
      op.ws_floats = (size_t)ws_tiles * bn * 128;
      op.ws_counters = ws_tiles;
    }
    p.total_tiles = tile0;
    p.scale = Wt.scale;
    p.shift = Wt.shift;
    p.relu = relu;
    p.sigmoid = sigmoid;
    p.out_kind = o.kind;
    p.out = o.p;
    p.out_part = o.part;
    p.out_c = o.c;
    p.out_h = o.h;
    p.out_w = o.w;
    p.out_halo = o.halo;
    p.out_reflect = o.reflect;
    p.skip = o.skip;
    p.err = e.d_err;
    // outputs of pixel-major tiles leave through TMA stores (TMA boxes need a
    // 16-byte aligned innermost coordinate: channel starts on multiples of
    // 32; fp32 NCHW, whose innermost coordinate is x, needs dense placement
    // and 16-byte rows and tile columns)
    bool aligned = o.c % 32 == 0, dense = true;
    for (auto& c : classes) {
      aligned = aligned && c.n0 % 32 == 0;
      dense = dense && c.oy_mul == 1 && c.ox_mul == 1 && c.oy_add == 0 && c.ox_add == 0;
    }
    if (!swap && (bn == 64 || bn == 128 || bn == 192) && aligned &&
        (bw >= 32 ? bw % 32 == 0 : 32 % bw == 0)) {
      if (o.kind == OUT_SPLIT) {
        for (size_t ci = 0; ci < classes.size(); ci++) {
          const ClassSpec& c = classes[ci];
          p.omap[ci] = out_map(o.p, o.part, B, o.c, o.h, o.w, o.halo, bw, c.oy_mul, c.oy_add, c.ox_mul, c.ox_add);
        }
        p.ostore = 1;
      } else if (dense && o.halo == 0 &&
                 (o.kind == OUT_F32_NHWC || (o.kind == OUT_F32_NCHW && bw % 4 == 0 && o.w % 4 == 0))) {
        for (size_t ci = 0; ci < classes.size(); ci++)
          p.omap[ci] = out_map_f32(o.p, o.kind == OUT_F32_NCHW, B, o.c, o.h, o.w, bw);
        p.ostore = o.kind == OUT_F32_NCHW ? 2 : 3;
      }
      p.obox_w = std::min(bw, 32);
    }
    op.grid = pair ? 2 * std::min(p.total_tiles, clusters) : std::min(p.total_tiles, sms);
    // Launches of a few tiles per slot whose tiles differ in K (classes of
    // different K, split-K parts) get a static longest-first schedule: round
    // robin would leave some slots with a long tile more than others.
    {
      const int nslot = pair ? op.grid / 2 : op.grid;
      std::vector<int> cost(p.total_tiles);
      for (int t = 0; t < p.total_tiles; t++) {
        int c = 0;
        while (c + 1 < p.nclass && t >= p.cls[c + 1].tile0) c++;
        const GemmClass& C = p.cls[c];
        const int part = C.part0 + (t - C.tile0) % C.nparts;
        int kb = 0;
        for (int u = C.kcut[part]; u < C.kcut[part + 1]; u++) kb += unit_kb[c][u];
        cost[t] = kb + 4;  // + the epilogue, about four K blocks' time
      }
      bool uneven = p.total_tiles % nslot != 0;
      for (int t = 1; t < p.total_tiles; t++) uneven = uneven || cost[t] != cost[0];
      bool grouped = class_groups && p.nclass > 1;
      for (int c = 0; c < p.nclass && grouped; c++)
        grouped = p.cls[c].nparts == 1 && p.cls[c].ntiles_n == p.cls[0].ntiles_n;
      std::vector<std::vector<int>> lists;
      if (grouped) {
        // every class's tile of one (pixel tile, N tile) on the same slot,
        // one after another: classes that read the same input rows (the
        // phases of a transposed convolution) find them in L2
        lists.assign(nslot, {});
        const long long ngroups = mt_sched * p.cls[0].ntiles_n;
        for (long long g = 0; g < ngroups; g++)
          for (int c = 0; c < p.nclass; c++) lists[(size_t)(g % nslot)].push_back(p.cls[c].tile0 + (int)g);
      } else if (uneven && p.total_tiles <= 16 * nslot) {
        std::vector<int> order(p.total_tiles);
        for (int t = 0; t < p.total_tiles; t++) order[t] = t;
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost[a] > cost[b]; });
        std::vector<long long> load(nslot, 0);
        lists.assign(nslot, {});
        for (int t : order) {
          int best = 0;
          for (int sl = 1; sl < nslot; sl++)
            if (load[sl] < load[best]) best = sl;
          load[best] += cost[t];
          lists[best].push_back(t);
        }
      }
      if (!lists.empty()) {
        std::vector<int> h_off(nslot + 1, 0), h_sched;
        for (int sl = 0; sl < nslot; sl++) {
          h_sched.insert(h_sched.end(), lists[sl].begin(), lists[sl].end());
          h_off[sl + 1] = (int)h_sched.size();
        }
        int* d = (int*)pl.mem.alloc((h_sched.size() + h_off.size()) * sizeof(int), false);
        if (!pl.mem.dry) {
          CK(cudaMemcpy(d, h_off.data(), h_off.size() * sizeof(int), cudaMemcpyHostToDevice));
          CK(cudaMemcpy(d + h_off.size(), h_sched.data(), h_sched.size() * sizeof(int), cudaMemcpyHostToDevice));
        }
        p.sched_off = d;
        p.sched = d + h_off.size();
      }
    }
    op.out_ptr = o.p;
    op.out_split = o.kind == OUT_SPLIT;
    op.out_part = o.part;
    if (o.kind == OUT_F32_NCHW) {
      op.dims[0] = B; op.dims[1] = o.c; op.dims[2] = o.h; op.dims[3] = o.w;
    } else {
      op.dims[0] = B; op.dims[1] = o.h + 2 * o.halo; op.dims[2] = o.w + 2 * o.halo; op.dims[3] = o.c;
    }
    if (tail_class < 0) {
      pl.ops.push_back(std::move(op));
      return;
    }
    // the tail launch: the tail class alone, its last part, same workspace slices
    Op tl;
    tl.kind = OP_GEMM;
    tl.name = name;
    tl.bn = op.bn;
    tl.flops = tail_flops;
    op.flops -= tail_flops;
    tl.g.reset(new GemmParams(p));
    GemmParams& q = *tl.g;
    q.sched = nullptr;  // one class of equal tiles: round robin
    q.sched_off = nullptr;
    q.nclass = 1;
    q.cls[0] = p.cls[tail_class];
    q.cls[0].part0 = q.cls[0].ksplit - 1;
    q.cls[0].nparts = 1;
    q.cls[0].tile0 = 0;
    q.bmap[0] = p.bmap[tail_class];
    q.omap[0] = p.omap[tail_class];
    q.total_tiles = (int)mt_sched * q.cls[0].ntiles_n;
    tl.grid = pair ? 2 * std::min(q.total_tiles, clusters) : std::min(q.total_tiles, sms);
    tl.ws_floats = op.ws_floats;
    tl.ws_counters = op.ws_counters;
    tl.out_ptr = op.out_ptr;
    tl.out_split = op.out_split;
    tl.out_part = op.out_part;
    for (int i = 0; i < 4; i++) tl.dims[i] = op.dims[i];
    pl.ops.push_back(std::move(op));
    pl.ops.push_back(std::move(tl));
  }

  static OutSpec split_out(const Act& a, const void* skip = nullptr) {
    return OutSpec{OUT_SPLIT, a.p, a.part(), a.C, a.H, a.W, a.halo, a.halo > 0 ? 1 : 0, skip};
  }

  static std::vector<std::pair<int, int>> square_taps(int k, int off) {
    std::vector<std::pair<int, int>> t;
    for (int ky = 0; ky < k; ky++)
      for (int kx = 0; kx < k; kx++) t.push_back({ky + off, kx + off});
    return t;
  }

  float2* twiddles(int n) {
    std::vector<float2> t(n);
    for (int k = 0; k < n; k++) {
      double a = 2.0 * M_PI * (double)k / (double)n;
      t[k] = make_float2((float)std::cos(a), (float)std::sin(a));
    }
    float2* d = (float2*)pl.mem.alloc((size_t)n * sizeof(float2), false);
    if (!pl.mem.dry) CK(cudaMemcpy(d, t.data(), (size_t)n * sizeof(float2), cudaMemcpyHostToDevice));
    return d;
  }

  static int log2_or_neg(int n) {
    if (n <= 0 || (n & (n - 1))) return -1;
    int l = 0;
    while ((1 << l) < n) l++;
    return l;
  }

  // Resblock stack on XA (in place), using XB / spectral scratch.
  void resblocks(const Act& XA, const Act& XB, int nblocks) {
    const int B = XA.B, h = XA.H, w = XA.W, wh = w / 2 + 1;
    float* feat = (float*)pl.mem.alloc((size_t)B * h * w * 192 * 4);
    Act spec{};
    spec.B = B; spec.H = 1; spec.W = h * wh; spec.C = 384; spec.halo = 0;
    spec.p = pl.mem.alloc(spec.bytes());
    float* fu = (float*)pl.mem.alloc((size_t)B * h * wh * 384 * 4);
    Act S = act(B, h, w, 192, 0);
    FftParams fp{};
    fp.batch = B; fp.c = 192; fp.h = h; fp.w = w; fp.wh = wh;
    fp.log2h = log2_or_neg(h); fp.log2w = log2_or_neg(w);
    fp.scale = (float)(1.0 / std::sqrt((double)h * (double)w));
    fp.tw_h = twiddles(h);
    fp.tw_w = twiddles(w);
    fp.feat = feat;
    fp.spec = spec.p;
    fp.spec_part = spec.part();
    fp.fu = fu;
    fp.s_out = S.p;
    fp.s_part = S.part();
    if (!fft_tiles(fp, kFftSmem))
      throw EngineError{LAMA_EUNSUPPORTED, "latent plane " + std::to_string(h) + "x" + std::to_string(w) +
                                               " needs more shared memory than the spectral kernels have"};
    fp.err = e.d_err;
    const bool reg = fft_reg_supported(h, w) && use_reg_fft();
    if (!reg) fp.tmp = (float2*)pl.mem.alloc(fft_tmp_elems(fp) * sizeof(float2));
    // the prefetching rfft2 beats the register one at batch 1, 8 and 32 (64x64 planes)
    // the tensor-core rfft2 beats the prefetching one from 8 images up (64x64
    // planes, per pass of 36 launches: 8.2 -> 6.0 ms at 64 images, 1.8 -> 1.7
    // at 16, 1.07 -> 1.05 at 8); below that its per-CTA set-up (TMEM, the 80 KB
    // DFT table) makes it slower (0.75 -> 0.83 ms at 4, 0.55 -> 0.79 at 1)
    const bool tc = (e.spectral == LAMA_SPECTRAL_TENSOR || (e.spectral == LAMA_SPECTRAL_AUTO && B >= 8)) &&
                    fft_tc_supported(192, h, w);
    const bool pf = (e.spectral == LAMA_SPECTRAL_PREFETCH || e.spectral == LAMA_SPECTRAL_AUTO || tc) &&
                    fft_pf_supported(192, h, w);
    CUtensorMap feat_map{}, feat_map_tc{};
    const void* tc_tab = nullptr;
    if (tc) {
      // feat as rows of 64 floats, boxes of 32 floats x 128 rows (2 channels' x-halves)
      cuuint64_t dims[2] = {64, (cuuint64_t)B * 192 * 64};
      cuuint64_t strides[1] = {256};
      cuuint32_t box[2] = {32, 128};
      cuuint32_t estr[2] = {1, 1};
      CUresult r = encode_tiled(&feat_map_tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, feat, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS)
        throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled (feat rows, 128) failed: " + std::to_string((int)r)};
      std::vector<uint8_t> tab(fft_tc_table_bytes());
      fft_tc_table(tab.data());
      void* d = pl.mem.alloc(tab.size(), false);
      if (!pl.mem.dry) CK(cudaMemcpy(d, tab.data(), tab.size(), cudaMemcpyHostToDevice));
      tc_tab = d;
    }
    if (pf && !tc) {
      // feat as rows of 64 floats, boxes of 32 floats x 256 rows (4 channels' x-halves)
      cuuint64_t dims[2] = {64, (cuuint64_t)B * 192 * 64};
      cuuint64_t strides[1] = {256};
      cuuint32_t box[2] = {32, 256};
      cuuint32_t estr[2] = {1, 1};
      CUresult r = encode_tiled(&feat_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, feat, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS)
        throw EngineError{LAMA_ECUDA, "cuTensorMapEncodeTiled (feat rows) failed: " + std::to_string((int)r)};
    }
    const double px = (double)B * h * w, pxs = (double)B * h * wh;
    // Small batches run each FFC layer on two graph lanes: the spectral chain
    // (conv1, rfft2, FourierUnit conv, irfft2: short launches of a few dozen
    // CTAs each) on `chain` SMs, concurrently with the part of the FFC GEMM
    // that does not need its result (the local class, and the l2g segment of
    // the global class as split-K parts) on the other SMs; a tail launch then
    // adds the conv2 segment over S and finishes the global class.
    const int chain = lanes_for(B, h, w);
    int prev0 = (int)pl.ops.size() - 1;  // last lane-0 op before the stack
    auto on_lane1 = [&](int wait_for) {
      if (!chain) return;
      pl.ops.back().lane = 1;
      if (wait_for >= 0) pl.ops.back().waits.push_back(wait_for);
    };
    for (int blk = 0; blk < nblocks; blk++)
      for (int sub = 0; sub < 2; sub++) {
        const FfcW& F = e.W.ffc[(size_t)blk * 2 + sub];
        const Act& Xin = sub == 0 ? XA : XB;
        const Act& Xout = sub == 0 ? XB : XA;
        // conv1 1x1 384 -> 192 on the global channels, BN, ReLU -> feat (fp32)
        gemm("spectral_conv1", F.conv1, {{Xin, 1, false}}, {one_seg(0, 0, 192, SegSpec{0, 128, 384, 1, {{1, 1}}})}, 64, B, h, w,
             OutSpec{OUT_F32_NCHW, feat, 0, 192, h, w, 0, 0, nullptr}, 1, 0, 2.0 * px * 192 * 384, chain);
        on_lane1(prev0);
        Op r;
        r.kind = tc ? OP_RFFT_TC : pf ? OP_RFFT_PF : reg ? OP_RFFT_REG : OP_RFFT;
        r.name = "rfft2";
        r.f = fp;
        if (tc) {
          r.ftc.reset(new FftTcParams{feat_map_tc, fp, tc_tab});
          r.grid = std::min(B * 192 / 4, chain ? chain : e.sms);  // one CTA per SM
        } else if (pf) {
          r.fpf.reset(new FftPfParams{feat_map, fp});
          r.grid = std::min(B * 192 / 4, 2 * (chain ? chain : e.sms));  // two CTAs per SM
        }
        r.bytes = px * 192 * 4 + pxs * 384 * 4;
        r.out_ptr = spec.p; r.out_split = 1; r.out_part = spec.part();
        r.dims[0] = B; r.dims[1] = h; r.dims[2] = wh; r.dims[3] = 384;
        pl.ops.push_back(std::move(r));
        on_lane1(-1);
        // FourierUnit 1x1 384 -> 384 on the stacked spectrum, BN, ReLU -> fu (fp32)
        gemm("fourier_conv", F.fu, {{spec, 1, false}}, {one_seg(0, 0, 384, SegSpec{0, 0, 384, 1, {{0, 0}}})}, 64, B, 1, h * wh,
             OutSpec{OUT_F32_NHWC, fu, 0, 384, 1, h * wh, 0, 0, nullptr}, 1, 0, 2.0 * pxs * 384 * 384, chain);
        on_lane1(-1);
        Op ir;
        ir.kind = pf ? OP_IRFFT_PAR : reg ? OP_IRFFT_REG : OP_IRFFT;
        ir.name = "irfft2";
        ir.f = fp;
        ir.grid = e.sms;  // OP_IRFFT_PAR: picks its channels per CTA from the SM count
        ir.bytes = pxs * 384 * 4 + px * 192 * 4 + px * 192 * 4;
        ir.out_ptr = S.p; ir.out_split = 1; ir.out_part = S.part();
        ir.dims[0] = B; ir.dims[1] = h; ir.dims[2] = w; ir.dims[3] = 192;
        pl.ops.push_back(std::move(ir));
        on_lane1(-1);
        const int i_irfft = (int)pl.ops.size() - 1;
        // FFC outputs: local = 3x3 over [x_l | x_g]; global = 3x3 over x_l + 1x1 over S
        ClassSpec cl{0, 0, 128};
        cl.segs.push_back({0, 0, 512, 1, square_taps(3, 0)});
        ClassSpec cgl{1, 128, 384};
        cgl.segs.push_back({0, 0, 128, 1, square_taps(3, 0)});
        cgl.segs.push_back({1, 0, 192, 1, {{0, 0}}});
        // (two lanes: measured faster than running the whole global class
        // after the chain, 3.73 vs 4.13 ms per batch-1 512x512 pass)
        gemm("ffc_out", F.out, {{Xin, 1, false}, {S, 1, false}}, {cl, cgl}, 64, B, h, w,
             split_out(Xout, sub == 1 ? XA.p : nullptr), 1, 0, 2.0 * px * (128.0 * 4608 + 384.0 * 1344),
             chain ? e.sms - chain : 0, chain ? 1 : -1, 2.0 * px * 384.0 * 192);
        if (chain) pl.ops.back().waits.push_back(i_irfft);  // the tail launch reads S
        prev0 = (int)pl.ops.size() - 1;
      }
  }

  // comp: the u8 path's composite, fused into the OutConv (out is then unused)
  // win: one --sections pass, fill written into the working image (out unused)
  void core(const Act& U, int B, int H, int W, float* out, const CompositeParams* comp = nullptr,
            const WinDesc* win = nullptr) {
    const int h2 = H / 2, w2 = W / 2, h4 = H / 4, w4 = W / 4, h8 = H / 8, w8 = W / 8;
    Act X1 = act(B, H, W, 64, 1);
    Act X2 = act(B, h2, w2, 128, 1);
    Act X3 = act(B, h4, w4, 256, 1);
    Act XA = act(B, h8, w8, 512, 1);
    Act XB = act(B, h8, w8, 512, 1);
    // model.1: 7x7 valid over the pad-3 input: 8 row taps (the 8th has zero weights)
    {
      ClassSpec c{0, 0, 64};
      std::vector<std::pair<int, int>> t;
      for (int ky = 0; ky < 8; ky++) t.push_back({ky, 0});
      c.segs.push_back({0, 0, 32, 1, t});
      gemm("model1_7x7", e.W.m1, {{U, 1, false}}, {c}, 32, B, H, W, split_out(X1), 1, 0,
           2.0 * B * H * W * 64 * 196);
    }
    // model.2 .. model.4: 3x3 stride 2, reflect pad 1 (the halo)
    {
      ClassSpec c{0, 0, 128};
      c.segs.push_back({0, 0, 64, 2, square_taps(3, 0)});
      gemm("model2_3x3s2", e.W.m2, {{X1, 2, false}}, {c}, 64, B, h2, w2, split_out(X2), 1, 0,
           2.0 * B * h2 * w2 * 128 * 576);
    }
    {
      ClassSpec c{0, 0, 256};
      c.segs.push_back({0, 0, 128, 2, square_taps(3, 0)});
      gemm("model3_3x3s2", e.W.m3, {{X2, 2, false}}, {c}, 64, B, h4, w4, split_out(X3), 1, 0,
           2.0 * B * h4 * w4 * 256 * 1152);
    }
    {
      ClassSpec c{0, 0, 512};
      c.segs.push_back({0, 0, 256, 2, square_taps(3, 0)});
      gemm("model4_3x3s2", e.W.m4, {{X3, 2, false}}, {c}, 64, B, h8, w8, split_out(XA), 1, 0,
           2.0 * B * h8 * w8 * 512 * 2304);
    }
    resblocks(XA, XB, 18);
    // decoder: three ConvTranspose2d + BN + ReLU as phase GEMMs, Concat is XA itself
    static const int taps[4][4][2] = {{{0, 0}}, {{0, 1}, {0, 0}}, {{1, 0}, {0, 0}}, {{1, 1}, {1, 0}, {0, 1}, {0, 0}}};
    static const int ntaps[4] = {1, 2, 2, 4};
    Act U1 = act(B, 2 * h8, 2 * w8, 256, 0);
    Act U2 = act(B, 4 * h8, 4 * w8, 128, 0);
    Act U3 = act(B, H, W, 64, 3);
    const Act ins[3] = {XA, U1, U2};
    const Act outs[3] = {U1, U2, U3};
    const char* names[3] = {"convT1", "convT2", "convT3"};
    for (int u = 0; u < 3; u++) {
      const Act& in = ins[u];
      const int cout = outs[u].C;
      std::vector<ClassSpec> cls;
      for (int ph = 0; ph < 4; ph++) {
        ClassSpec c{ph, 0, cout, 2, ph / 2, 2, ph % 2};
        std::vector<std::pair<int, int>> t;
        for (int ti = 0; ti < ntaps[ph]; ti++) t.push_back({taps[ph][ti][0], taps[ph][ti][1]});
        c.segs.push_back({0, 0, in.C, 1, t});
        cls.push_back(c);
      }
      gemm(names[u], e.W.ct[u], {{in, 1, true}}, cls, 64, B, in.H, in.W, split_out(outs[u]), 1, 0,
           2.0 * B * in.H * in.W * cout * in.C * 9, 0, -1, 0, kConvTClassGroups && u > 0);
    }
    // OutConv 7x7 64 -> 3 over the reflect-pad-3 halo, + bias, sigmoid -> fp32 NCHW:
    // all 147 tap products of each input row at once, summed in a ring of
    // output rows (outconv.cu), every input row read once
    {
      Op op;
      op.kind = OP_OUTCONV;
      op.name = "outconv_7x7";
      op.flops = 2.0 * B * H * W * 3 * 3136;
      op.oc.reset(new OutConvParams());
      OutConvParams& q = *op.oc;
      q.amap = act_map(U3, 64, 32, 1, 1, false);  // 32-column boxes, four per row and part
      q.wmap = w_map(e.W.outc.cls[0], 160);
      q.bias = e.W.outc.shift;
      q.out = out;
      q.win = win;
      if (comp) {
        q.mask = comp->mask;
        q.dst = comp->dst;
        q.ih = comp->h;
        q.iw = comp->w;
      }
      q.batch = B;
      q.h = H;
      q.w = W;
      q.err = e.d_err;
      outconv_units(q, e.sms);
      op.grid = e.sms;
      op.out_ptr = out;
      op.out_split = 0;
      op.dims[0] = B; op.dims[1] = 3; op.dims[2] = H; op.dims[3] = W;
      pl.ops.push_back(std::move(op));
    }
  }
};

// Events destroyed on every exit path, the error ones included.
struct EventSet {
  std::vector<cudaEvent_t> ev;
  explicit EventSet(size_t n) : ev(n, nullptr) {}
  ~EventSet() {
    for (cudaEvent_t x : ev)
      if (x) cudaEventDestroy(x);
  }
};

void check_device_error(lama_engine* e) {
  int v = 0;
  CK(cudaMemcpy(&v, e->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) {
    cudaMemset(e->d_err, 0, sizeof(int));
    throw EngineError{LAMA_EDEVICE, "a kernel wait timed out on the device (code " + std::to_string(v) + ")"};
  }
}

// Every launch of a pass and the device memory it needs (all but the graph).
void build_plan(lama_engine* e, Plan* pl) {
  Builder b{*e, *pl};
  b.build_ops();
  // Programmatic dependent launch (a kernel's set-up overlapping the end of
  // the previous one) is off: measured on one B200 it made the batch-1
  // 512x512 pass slower (3.71 -> 4.14 ms, graph replay) and a 64-image pass
  // too (93.2 -> 97.0 ms).  LAMA_PDL=1 turns it on for experiments.
  {
    static const bool pdl = [] {
      const char* v = std::getenv("LAMA_PDL");
      return v && std::atoi(v) == 1;
    }();
    for (Op& op : pl->ops) op.pdl = pdl && op.kind != OP_COPY;
  }
  // one split-K workspace per lane, sized for its largest GEMM
  size_t wsf[2] = {0, 0};
  int wsc[2] = {0, 0};
  for (const Op& op : pl->ops) {
    wsf[op.lane] = std::max(wsf[op.lane], op.ws_floats);
    wsc[op.lane] = std::max(wsc[op.lane], op.ws_counters);
  }
  for (int l = 0; l < 2; l++) {
    if (!wsc[l]) continue;
    float* ws = (float*)pl->mem.alloc(wsf[l] * sizeof(float), false);
    int* cnt = (int*)pl->mem.alloc((size_t)wsc[l] * sizeof(int));  // zeroed; reset by each tile's finisher
    for (Op& op : pl->ops)
      if (op.kind == OP_GEMM && op.lane == l && op.ws_counters) {
        op.g->ws = ws;
        op.g->cnt = cnt;
      }
  }
}

void Builder::build_ops() {
  const int kind = pl.kind, B = pl.B, H = pl.H, W = pl.W, h = pl.h, w = pl.w, nblocks = pl.nblocks;
  Plan* const pl_ = &pl;
  Builder& b = *this;
  if (kind == 0 || kind == 1 || kind == 3) {
    Act U = b.act(B, H + 6, W, 32, 0);
    if (kind == 0) pl_->out = (float*)pl_->mem.alloc((size_t)B * 3 * H * W * 4);
    Op un;
    un.name = "unfold_input";
    un.u.batch = B; un.u.H = H; un.u.W = W; un.u.h = h; un.u.w = w;
    un.u.out = U.p;
    un.u.out_part = U.part();
    un.out_ptr = U.p; un.out_split = 1; un.out_part = U.part();
    un.dims[0] = B; un.dims[1] = H + 6; un.dims[2] = W; un.dims[3] = 32;
    if (kind == 0) {
      pl_->in_f32 = (float*)pl_->mem.alloc((size_t)B * 4 * H * W * 4);
      un.kind = OP_UNFOLD_F32;
      un.u.in = pl_->in_f32;
    } else if (kind == 3) {
      pl_->win = (WinDesc*)pl_->mem.alloc(sizeof(WinDesc));
      un.kind = OP_UNFOLD_U8;
      un.u.win = pl_->win;
    } else {
      pl_->rgb = (uint8_t*)pl_->mem.alloc((size_t)B * h * w * 3);
      pl_->mask = (uint8_t*)pl_->mem.alloc((size_t)B * h * w);
      pl_->out_rgb = (uint8_t*)pl_->mem.alloc((size_t)B * h * w * 3);
      un.kind = OP_UNFOLD_U8;
      un.u.rgb = pl_->rgb;
      un.u.mask = pl_->mask;
    }
    pl_->ops.push_back(std::move(un));
    if (kind == 1) {
      // the composite's unmasked bytes are the source bytes: copied whole
      // here, and the OutConv writes only the masked pixels
      Op cp;
      cp.kind = OP_COPY;
      cp.name = "copy_source";
      cp.csrc = pl_->rgb;
      cp.cdst = pl_->out_rgb;
      cp.cbytes = (size_t)B * h * w * 3;
      pl_->ops.push_back(std::move(cp));
      const CompositeParams comp{B, h, w, H, W, pl_->rgb, pl_->mask, pl_->out_rgb};
      b.core(U, B, H, W, nullptr, &comp);
    } else if (kind == 3) {
      const CompositeParams comp{B, h, w, H, W, nullptr, nullptr, nullptr};
      b.core(U, B, H, W, nullptr, &comp, pl_->win);
    } else {
      b.core(U, B, H, W, pl_->out);
    }
  } else {
    Act XA = b.act(B, H, W, 512, 1);
    Act XB = b.act(B, H, W, 512, 1);
    pl_->l_in = (float*)pl_->mem.alloc((size_t)B * 128 * H * W * 4);
    pl_->g_in = (float*)pl_->mem.alloc((size_t)B * 384 * H * W * 4);
    pl_->l_out = (float*)pl_->mem.alloc((size_t)B * 128 * H * W * 4);
    pl_->g_out = (float*)pl_->mem.alloc((size_t)B * 384 * H * W * 4);
    for (int i = 0; i < 2; i++) {
      Op cv;
      cv.kind = OP_TO_SPLIT;
      cv.name = "nchw_to_split";
      cv.cv = ConvertParams{B, i == 0 ? 128 : 384, H, W, 1, 512, i == 0 ? 0 : 128, i == 0 ? pl_->l_in : pl_->g_in,
                            XA.p, XA.part()};
      pl_->ops.push_back(std::move(cv));
    }
    b.resblocks(XA, XB, nblocks);
    for (int i = 0; i < 2; i++) {
      Op cv;
      cv.kind = OP_TO_NCHW;
      cv.name = "split_to_nchw";
      cv.cv = ConvertParams{B, i == 0 ? 128 : 384, H, W, 1, 512, i == 0 ? 0 : 128,
                            i == 0 ? pl_->l_out : pl_->g_out, XA.p, XA.part()};
      pl_->ops.push_back(std::move(cv));
    }
  }
}

// Device bytes of a plan, from a dry build (the same code, no allocation).
size_t plan_bytes_dry(lama_engine* e, int kind, int B, int H, int W, int h, int w, int nblocks) {
  struct DryBuild {
    DryBuild() { t_dry_build = true; }
    ~DryBuild() { t_dry_build = false; }
  } dry;
  Plan pl;
  pl.kind = kind; pl.B = B; pl.H = H; pl.W = W; pl.h = h; pl.w = w; pl.nblocks = nblocks;
  pl.mem.dry = true;
  build_plan(e, &pl);
  return pl.mem.total;
}

std::string human_bytes(double b) {
  char buf[32];
  if (b >= (double)(1ull << 30)) snprintf(buf, sizeof(buf), "%.1f GB", b / (double)(1ull << 30));
  else snprintf(buf, sizeof(buf), "%.0f MB", b / (double)(1ull << 20));
  return buf;
}

// Capture a plan's pass into an instantiated CUDA graph: lane 1 forks off the
// engine stream at its first op and joins back after its last, cross-lane
// waits become graph edges through events.  With `stamps` (ops + 1 timing
// events), the graph also records stamps[0] before the first op and
// stamps[i + 1] after op i on its lane (external event-record nodes), for
// lama_profile_timeline.
cudaGraphExec_t capture_plan(lama_engine* e, const Plan& pl, std::vector<cudaEvent_t>* stamps) {
  cudaGraph_t graph = nullptr;
  bool two_lanes = false;
  for (const Op& op : pl.ops) two_lanes = two_lanes || op.lane == 1;
  EventSet done(two_lanes ? pl.ops.size() + 1 : 0);
  for (auto& x : done.ev) CK(cudaEventCreateWithFlags(&x, cudaEventDisableTiming));
  std::vector<char> waited(pl.ops.size(), 0);
  for (const Op& op : pl.ops)
    for (int j : op.waits) waited[(size_t)j] = 1;
  CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  int lerr = 0;
  const cudaStream_t lane_stream[2] = {e->stream, e->side_stream};
  if (stamps) lerr = (int)cudaEventRecordWithFlags((*stamps)[0], e->stream, cudaEventRecordExternal);
  if (two_lanes && !lerr) {  // the side stream joins the capture from the engine stream
    lerr = (int)cudaEventRecord(done.ev.back(), e->stream);
    if (!lerr) lerr = (int)cudaStreamWaitEvent(e->side_stream, done.ev.back(), 0);
  }
  for (size_t i = 0; i < pl.ops.size() && !lerr; i++) {
    const Op& op = pl.ops[i];
    const cudaStream_t st = lane_stream[two_lanes ? op.lane : 0];
    for (int j : op.waits)
      if (!lerr && two_lanes) lerr = (int)cudaStreamWaitEvent(st, done.ev[(size_t)j], 0);
    if (!lerr) lerr = launch_op(op, st);
    if (!lerr && two_lanes && waited[i]) lerr = (int)cudaEventRecord(done.ev[i], st);
    if (!lerr && stamps) lerr = (int)cudaEventRecordWithFlags((*stamps)[i + 1], st, cudaEventRecordExternal);
  }
  if (two_lanes && !lerr) {  // join: the engine stream waits for the side stream's last op
    lerr = (int)cudaEventRecord(done.ev.back(), e->side_stream);
    if (!lerr) lerr = (int)cudaStreamWaitEvent(e->stream, done.ev.back(), 0);
  }
  cudaError_t ce = cudaStreamEndCapture(e->stream, &graph);
  if (lerr) {
    if (graph) cudaGraphDestroy(graph);
    throw EngineError{LAMA_ECUDA, std::string("kernel launch during capture: ") + cudaGetErrorString((cudaError_t)lerr)};
  }
  CK(ce);
  cudaGraphExec_t exec = nullptr;
  cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  CK(ie);
  return exec;
}

Plan& get_plan(lama_engine* e, int kind, int B, int H, int W, int h, int w, int nblocks) {
  auto key = std::make_tuple(kind, B, H, W, h, w, nblocks);
  auto it = e->plans.find(key);
  if (it != e->plans.end()) return *it->second;
  // Capacity guard (lama-rs/src/mem.rs:49-73): refuse a pass the device
  // cannot hold before anything is allocated, keeping the reference's 10 %
  // headroom of free memory.  The estimate is the plan's exact footprint.
  {
    const size_t need = plan_bytes_dry(e, kind, B, H, W, h, w, nblocks);
    size_t free_b = 0, total_b = 0;
    CK(cudaMemGetInfo(&free_b, &total_b));
    if (need > free_b - free_b / 10)
      throw EngineError{LAMA_ENOMEM, "an inference over " + std::to_string(W) + "x" + std::to_string(H) +
                                         (B > 1 ? " (batch " + std::to_string(B) + ")" : std::string()) +
                                         " needs about " + human_bytes((double)need) +
                                         " of device memory, but only " + human_bytes((double)free_b) +
                                         " is free of " + human_bytes((double)total_b) + " on \"" + e->gpu_name +
                                         "\""};
  }
  std::unique_ptr<Plan> pl(new Plan());
  pl->kind = kind; pl->B = B; pl->H = H; pl->W = W; pl->h = h; pl->w = w; pl->nblocks = nblocks;
  build_plan(e, pl.get());
  pl->exec = capture_plan(e, *pl, nullptr);
  Plan& ref = *pl;
  e->plans[key] = std::move(pl);
  return ref;
}

void run_plan(lama_engine* e, Plan& pl) { CK(cudaGraphLaunch(pl.exec, e->stream)); }

void sync_check(lama_engine* e) {
  CK(cudaStreamSynchronize(e->stream));
  check_device_error(e);
}

template <class F>
int guarded(lama_engine* e, F&& f) {
  if (!e) return LAMA_EINVAL;
  try {
    if (!e->stream) throw EngineError{LAMA_EINVAL, "engine was not opened successfully"};
    CK(cudaSetDevice(e->device));
    cudaGetLastError();  // a pending error from an earlier, unrelated call must not be reported here
    f();
    e->err.clear();
    return LAMA_OK;
  } catch (const EngineError& x) {
    e->err = x.msg;
    return x.code;
  } catch (const std::exception& x) {
    e->err = x.what();
    return LAMA_EINVAL;
  }
}

void check_shape(int batch, int h, int w, bool mult8) {
  if (batch < 1 || h < 1 || w < 1) throw EngineError{LAMA_EINVAL, "batch, h and w must be positive"};
  if (mult8 && (h % 8 || w % 8))
    throw EngineError{LAMA_EINVAL, "h and w must be multiples of 8 (the generator has three stride-2 stages)"};
}

// An op launched on its own (profiling and debug runs, not the captured
// graph).  With LAMA_NVTX set in the environment it runs inside an NVTX range
// named after the op, so a profiler can pick layers out
// (`LAMA_NVTX=1 ncu --nvtx --nvtx-include "ffc_out/" ...`); without it no NVTX
// call is made.
int launch_named(const Op& op, cudaStream_t st) {
  static const bool nvtx = std::getenv("LAMA_NVTX") != nullptr;
  if (!nvtx) return launch_op(op, st);
  nvtxRangePushA(op.name.c_str());
  const int r = launch_op(op, st);
  nvtxRangePop();
  return r;
}

}  // namespace

extern "C" {

int lama_abi_version(void) { return 1; }

int lama_open(const char* weights_path, int device, lama_engine** out) {
  if (!out) return LAMA_EINVAL;
  *out = nullptr;
  lama_engine* e = new lama_engine();
  e->device = device;
  *out = e;
  if (!weights_path) {
    e->err = "weights path is null";
    return LAMA_EINVAL;
  }
  try {
    WeightFile wf;
    std::string err;
    if (!wf.open(weights_path, err)) throw EngineError{LAMA_EWEIGHTS, err};
    load_weights(wf, e->W);
    check_weight_shapes(e->W);
  } catch (const EngineError& x) {
    e->err = x.msg;
    return x.code;
  }
  try {
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev)
      throw EngineError{LAMA_EINVAL, "device " + std::to_string(device) + " does not exist (" + std::to_string(ndev) +
                                         " visible)"};
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw EngineError{LAMA_EUNSUPPORTED, std::string("this engine is built for sm_100a (B200); device is ") +
                                               prop.name + " sm_" + std::to_string(prop.major) +
                                               std::to_string(prop.minor)};
    e->sms = prop.multiProcessorCount;
    e->gpu_name = prop.name;
    CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&e->side_stream, cudaStreamNonBlocking));
    CKL(conv_gemm_prepare());
    e->pair_clusters = conv_gemm_pair_clusters();
    CKL(fft_prepare(kFftSmem));
    CKL(fft_reg_prepare());
    CKL(fft_pf_prepare());
    CKL(fft_tc_prepare());
    CKL(outconv_prepare());
    e->d_err = (int*)e->wmem.alloc(256);
    upload_weights(e->W, e->wmem);
  } catch (const EngineError& x) {
    e->err = x.msg;
    return x.code;
  }
  e->err.clear();
  return LAMA_OK;
}

int lama_forward(lama_engine* e, const float* in, int batch, int h, int w, float* out) {
  return guarded(e, [&] {
    if (!in || !out) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, true);
    Plan& pl = get_plan(e, 0, batch, h, w, h, w, 18);
    const size_t nin = (size_t)batch * 4 * h * w, nout = (size_t)batch * 3 * h * w;
    CK(cudaMemcpyAsync(pl.in_f32, in, nin * 4, cudaMemcpyHostToDevice, e->stream));
    run_plan(e, pl);
    CK(cudaMemcpyAsync(out, pl.out, nout * 4, cudaMemcpyDeviceToHost, e->stream));
    sync_check(e);
  });
}

int lama_forward_device(lama_engine* e, const float* d_in, int batch, int h, int w, float* d_out) {
  return guarded(e, [&] {
    if (!d_in || !d_out) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, true);
    Plan& pl = get_plan(e, 0, batch, h, w, h, w, 18);
    const size_t nin = (size_t)batch * 4 * h * w, nout = (size_t)batch * 3 * h * w;
    CK(cudaMemcpyAsync(pl.in_f32, d_in, nin * 4, cudaMemcpyDeviceToDevice, e->stream));
    run_plan(e, pl);
    CK(cudaMemcpyAsync(d_out, pl.out, nout * 4, cudaMemcpyDeviceToDevice, e->stream));
  });
}

int lama_inpaint_u8(lama_engine* e, const uint8_t* rgb, const uint8_t* mask, int batch, int h, int w,
                    uint8_t* out_rgb) {
  return guarded(e, [&] {
    if (!rgb || !mask || !out_rgb) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, false);
    const int H = (h + 7) / 8 * 8, W = (w + 7) / 8 * 8;
    Plan& pl = get_plan(e, 1, batch, H, W, h, w, 18);
    const size_t npx = (size_t)batch * h * w;
    CK(cudaMemcpyAsync(pl.rgb, rgb, npx * 3, cudaMemcpyHostToDevice, e->stream));
    CK(cudaMemcpyAsync(pl.mask, mask, npx, cudaMemcpyHostToDevice, e->stream));
    run_plan(e, pl);
    CK(cudaMemcpyAsync(out_rgb, pl.out_rgb, npx * 3, cudaMemcpyDeviceToHost, e->stream));
    sync_check(e);
  });
}

int lama_inpaint_u8_device(lama_engine* e, const uint8_t* d_rgb, const uint8_t* d_mask, int batch, int h, int w,
                           uint8_t* d_out_rgb) {
  return guarded(e, [&] {
    if (!d_rgb || !d_mask || !d_out_rgb) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, false);
    const int H = (h + 7) / 8 * 8, W = (w + 7) / 8 * 8;
    Plan& pl = get_plan(e, 1, batch, H, W, h, w, 18);
    const size_t npx = (size_t)batch * h * w;
    CK(cudaMemcpyAsync(pl.rgb, d_rgb, npx * 3, cudaMemcpyDeviceToDevice, e->stream));
    CK(cudaMemcpyAsync(pl.mask, d_mask, npx, cudaMemcpyDeviceToDevice, e->stream));
    run_plan(e, pl);
    CK(cudaMemcpyAsync(d_out_rgb, pl.out_rgb, npx * 3, cudaMemcpyDeviceToDevice, e->stream));
  });
}

int lama_inpaint_u8_stream(lama_engine* e, const uint8_t* rgb, const uint8_t* mask, int n, int h, int w, int chunk,
                           uint8_t* out_rgb) {
  return guarded(e, [&] {
    if (!rgb || !mask || !out_rgb) throw EngineError{LAMA_EINVAL, "null buffer"};
    if (n < 1 || chunk < 1) throw EngineError{LAMA_EINVAL, "n and chunk must be positive"};
    check_shape(std::min(n, chunk), h, w, false);
    const int H = (h + 7) / 8 * 8, W = (w + 7) / 8 * 8;
    const size_t px = (size_t)h * w;
    const size_t set = (size_t)chunk * px * 7;  // rgb + mask + out of one chunk
    if (!e->copy_stream) {
      CK(cudaStreamCreateWithFlags(&e->copy_stream, cudaStreamNonBlocking));
      for (int i = 0; i < 2; i++) {
        CK(cudaEventCreateWithFlags(&e->ev_in[i], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&e->ev_done[i], cudaEventDisableTiming));
      }
    }
    if (e->pipe_bytes < set) {
      sync_check(e);
      CK(cudaStreamSynchronize(e->copy_stream));
      e->pipe_mem.free_all();
      e->pipe_bytes = set;
      for (int i = 0; i < 2; i++) e->pipe_buf[i] = (uint8_t*)e->pipe_mem.alloc(set, false);
    }
    // Copy stream: H2D(0), H2D(1), D2H(0), H2D(2), D2H(1), ...; engine stream:
    // per chunk staging -> plan, the pass, plan -> staging.  So chunk i + 1's
    // upload and chunk i - 1's download run while chunk i is in the pass.
    // Staging set i % 2 is refilled (H2D(i + 2)) only after D2H(i), which
    // the copy stream runs first; the pass of chunk i waits for H2D(i), which
    // the copy stream runs after D2H(i - 2), the set's previous reader.
    const int nchunks = (n + chunk - 1) / chunk;
    auto set_of = [&](int i, uint8_t*& srgb, uint8_t*& smask, uint8_t*& sout) {
      srgb = e->pipe_buf[i & 1];
      smask = srgb + (size_t)chunk * px * 3;
      sout = smask + (size_t)chunk * px;
    };
    auto upload = [&](int i) {
      uint8_t *srgb, *smask, *sout;
      set_of(i, srgb, smask, sout);
      const int b0 = i * chunk, cb = std::min(chunk, n - b0);
      CK(cudaMemcpyAsync(srgb, rgb + (size_t)b0 * px * 3, (size_t)cb * px * 3, cudaMemcpyHostToDevice, e->copy_stream));
      CK(cudaMemcpyAsync(smask, mask + (size_t)b0 * px, (size_t)cb * px, cudaMemcpyHostToDevice, e->copy_stream));
      CK(cudaEventRecord(e->ev_in[i & 1], e->copy_stream));
    };
    upload(0);
    for (int i = 0; i < nchunks; i++) {
      const int s = i & 1, b0 = i * chunk, cb = std::min(chunk, n - b0);
      uint8_t *srgb, *smask, *sout;
      set_of(i, srgb, smask, sout);
      Plan& pl = get_plan(e, 1, cb, H, W, h, w, 18);
      CK(cudaStreamWaitEvent(e->stream, e->ev_in[s], 0));
      CK(cudaMemcpyAsync(pl.rgb, srgb, (size_t)cb * px * 3, cudaMemcpyDeviceToDevice, e->stream));
      CK(cudaMemcpyAsync(pl.mask, smask, (size_t)cb * px, cudaMemcpyDeviceToDevice, e->stream));
      run_plan(e, pl);
      CK(cudaMemcpyAsync(sout, pl.out_rgb, (size_t)cb * px * 3, cudaMemcpyDeviceToDevice, e->stream));
      CK(cudaEventRecord(e->ev_done[s], e->stream));
      if (i + 1 < nchunks) upload(i + 1);
      CK(cudaStreamWaitEvent(e->copy_stream, e->ev_done[s], 0));
      CK(cudaMemcpyAsync(out_rgb + (size_t)b0 * px * 3, sout, (size_t)cb * px * 3, cudaMemcpyDeviceToHost,
                         e->copy_stream));
    }
    CK(cudaStreamSynchronize(e->copy_stream));
    sync_check(e);
  });
}

int lama_inpaint_sections_u8(lama_engine* e, const uint8_t* rgb, const uint8_t* mask, int w, int h, const int* rects,
                             int n, int side, uint8_t* out_rgb) {
  return guarded(e, [&] {
    if (!rgb || !mask || !out_rgb || (n > 0 && !rects)) throw EngineError{LAMA_EINVAL, "null buffer"};
    if (w < 1 || h < 1 || n < 0) throw EngineError{LAMA_EINVAL, "w, h must be positive and n non-negative"};
    const size_t npx = (size_t)w * h;
    if (n == 0) {
      memcpy(out_rgb, rgb, npx * 3);
      return;
    }
    if (side < 1 || side > std::min(w, h)) throw EngineError{LAMA_EINVAL, "side must be in 1..min(w, h)"};
    std::vector<WinDesc> d((size_t)n);
    for (int i = 0; i < n; i++) {
      const int* r = rects + 4 * i;
      if (r[0] < 0 || r[1] < 0 || r[2] > w || r[3] > h || r[0] >= r[2] || r[1] >= r[3])
        throw EngineError{LAMA_EINVAL, "section " + std::to_string(i) + " is not a non-empty rectangle inside the image"};
      const int wx0 = lama_window_origin((r[0] + r[2]) / 2, side, w), wy0 = lama_window_origin((r[1] + r[3]) / 2, side, h);
      if (r[0] < wx0 || r[1] < wy0 || r[2] > wx0 + side || r[3] > wy0 + side)
        throw EngineError{LAMA_EINVAL, "section " + std::to_string(i) + " does not fit its window"};
      d[i] = WinDesc{nullptr, nullptr, w, h, wx0, wy0, r[0], r[1], r[2], r[3]};
    }
    const int S = (side + 7) / 8 * 8;
    check_shape(1, side, side, false);
    Plan& pl = get_plan(e, 3, 1, S, S, side, side, 18);
    if (e->sec_px < npx || e->sec_n < (size_t)n) {  // grow the device-resident buffers
      sync_check(e);
      e->sec_mem.free_all();
      e->sec_px = std::max(e->sec_px, npx);
      e->sec_n = std::max(e->sec_n, (size_t)n);
      e->sec_img = (uint8_t*)e->sec_mem.alloc(e->sec_px * 3, false);
      e->sec_mask = (uint8_t*)e->sec_mem.alloc(e->sec_px, false);
      e->sec_desc = (WinDesc*)e->sec_mem.alloc(e->sec_n * sizeof(WinDesc), false);
    }
    for (auto& x : d) {
      x.img = e->sec_img;
      x.mask = e->sec_mask;
    }
    CK(cudaMemcpyAsync(e->sec_img, rgb, npx * 3, cudaMemcpyHostToDevice, e->stream));
    CK(cudaMemcpyAsync(e->sec_mask, mask, npx, cudaMemcpyHostToDevice, e->stream));
    CK(cudaMemcpyAsync(e->sec_desc, d.data(), (size_t)n * sizeof(WinDesc), cudaMemcpyHostToDevice, e->stream));
    // pass i reads its window of the working image, which holds the fills of
    // passes 0..i-1, and writes its own fill back (stream order)
    for (int i = 0; i < n; i++) {
      CK(cudaMemcpyAsync(pl.win, e->sec_desc + i, sizeof(WinDesc), cudaMemcpyDeviceToDevice, e->stream));
      run_plan(e, pl);
    }
    CK(cudaMemcpyAsync(out_rgb, e->sec_img, npx * 3, cudaMemcpyDeviceToHost, e->stream));
    sync_check(e);
  });
}

static int resblocks_impl(lama_engine* e, const float* l_in, const float* g_in, int batch, int h, int w, int nblocks,
                          float* l_out, float* g_out, cudaMemcpyKind kin, cudaMemcpyKind kout, bool sync) {
  return guarded(e, [&] {
    if (!l_in || !g_in || !l_out || !g_out) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, false);
    if (nblocks < 0 || nblocks > 18) throw EngineError{LAMA_EINVAL, "nblocks must be in 0..18"};
    Plan& pl = get_plan(e, 2, batch, h, w, h, w, nblocks);
    const size_t nl = (size_t)batch * 128 * h * w, ng = (size_t)batch * 384 * h * w;
    CK(cudaMemcpyAsync(pl.l_in, l_in, nl * 4, kin, e->stream));
    CK(cudaMemcpyAsync(pl.g_in, g_in, ng * 4, kin, e->stream));
    run_plan(e, pl);
    CK(cudaMemcpyAsync(l_out, pl.l_out, nl * 4, kout, e->stream));
    CK(cudaMemcpyAsync(g_out, pl.g_out, ng * 4, kout, e->stream));
    if (sync) sync_check(e);
  });
}

int lama_resblocks(lama_engine* e, const float* local_in, const float* global_in, int batch, int h, int w,
                   int nblocks, float* local_out, float* global_out) {
  return resblocks_impl(e, local_in, global_in, batch, h, w, nblocks, local_out, global_out, cudaMemcpyHostToDevice,
                        cudaMemcpyDeviceToHost, true);
}

int lama_resblocks_device(lama_engine* e, const float* d_local_in, const float* d_global_in, int batch, int h,
                          int w, int nblocks, float* d_local_out, float* d_global_out) {
  return resblocks_impl(e, d_local_in, d_global_in, batch, h, w, nblocks, d_local_out, d_global_out,
                        cudaMemcpyDeviceToDevice, cudaMemcpyDeviceToDevice, false);
}

int lama_set_tiling(lama_engine* e, int policy) {
  return guarded(e, [&] {
    if (policy < LAMA_TILING_AUTO || policy > LAMA_TILING_PAIRED) throw EngineError{LAMA_EINVAL, "unknown tiling policy"};
    CK(cudaStreamSynchronize(e->stream));
    e->plans.clear();
    e->tiling = policy;
  });
}

int lama_set_lanes(lama_engine* e, int chain_sms) {
  return guarded(e, [&] {
    if (chain_sms < -1 || chain_sms > e->sms / 2) throw EngineError{LAMA_EINVAL, "chain_sms must be in -1..sms/2"};
    CK(cudaStreamSynchronize(e->stream));
    e->plans.clear();
    e->chain_sms = chain_sms < 0 ? kDefaultChainSms : chain_sms;
  });
}

int lama_set_spectral_path(lama_engine* e, int path) {
  return guarded(e, [&] {
    if (path < LAMA_SPECTRAL_AUTO || path > LAMA_SPECTRAL_TENSOR) throw EngineError{LAMA_EINVAL, "unknown spectral path"};
    CK(cudaStreamSynchronize(e->stream));
    e->plans.clear();
    e->spectral = path;
  });
}

const char* lama_last_error(const lama_engine* e) { return e ? e->err.c_str() : "null engine"; }

int lama_synchronize(lama_engine* e) {
  return guarded(e, [&] { sync_check(e); });
}

void* lama_stream(lama_engine* e) { return e ? (void*)e->stream : nullptr; }

int lama_launch_count(lama_engine* e, int batch, int h, int w) {
  int n = 0;
  int rc = guarded(e, [&] {
    check_shape(batch, h, w, true);
    n = (int)get_plan(e, 0, batch, h, w, h, w, 18).ops.size();
  });
  return rc ? rc : n;
}

long long lama_estimate_bytes(int batch, int h, int w) {
  if (batch < 1 || h < 1 || w < 1) return LAMA_EINVAL;
  if ((long long)h * w > (1LL << 28) || batch > (1 << 16)) return LAMA_EINVAL;
  try {
    // a B200 as the engine sees it: 148 SMs, CTA-pair clusters available,
    // automatic tiling and spectral paths
    static lama_engine* shape_engine = [] {
      lama_engine* x = new lama_engine();
      weight_shapes(x->W);
      x->sms = 148;
      x->pair_clusters = 74;
      return x;
    }();
    const int H = (h + 7) / 8 * 8, W = (w + 7) / 8 * 8;
    return (long long)plan_bytes_dry(shape_engine, 1, batch, H, W, h, w, 18);
  } catch (const EngineError& x) {
    return x.code;
  } catch (const std::exception&) {
    return LAMA_EINVAL;
  }
}

int lama_plan_bytes(lama_engine* e, int batch, int h, int w, long long* bytes) {
  return guarded(e, [&] {
    if (!bytes) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, false);
    const int H = (h + 7) / 8 * 8, W = (w + 7) / 8 * 8;
    *bytes = (long long)get_plan(e, 1, batch, H, W, h, w, 18).mem.total;
  });
}

int lama_profile_forward(lama_engine* e, const float* d_in, int batch, int h, int w, float* d_out,
                         lama_kernel_stat* stats, int max_stats, int* n_stats) {
  return guarded(e, [&] {
    check_shape(batch, h, w, true);
    Plan& pl = get_plan(e, 0, batch, h, w, h, w, 18);
    const size_t nin = (size_t)batch * 4 * h * w, nout = (size_t)batch * 3 * h * w;
    CK(cudaMemcpyAsync(pl.in_f32, d_in, nin * 4, cudaMemcpyDeviceToDevice, e->stream));
    EventSet evs(pl.ops.size() + 1);
    std::vector<cudaEvent_t>& ev = evs.ev;
    for (auto& x : ev) CK(cudaEventCreate(&x));
    CK(cudaEventRecord(ev[0], e->stream));
    for (size_t i = 0; i < pl.ops.size(); i++) {
      CKL(launch_named(pl.ops[i], e->stream));
      CK(cudaEventRecord(ev[i + 1], e->stream));
    }
    CK(cudaMemcpyAsync(d_out, pl.out, nout * 4, cudaMemcpyDeviceToDevice, e->stream));
    sync_check(e);
    std::vector<std::string> names;
    std::map<std::string, lama_kernel_stat> agg;
    for (size_t i = 0; i < pl.ops.size(); i++) {
      float ms = 0;
      CK(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
      const std::string& nm = pl.ops[i].name;
      if (!agg.count(nm)) {
        lama_kernel_stat s{};
        snprintf(s.name, sizeof(s.name), "%s", nm.c_str());
        agg[nm] = s;
        names.push_back(nm);
      }
      lama_kernel_stat& s = agg[nm];
      s.launches++;
      s.ms += ms;
      s.flops += pl.ops[i].flops;
      s.bytes += pl.ops[i].bytes;
    }
    int n = 0;
    for (const std::string& nm : names) {
      if (n < max_stats && stats) stats[n] = agg[nm];
      n++;
    }
    if (n_stats) *n_stats = n;
  });
}

int lama_profile_timeline(lama_engine* e, const float* d_in, int batch, int h, int w, float* d_out,
                          lama_op_time* times, int max_ops, int* n_ops) {
  return guarded(e, [&] {
    if (!d_in || !d_out) throw EngineError{LAMA_EINVAL, "null buffer"};
    check_shape(batch, h, w, true);
    Plan& pl = get_plan(e, 0, batch, h, w, h, w, 18);
    const size_t nin = (size_t)batch * 4 * h * w, nout = (size_t)batch * 3 * h * w;
    EventSet evs(pl.ops.size() + 1);
    for (auto& x : evs.ev) CK(cudaEventCreate(&x));
    cudaGraphExec_t exec = capture_plan(e, pl, &evs.ev);
    struct ExecGuard {
      cudaGraphExec_t x;
      ~ExecGuard() { cudaGraphExecDestroy(x); }
    } guard{exec};
    CK(cudaMemcpyAsync(pl.in_f32, d_in, nin * 4, cudaMemcpyDeviceToDevice, e->stream));
    for (int rep = 0; rep < 2; rep++) CK(cudaGraphLaunch(exec, e->stream));  // the second replay is read
    CK(cudaMemcpyAsync(d_out, pl.out, nout * 4, cudaMemcpyDeviceToDevice, e->stream));
    sync_check(e);
    std::vector<float> end(pl.ops.size(), 0.f);
    int last[2] = {-1, -1};
    for (size_t i = 0; i < pl.ops.size(); i++) {
      const Op& op = pl.ops[i];
      CK(cudaEventElapsedTime(&end[i], evs.ev[0], evs.ev[i + 1]));
      float ready = last[op.lane] >= 0 ? end[(size_t)last[op.lane]] : 0.f;
      for (int j : op.waits) ready = std::max(ready, end[(size_t)j]);
      last[op.lane] = (int)i;
      if ((int)i < max_ops && times) {
        lama_op_time& t = times[i];
        snprintf(t.name, sizeof(t.name), "%s", op.name.c_str());
        t.lane = op.lane;
        t.ready_ms = ready;
        t.end_ms = end[i];
      }
    }
    if (n_ops) *n_ops = (int)pl.ops.size();
  });
}

namespace {
// One CTA waits on an mbarrier that never completes, with a bounded spin:
// the same give-up path as the pass kernels' waits, with a short limit.
__global__ void k_wait_probe(int* err, long long limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  fence_mbar_init();
  const long long t0 = clock64();
  while (!mbar_try_wait(b, 0)) {
    if (clock64() - t0 > limit_cycles) {
      atomicCAS(err, 0, 6);
      return;
    }
  }
}
}  // namespace

int lama_debug_wait_timeout(lama_engine* e, int limit_ms) {
  return guarded(e, [&] {
    if (limit_ms < 1 || limit_ms > 1000) throw EngineError{LAMA_EINVAL, "limit_ms must be in 1..1000"};
    int khz = 0;
    CK(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, e->device));
    k_wait_probe<<<1, 32, 0, e->stream>>>(e->d_err, (long long)khz * limit_ms);
    CKL((int)cudaGetLastError());
    sync_check(e);
  });
}

int lama_debug_run(lama_engine* e, const float* in, int batch, int h, int w, int n_ops) {
  return guarded(e, [&] {
    check_shape(batch, h, w, true);
    Plan& pl = get_plan(e, 0, batch, h, w, h, w, 18);
    CK(cudaMemcpyAsync(pl.in_f32, in, (size_t)batch * 4 * h * w * 4, cudaMemcpyHostToDevice, e->stream));
    const int n = std::min<int>(n_ops, (int)pl.ops.size());
    for (int i = 0; i < n; i++) CKL(launch_named(pl.ops[i], e->stream));
    sync_check(e);
  });
}

int lama_debug_read(lama_engine* e, int batch, int h, int w, int op, float* out, long long cap, int* dims,
                    char* name) {
  return guarded(e, [&] {
    Plan& pl = get_plan(e, 0, batch, h, w, h, w, 18);
    if (op < 0 || op >= (int)pl.ops.size()) throw EngineError{LAMA_EINVAL, "op index out of range"};
    const Op& o = pl.ops[op];
    if (!o.out_ptr) throw EngineError{LAMA_EINVAL, "op has no recorded output"};
    const long long n = (long long)o.dims[0] * o.dims[1] * o.dims[2] * o.dims[3];
    for (int i = 0; i < 4; i++) dims[i] = o.dims[i];
    if (name) snprintf(name, 32, "%s", o.name.c_str());
    if (!out) return;
    if (n > cap) throw EngineError{LAMA_EINVAL, "buffer too small"};
    if (o.out_split) {
      std::vector<uint16_t> hl((size_t)2 * n);
      CK(cudaMemcpy(hl.data(), o.out_ptr, (size_t)n * 2, cudaMemcpyDeviceToHost));
      CK(cudaMemcpy(hl.data() + n, (uint16_t*)o.out_ptr + o.out_part, (size_t)n * 2, cudaMemcpyDeviceToHost));
      for (long long i = 0; i < n; i++) out[i] = bf2f(hl[i]) + bf2f(hl[n + i]);
    } else {
      CK(cudaMemcpy(out, o.out_ptr, (size_t)n * 4, cudaMemcpyDeviceToHost));
    }
  });
}

void lama_close(lama_engine* e) {
  if (!e) return;
  if (e->stream) {
    cudaSetDevice(e->device);
    cudaStreamSynchronize(e->stream);
  }
  e->plans.clear();
  e->sec_mem.free_all();
  e->pipe_mem.free_all();
  for (int i = 0; i < 2; i++) {
    if (e->ev_in[i]) cudaEventDestroy(e->ev_in[i]);
    if (e->ev_done[i]) cudaEventDestroy(e->ev_done[i]);
  }
  if (e->copy_stream) cudaStreamDestroy(e->copy_stream);
  e->wmem.free_all();
  if (e->side_stream) cudaStreamDestroy(e->side_stream);
  if (e->stream) cudaStreamDestroy(e->stream);
  cudaGetLastError();
  delete e;
}

}  // extern "C"
