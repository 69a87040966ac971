// Harness for the reference's CUDA path on a B200: times it, and runs it on
// given weights and inputs so the tests can check the CPU oracle against it.
// Test and measurement infrastructure only: nothing here is part of the engine.
//
// The reference's own kernel file (lama-rs/cuda/lama.cu) is compiled into this
// translation unit from where it lies in the reference checkout (the oracle
// Makefile passes its directory with -I; no copy is kept in this repository).
// The host side replays the launch sequence of the reference's `cuda::run`
// (lama-rs/src/cuda.rs:1542-1691) for one big-lama forward pass:
//   conv_forward   (cuda.rs:973-1040)   k_im2col + k_sgemm_slab (+ k_bias_plane)
//   conv_1x1       (cuda.rs:1141-1163)  k_sgemm_slab
//   conv_7x7_direct(cuda.rs:1042-1066)  k_conv7x7 (the OutConv)
//   bn_relu / bn_relu_add (cuda.rs:1165-1198), reflect_pad (:1227-1240),
//   concat (:1259-1278), conv_transpose_phases (:1280-1331),
//   run_dffc (:1364-1434), spectral_forward (:1460-1539)
// with the same grid/block shapes (256-thread blocks, 64x64 GEMM tiles).
//
// The five toolkit kernels of the `lightgpu` dependency, which is not in the
// reference tree, are stand-ins here: lg_sigmoid, lg_add_inplace and lg_copy are
// one-line elementwise kernels written for this harness; lg_fft2_r2c / lg_fft2_c2r
// are cuFFT batched 2-D transforms (plus a scale pass after the inverse), so the
// FFT share of the figure is approximate.  Allocation follows the reference's
// pool in spirit: a bump arena reset per pass, no cudaMalloc in the timed loop.
// Weights are seeded pseudo-random values of the big-lama shapes (timing does not
// depend on them).
//
// Usage:
//   ref_cuda_bench [side=512] [passes=5] [warmup=2]
//     times passes with seeded pseudo-random weights; prints one line
//     "ref_cuda side=S ms_per_pass=T passes=K arena_used_gb=G".
//   ref_cuda_bench --run WEIGHTS.safetensors IN.f32 OUT.f32 H W
//     one pass with the checkpoint's weights (F32 safetensors, big-lama names,
//     BN folded as cuda.rs:737-756 folds it, ConvT phase matrices built as
//     cuda.rs:913-945 builds them) on IN = [4][H][W] f32; writes the sigmoid
//     output [3][H][W] f32 to OUT.  This is how the tests check the CPU oracle
//     against the reference's own kernels.
#include <cuda_runtime.h>
#include <cufft.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "lama.cu"

namespace {

#define CK(x)                                                                              \
  do {                                                                                     \
    cudaError_t e_ = (x);                                                                  \
    if (e_ != cudaSuccess) {                                                               \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_));   \
      exit(1);                                                                             \
    }                                                                                      \
  } while (0)

constexpr int BLOCK = 256;
unsigned grid_for(long long n, int block) { return (unsigned)((n + block - 1) / block); }

// ---- toolkit stand-ins
__global__ void h_sigmoid(const float* x, float* y, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = 1.0f / (1.0f + __expf(-x[i]));
}
__global__ void h_add_inplace(float* a, const float* b, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] += b[i];
}
__global__ void h_copy(const float* s, float* d, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) d[i] = s[i];
}
__global__ void h_scale(float* x, float s, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] *= s;
}
__global__ void h_fill(float* x, long long n, unsigned seed, float amp) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  unsigned v = (unsigned)i * 2654435761u ^ seed;
  v ^= v >> 15; v *= 2246822519u; v ^= v >> 13;
  x[i] = amp * (((float)(v & 0xffffff) / 16777216.0f) * 2.0f - 1.0f);
}

// ---- memory: weights stay, activations come from a per-pass bump arena
struct Arena {
  char* base = nullptr;
  size_t cap = 0, used = 0;
  float* get(long long n) {
    const size_t b = ((size_t)n * 4 + 255) & ~size_t(255);
    if (used + b > cap) { fprintf(stderr, "arena exhausted\n"); exit(1); }
    float* p = (float*)(base + used);
    used += b;
    return p;
  }
};
Arena g_arena;
unsigned g_seed = 1;
cudaStream_t g_st;

float* weight(long long n, float amp) {
  float* p;
  CK(cudaMalloc(&p, (size_t)n * 4));
  h_fill<<<grid_for(n, BLOCK), BLOCK>>>(p, n, g_seed++ * 7919u, amp);
  return p;
}
float* upload(const std::vector<float>& v) {
  float* p;
  CK(cudaMalloc(&p, v.size() * 4));
  CK(cudaMemcpy(p, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return p;
}

// F32 safetensors: an 8-byte header length, a JSON header, then the data.
struct Checkpoint {
  std::vector<char> bytes;
  size_t data0 = 0;
  std::string header;
  bool open(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return false;
    fseek(f, 0, SEEK_END);
    bytes.resize((size_t)ftell(f));
    fseek(f, 0, SEEK_SET);
    const bool ok = fread(bytes.data(), 1, bytes.size(), f) == bytes.size();
    fclose(f);
    if (!ok || bytes.size() < 8) return false;
    unsigned long long n = 0;
    memcpy(&n, bytes.data(), 8);
    if (8 + n > bytes.size()) return false;
    header.assign(bytes.data() + 8, (size_t)n);
    data0 = 8 + (size_t)n;
    return true;
  }
  std::vector<float> get(const std::string& name, size_t expect) const {
    const std::string key = "\"" + name + "\":";
    const size_t at = header.find(key);
    if (at == std::string::npos) { fprintf(stderr, "missing tensor %s\n", name.c_str()); exit(1); }
    const size_t off = header.find("\"data_offsets\"", at);
    unsigned long long a = 0, b = 0;
    if (off == std::string::npos || sscanf(header.c_str() + header.find('[', off), "[%llu,%llu]", &a, &b) != 2 ||
        (b - a) != expect * 4 || data0 + b > bytes.size()) {
      fprintf(stderr, "bad tensor %s\n", name.c_str());
      exit(1);
    }
    std::vector<float> v(expect);
    memcpy(v.data(), bytes.data() + data0 + a, (size_t)(b - a));
    return v;
  }
};
const Checkpoint* g_ckpt = nullptr;

struct Acts { float* p; int c, h, w; long long n() const { return (long long)c * h * w; } };
struct Conv { float* w; float* bias; float* w_t; int cin, cout, k; };
struct Bn { float* scale; float* shift; int c; };
struct ConvT { float* phase[4]; float* bias; int cin, cout; };

// A convolution `prefix`.weight [cout][cin][k][k] (and .bias): from the
// checkpoint when one is loaded, else seeded values.  `direct`: also the
// [cin][cout][k][k] copy the direct 7x7 kernel reads (cuda.rs:709-723).
Conv conv(const std::string& prefix, int cin, int cout, int k, bool bias = false, bool direct = false) {
  const long long n = (long long)cout * cin * k * k;
  if (!g_ckpt) {
    Conv c{weight(n, 1.0f / std::sqrt((float)cin * k * k)), nullptr, nullptr, cin, cout, k};
    if (bias) c.bias = weight(cout, 0.05f);
    if (direct) c.w_t = weight(n, 1.0f / std::sqrt((float)cin * k * k));
    return c;
  }
  const std::vector<float> w = g_ckpt->get(prefix + ".weight", (size_t)n);
  Conv c{upload(w), nullptr, nullptr, cin, cout, k};
  if (bias) c.bias = upload(g_ckpt->get(prefix + ".bias", (size_t)cout));
  if (direct) {
    std::vector<float> t((size_t)n);
    for (int co = 0; co < cout; co++)
      for (int ci = 0; ci < cin; ci++)
        for (int q = 0; q < k * k; q++) t[((size_t)ci * cout + co) * k * k + q] = w[((size_t)co * cin + ci) * k * k + q];
    c.w_t = upload(t);
  }
  return c;
}
// BatchNorm `prefix` folded to (scale, shift) in f32: s = w / sqrt(var + 1e-5), t = b - mean * s.
Bn bn(const std::string& prefix, int c) {
  if (!g_ckpt) return Bn{weight(c, 0.2f), weight(c, 0.05f), c};
  const auto w = g_ckpt->get(prefix + ".weight", c), b = g_ckpt->get(prefix + ".bias", c);
  const auto mean = g_ckpt->get(prefix + ".running_mean", c), var = g_ckpt->get(prefix + ".running_var", c);
  std::vector<float> sc(c), sh(c);
  for (int i = 0; i < c; i++) {
    sc[i] = w[i] / std::sqrt(var[i] + 1e-5f);
    sh[i] = b[i] - mean[i] * sc[i];
  }
  return Bn{upload(sc), upload(sh), c};
}
const int kTaps[4] = {1, 2, 2, 4};
// Output-phase tap sets of a k3 s2 p1 transposed conv (cuda.rs:566-577), phase = py * 2 + px.
const int kTapY[4][4] = {{1, 0, 0, 0}, {1, 1, 0, 0}, {0, 2, 0, 0}, {0, 0, 2, 2}};
const int kTapX[4][4] = {{1, 0, 0, 0}, {0, 2, 0, 0}, {1, 1, 0, 0}, {0, 2, 0, 2}};
// ConvT `prefix`.weight [cin][cout][3][3] regrouped into one [cout][cin * taps]
// matrix per phase, column ci * taps + t (cuda.rs:913-945).
ConvT convt(const std::string& prefix, int cin, int cout) {
  ConvT t{};
  t.cin = cin;
  t.cout = cout;
  if (!g_ckpt) {
    for (int ph = 0; ph < 4; ph++) t.phase[ph] = weight((long long)cout * cin * kTaps[ph], 1.0f / std::sqrt(cin * 2.25f));
    t.bias = weight(cout, 0.05f);
    return t;
  }
  const auto w = g_ckpt->get(prefix + ".weight", (size_t)cin * cout * 9);
  for (int ph = 0; ph < 4; ph++) {
    const int taps = kTaps[ph], k = cin * taps;
    std::vector<float> m((size_t)cout * k);
    for (int ci = 0; ci < cin; ci++)
      for (int ti = 0; ti < taps; ti++)
        for (int co = 0; co < cout; co++)
          m[(size_t)co * k + ci * taps + ti] = w[(((size_t)ci * cout + co) * 3 + kTapY[ph][ti]) * 3 + kTapX[ph][ti]];
    t.phase[ph] = upload(m);
  }
  t.bias = upload(g_ckpt->get(prefix + ".bias", cout));
  return t;
}

// ---- the reference's launch helpers (cuda.rs)
void sgemm(const float* a, const float* b, float* out, int k, int cout, long long n) {
  const int nb_cols = (int)grid_for(n, 64);
  const unsigned grid = (unsigned)nb_cols * grid_for(cout, 64);
  k_sgemm_slab<<<grid, BLOCK, 0, g_st>>>(a, b, out, (int)n, k, (int)n, k, cout, (int)n, nb_cols, 0);
}
Acts conv_forward(const Conv& cv, const Acts& src, int pad, int stride, bool reflect) {
  const long long n0 = (long long)src.h * src.w;
  if (cv.k == 1 && stride == 1) {  // conv_1x1
    float* out = g_arena.get((long long)cv.cout * n0);
    sgemm(src.p, cv.w, out, cv.cin, cv.cout, n0);
    if (cv.bias) k_bias_plane<<<grid_for(cv.cout * n0, BLOCK), BLOCK, 0, g_st>>>(out, cv.bias, cv.cout, n0);
    return Acts{out, cv.cout, src.h, src.w};
  }
  if (cv.k == 7 && stride == 1 && pad == 0 && cv.w_t) {  // conv_7x7_direct
    const int oh = src.h - 6, ow = src.w - 6;
    float* out = g_arena.get((long long)cv.cout * oh * ow);
    k_conv7x7<<<grid_for((long long)oh * ow, BLOCK), BLOCK, 0, g_st>>>(src.p, cv.w_t, cv.bias, out, cv.cin, cv.cout,
                                                                       src.h, src.w, oh, ow);
    return Acts{out, cv.cout, oh, ow};
  }
  const int oh = (src.h + 2 * pad - cv.k) / stride + 1, ow = (src.w + 2 * pad - cv.k) / stride + 1;
  const int k = cv.cin * cv.k * cv.k;
  const long long n = (long long)oh * ow;
  float* col = g_arena.get((long long)k * n);
  float* out = g_arena.get((long long)cv.cout * n);
  k_im2col<<<grid_for((long long)k * n, BLOCK), BLOCK, 0, g_st>>>(src.p, col, cv.cin, src.h, src.w, cv.k, cv.k, pad, pad,
                                                                 stride, oh, ow, reflect ? 1 : 0);
  sgemm(col, cv.w, out, k, cv.cout, n);
  if (cv.bias) k_bias_plane<<<grid_for(cv.cout * n, BLOCK), BLOCK, 0, g_st>>>(out, cv.bias, cv.cout, n);
  return Acts{out, cv.cout, oh, ow};
}
void bn_relu(Acts& x, const Bn& b) {
  k_bn_relu<<<grid_for(x.n(), BLOCK), BLOCK, 0, g_st>>>(x.p, b.scale, b.shift, (long long)x.h * x.w, b.c);
}
void bn_relu_add(Acts& x, const Bn& b, const Acts* skip) {
  k_bn_relu_add<<<grid_for(x.n(), BLOCK), BLOCK, 0, g_st>>>(x.p, skip ? skip->p : nullptr, b.scale, b.shift,
                                                           (long long)x.h * x.w, b.c);
}
void add_inplace(Acts& a, const Acts& b) { h_add_inplace<<<grid_for(a.n(), BLOCK), BLOCK, 0, g_st>>>(a.p, b.p, a.n()); }
Acts reflect_pad(const Acts& s, int pad) {
  Acts o{g_arena.get((long long)s.c * (s.h + 2 * pad) * (s.w + 2 * pad)), s.c, s.h + 2 * pad, s.w + 2 * pad};
  k_reflect_pad<<<grid_for(o.n(), BLOCK), BLOCK, 0, g_st>>>(s.p, o.p, s.c, s.h, s.w, pad);
  return o;
}
Acts copy_acts(const Acts& s) {
  Acts o{g_arena.get(s.n()), s.c, s.h, s.w};
  h_copy<<<grid_for(s.n(), BLOCK), BLOCK, 0, g_st>>>(s.p, o.p, s.n());
  return o;
}
Acts view(const Acts& a, int first, int c) { return Acts{a.p + (long long)first * a.h * a.w, c, a.h, a.w}; }

// ---- spectral branch (cuda.rs:1460-1539), FFT by cuFFT plans made once per size
struct Spectral { Conv conv1; Bn bn1; Conv fu; Bn fu_bn; Conv conv2; int half; };
struct FftPlans { int h = 0; cufftHandle r2c = 0, c2r = 0; };
FftPlans g_fft;
void fft_plans(int h, int w, int half) {
  if (g_fft.h == h) return;
  int n[2] = {h, w};
  if (cufftPlanMany(&g_fft.r2c, 2, n, nullptr, 1, 0, nullptr, 1, 0, CUFFT_R2C, half) != CUFFT_SUCCESS ||
      cufftPlanMany(&g_fft.c2r, 2, n, nullptr, 1, 0, nullptr, 1, 0, CUFFT_C2R, half) != CUFFT_SUCCESS) {
    fprintf(stderr, "cufftPlanMany failed\n");
    exit(1);
  }
  cufftSetStream(g_fft.r2c, g_st);
  cufftSetStream(g_fft.c2r, g_st);
  g_fft.h = h;
}
Acts spectral_forward(const Spectral& sp, const Acts& g) {
  Acts pooled = copy_acts(g);  // stride 1: the reference copies the global half
  Acts feat = conv_forward(sp.conv1, pooled, 0, 1, false);
  bn_relu(feat, sp.bn1);
  const int h = feat.h, w = feat.w, half = sp.half, hw = w / 2 + 1;
  const float scale = 1.0f / std::sqrt((float)(h * w));
  fft_plans(h, w, half);
  float* complex = g_arena.get(2LL * half * h * hw);
  cufftExecR2C(g_fft.r2c, feat.p, (cufftComplex*)complex);
  float* packed = g_arena.get(2LL * half * h * hw);
  k_spec_pack<<<grid_for((long long)half * h * hw, BLOCK), BLOCK, 0, g_st>>>(complex, packed, half, h * hw, scale);
  Acts spec{packed, 2 * half, h, hw};
  Acts fu = conv_forward(sp.fu, spec, 0, 1, false);
  bn_relu(fu, sp.fu_bn);
  float* complex2 = g_arena.get(2LL * half * h * hw);
  k_spec_unpack<<<grid_for((long long)half * h * hw, BLOCK), BLOCK, 0, g_st>>>(fu.p, complex2, half, h * hw);
  Acts inv{g_arena.get((long long)half * h * w), half, h, w};
  cufftExecC2R(g_fft.c2r, (cufftComplex*)complex2, inv.p);
  h_scale<<<grid_for(inv.n(), BLOCK), BLOCK, 0, g_st>>>(inv.p, scale, inv.n());
  add_inplace(inv, feat);
  return conv_forward(sp.conv2, inv, 0, 1, false);
}

// ---- FFC layer (cuda.rs:1364-1434)
struct Ffc {
  int in_l, in_g, out_l, out_g, k, stride, pad;
  bool reflect;
  Conv *l2l = nullptr, *l2g = nullptr, *g2l = nullptr;
  Spectral* sp = nullptr;
  Bn *bn_l = nullptr, *bn_g = nullptr;
};
void run_ffc(const Ffc& f, const Acts& inp, const Acts* glob, const Acts* skip_l, const Acts* skip_g, Acts& out_l,
             Acts& out_g, bool& has_g) {
  Acts local = f.in_g == 0 ? inp : view(inp, 0, f.in_l);
  if (f.out_l > 0) {
    Acts acc = conv_forward(*f.l2l, local, f.pad, f.stride, f.reflect);
    if (f.g2l) {
      Acts o = conv_forward(*f.g2l, *glob, f.pad, f.stride, f.reflect);
      add_inplace(acc, o);
    }
    bn_relu_add(acc, *f.bn_l, skip_l);
    out_l = acc;
  }
  has_g = f.out_g > 0;
  if (has_g) {
    Acts acc = conv_forward(*f.l2g, local, f.pad, f.stride, f.reflect);
    if (f.sp) {
      Acts gv = view(*glob, glob->c - f.in_g, f.in_g);
      Acts o = spectral_forward(*f.sp, gv);
      add_inplace(acc, o);
    }
    bn_relu_add(acc, *f.bn_g, skip_g);
    out_g = acc;
  }
}

// ---- ConvT through the four phase GEMMs (cuda.rs:1280-1331)
Acts conv_transpose_phases(const ConvT& cv, const Acts& src) {
  const int oh = src.h * 2, ow = src.w * 2;
  Acts out{g_arena.get((long long)cv.cout * oh * ow), cv.cout, oh, ow};
  for (int ph = 0; ph < 4; ph++) {
    const int py = ph / 2, px = ph % 2, taps = kTaps[ph], k = cv.cin * taps;
    const long long n = (long long)((oh + 1) / 2) * ((ow + 1) / 2);
    float* col = g_arena.get((long long)k * n);
    float* phase_out = g_arena.get((long long)cv.cout * n);
    k_convt_col<<<grid_for((long long)k * n, BLOCK), BLOCK, 0, g_st>>>(src.p, col, cv.cin, src.h, src.w, py, px, taps,
                                                                      (int)n, oh, ow);
    sgemm(col, cv.phase[ph], phase_out, k, cv.cout, n);
    k_convt_put<<<grid_for((long long)cv.cout * n, BLOCK), BLOCK, 0, g_st>>>(phase_out, out.p, cv.bias, cv.cout, (int)n,
                                                                            py, px, oh, ow, 1);
  }
  return out;
}

// ---- the big-lama network
struct Net {
  Ffc m1, m2, m3, m4;
  std::vector<Ffc> res;  // 36: block i conv1 / conv2
  ConvT ct[3];
  Bn ct_bn[3];
  Conv outc;
};
Ffc local_ffc(int idx, int cin, int cout, int k, int stride, int pad, bool reflect) {
  const std::string m = "model." + std::to_string(idx);
  Ffc f{cin, 0, cout, 0, k, stride, pad, reflect};
  f.l2l = new Conv(conv(m + ".ffc.convl2l", cin, cout, k));
  f.bn_l = new Bn(bn(m + ".bn_l", cout));
  return f;
}
// The big-lama topology (model.rs:135-257) with the checkpoint's module names.
Net build_net() {
  Net n;
  n.m1 = local_ffc(1, 4, 64, 7, 1, 0, false);
  n.m2 = local_ffc(2, 64, 128, 3, 2, 1, true);
  n.m3 = local_ffc(3, 128, 256, 3, 2, 1, true);
  n.m4 = Ffc{256, 0, 128, 384, 3, 2, 1, true};
  n.m4.l2l = new Conv(conv("model.4.ffc.convl2l", 256, 128, 3));
  n.m4.l2g = new Conv(conv("model.4.ffc.convl2g", 256, 384, 3));
  n.m4.bn_l = new Bn(bn("model.4.bn_l", 128));
  n.m4.bn_g = new Bn(bn("model.4.bn_g", 384));
  for (int i = 0; i < 36; i++) {
    const std::string p = "model." + std::to_string(5 + i / 2) + ".conv" + std::to_string(1 + i % 2);
    const std::string q = p + ".ffc";
    Ffc f{128, 384, 128, 384, 3, 1, 1, true};
    f.l2l = new Conv(conv(q + ".convl2l", 128, 128, 3));
    f.l2g = new Conv(conv(q + ".convl2g", 128, 384, 3));
    f.g2l = new Conv(conv(q + ".convg2l", 384, 128, 3));
    f.sp = new Spectral{conv(q + ".convg2g.conv1.0", 384, 192, 1), bn(q + ".convg2g.conv1.1", 192),
                        conv(q + ".convg2g.fu.conv_layer", 384, 384, 1), bn(q + ".convg2g.fu.bn", 384),
                        conv(q + ".convg2g.conv2", 192, 384, 1), 192};
    f.bn_l = new Bn(bn(p + ".bn_l", 128));
    f.bn_g = new Bn(bn(p + ".bn_g", 384));
    n.res.push_back(f);
  }
  const int cins[3] = {512, 256, 128}, couts[3] = {256, 128, 64}, mods[3] = {24, 27, 30};
  for (int u = 0; u < 3; u++) {
    n.ct[u] = convt("model." + std::to_string(mods[u]), cins[u], couts[u]);
    n.ct_bn[u] = bn("model." + std::to_string(mods[u] + 1), couts[u]);
  }
  n.outc = conv("model.34", 64, 3, 7, true, true);
  return n;
}

// One forward pass (cuda.rs:1542-1691); returns the sigmoid output.
Acts forward(const Net& net, const Acts& input) {
  g_arena.used = 0;
  Acts acts = reflect_pad(input, 3);
  Acts g{};
  bool has_g = false;
  Acts l;
  run_ffc(net.m1, acts, nullptr, nullptr, nullptr, l, g, has_g);
  acts = l;
  run_ffc(net.m2, acts, nullptr, nullptr, nullptr, l, g, has_g);
  acts = l;
  run_ffc(net.m3, acts, nullptr, nullptr, nullptr, l, g, has_g);
  acts = l;
  run_ffc(net.m4, acts, nullptr, nullptr, nullptr, l, g, has_g);
  acts = l;
  for (int b = 0; b < 18; b++) {
    Acts l1, g1, l2, g2;
    bool h1, h2;
    run_ffc(net.res[2 * b], acts, &g, nullptr, nullptr, l1, g1, h1);
    run_ffc(net.res[2 * b + 1], l1, &g1, &acts, &g, l2, g2, h2);
    acts = l2;
    g = g2;
  }
  // Concat (two copy launches)
  Acts cat{g_arena.get(acts.n() + g.n()), acts.c + g.c, acts.h, acts.w};
  h_copy<<<grid_for(acts.n(), BLOCK), BLOCK, 0, g_st>>>(acts.p, cat.p, acts.n());
  h_copy<<<grid_for(g.n(), BLOCK), BLOCK, 0, g_st>>>(g.p, cat.p + acts.n(), g.n());
  acts = cat;
  for (int u = 0; u < 3; u++) {
    Acts up = conv_transpose_phases(net.ct[u], acts);
    bn_relu(up, net.ct_bn[u]);
    acts = up;
  }
  acts = reflect_pad(acts, 3);
  Acts out = conv_forward(net.outc, acts, 0, 1, false);
  h_sigmoid<<<grid_for(out.n(), BLOCK), BLOCK, 0, g_st>>>(out.p, out.p, out.n());
  return out;
}

}  // namespace

int run_file(int argc, char** argv) {
  if (argc != 7) {
    fprintf(stderr, "usage: ref_cuda_bench --run WEIGHTS IN.f32 OUT.f32 H W\n");
    return 2;
  }
  const int h = atoi(argv[5]), w = atoi(argv[6]);
  if (h < 8 || w < 8 || h % 8 || w % 8 || h > 1024 || w > 1024) {
    fprintf(stderr, "H and W must be multiples of 8 in 8..1024\n");
    return 2;
  }
  static Checkpoint ck;
  if (!ck.open(argv[2])) {
    fprintf(stderr, "cannot read %s\n", argv[2]);
    return 1;
  }
  g_ckpt = &ck;
  std::vector<float> x((size_t)4 * h * w);
  FILE* f = fopen(argv[3], "rb");
  if (!f || fread(x.data(), 4, x.size(), f) != x.size()) {
    fprintf(stderr, "cannot read %s\n", argv[3]);
    return 1;
  }
  fclose(f);
  CK(cudaStreamCreateWithFlags(&g_st, cudaStreamNonBlocking));
  g_arena.cap = (size_t)std::max(h, w) * std::max(h, w) * 4 * 16000;
  CK(cudaMalloc(&g_arena.base, g_arena.cap));
  Net net = build_net();
  Acts in{upload(x), 4, h, w};
  CK(cudaDeviceSynchronize());
  Acts out = forward(net, in);
  CK(cudaStreamSynchronize(g_st));
  CK(cudaGetLastError());
  std::vector<float> y((size_t)out.n());
  CK(cudaMemcpy(y.data(), out.p, y.size() * 4, cudaMemcpyDeviceToHost));
  f = fopen(argv[4], "wb");
  if (!f || fwrite(y.data(), 4, y.size(), f) != y.size()) {
    fprintf(stderr, "cannot write %s\n", argv[4]);
    return 1;
  }
  fclose(f);
  printf("ref_cuda run %dx%d -> %s\n", h, w, argv[4]);
  return 0;
}

int main(int argc, char** argv) {
  if (argc > 1 && strcmp(argv[1], "--run") == 0) return run_file(argc, argv);
  const int side = argc > 1 ? atoi(argv[1]) : 512;
  const int passes = argc > 2 ? atoi(argv[2]) : 5;
  const int warmup = argc > 3 ? atoi(argv[3]) : 2;
  if (side < 8 || side % 8 || passes < 1 || warmup < 0) {
    fprintf(stderr, "usage: ref_cuda_bench [side (multiple of 8)] [passes] [warmup]\n");
    return 2;
  }
  CK(cudaStreamCreateWithFlags(&g_st, cudaStreamNonBlocking));
  if (side > 1024) {
    fprintf(stderr, "side > 1024: one pass's activations would not fit the arena\n");
    return 2;
  }
  // every intermediate of a pass gets its own block (as with the reference's
  // allocator, nothing is reused within a pass): ~16,000 floats per input pixel
  g_arena.cap = (size_t)side * side * 4 * 16000;
  CK(cudaMalloc(&g_arena.base, g_arena.cap));
  Net net = build_net();
  Acts in{nullptr, 4, side, side};
  CK(cudaMalloc(&in.p, (size_t)in.n() * 4));
  h_fill<<<grid_for(in.n(), BLOCK), BLOCK>>>(in.p, in.n(), 12345u, 1.0f);
  CK(cudaDeviceSynchronize());
  for (int i = 0; i < warmup; i++) forward(net, in);
  CK(cudaStreamSynchronize(g_st));
  CK(cudaGetLastError());
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0, g_st));
  for (int i = 0; i < passes; i++) forward(net, in);
  CK(cudaEventRecord(e1, g_st));
  CK(cudaEventSynchronize(e1));
  CK(cudaGetLastError());
  float ms = 0.f;
  CK(cudaEventElapsedTime(&ms, e0, e1));
  printf("ref_cuda side=%d ms_per_pass=%.3f passes=%d arena_used_gb=%.2f\n", side, ms / passes, passes,
         g_arena.used / 1e9);
  return 0;
}
