// CPU ORACLE - test infrastructure only, never the product path.
//
// A restatement in C++ of the reference's CPU engine for the big-lama
// generator forward pass (lama-rs/src/cpu.rs), used as the parity checker for
// the B200 engine and as the timed CPU baseline.  Only tests/, the smoke check
// and bench.py's cpu_baseline / reference legs load this library.
//
// Parity status: the reference ships no golden vectors and its Rust engine
// cannot be built offline (no cargo, and the `lightgpu` git dependency is not
// vendored).  This restatement is pinned against an independent PyTorch
// restatement (oracle/torch_ref.py), against torch.fft, and against the
// reference's own CUDA kernels: oracle/ref_cuda_bench.cu compiles
// lama-rs/cuda/lama.cu from the reference checkout and runs it in the launch
// order of cuda::run with the same weights (only the absent toolkit's FFT and
// elementwise kernels are stand-ins); full passes agree to 1e-4
// (tests/test_gpu_ref_cuda.py).  No reference-written output file exists to
// compare against.
//
// Arithmetic follows cpu.rs exactly so that it should be bit-identical to the
// Rust engine:
//   * f32 accumulation in the same loop order (ci, ky, kx innermost), each
//     product rounded before the add - Rust never contracts a*b+c, and this
//     file is compiled with -ffp-contract=off;
//   * BatchNorm folded to scale/shift in f32 (cpu.rs:45-64), applied as
//     x*s + t (cpu.rs:66-76);
//   * the FFT in f64: iterative radix-2 with the same twiddle recurrence for
//     powers of two (cpu.rs:888-927), Bluestein with the same chirp tables
//     otherwise (cpu.rs:947-1011), rows then columns (cpu.rs:846-871), ortho
//     scale 1/sqrt(hw) on each side, 2-D Hermitian completion in the inverse
//     (cpu.rs:801-837);
//   * sigmoid 1/(1+exp(-x)) in f32 (cpu.rs:384-388).
// Threading (OpenMP over the axes rayon splits) never changes a result: every
// output element is produced by one sequential loop.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <stdexcept>
#include <memory>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ------------------------------------------------------------ weight store
// safetensors: u64 LE header length, JSON header, payloads.  Minimal JSON
// scanner for the {name: {"dtype":..,"shape":[..],"data_offsets":[a,b]}} form.
struct TensorInfo {
  std::vector<size_t> shape;
  size_t a = 0, b = 0;
  std::string dtype;
};

struct Store {
  std::vector<uint8_t> data;
  size_t base = 0;
  std::map<std::string, TensorInfo> t;

  bool open(const char* path, std::string& err) {
    FILE* f = fopen(path, "rb");
    if (!f) { err = std::string(path) + ": cannot open"; return false; }
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    data.resize((size_t)n);
    if (n > 0 && fread(data.data(), 1, (size_t)n, f) != (size_t)n) { fclose(f); err = "short read"; return false; }
    fclose(f);
    if (n < 8) { err = "file too short"; return false; }
    uint64_t hl = 0;
    memcpy(&hl, data.data(), 8);
    if (8 + hl > (uint64_t)n) { err = "header length past end of file"; return false; }
    base = 8 + hl;
    std::string h((const char*)data.data() + 8, hl);
    size_t i = 0;
    auto skip = [&]() { while (i < h.size() && (h[i] == ' ' || h[i] == '\n' || h[i] == '\r' || h[i] == '\t' || h[i] == ',' || h[i] == ':')) i++; };
    auto str = [&]() { std::string s; if (h[i] != '"') return s; i++; while (i < h.size() && h[i] != '"') { if (h[i] == '\\') i++; s += h[i++]; } i++; return s; };
    auto skipval = [&]() {  // skip a JSON value (object/array/string/number)
      int depth = 0;
      do {
        if (h[i] == '"') { str(); continue; }
        if (h[i] == '{' || h[i] == '[') depth++;
        if (h[i] == '}' || h[i] == ']') depth--;
        i++;
      } while (i < h.size() && depth > 0);
    };
    skip();
    if (h[i] != '{') { err = "bad header"; return false; }
    i++;
    while (true) {
      skip();
      if (i >= h.size() || h[i] == '}') break;
      std::string name = str();
      skip();
      if (name == "__metadata__") { skipval(); continue; }
      TensorInfo ti;
      if (h[i] != '{') { err = "bad tensor entry"; return false; }
      i++;
      while (true) {
        skip();
        if (h[i] == '}') { i++; break; }
        std::string key = str();
        skip();
        if (key == "dtype") ti.dtype = str();
        else if (key == "shape" || key == "data_offsets") {
          std::vector<size_t> v;
          i++;  // [
          while (true) {
            skip();
            if (h[i] == ']') { i++; break; }
            size_t x = 0;
            while (h[i] >= '0' && h[i] <= '9') x = x * 10 + (h[i++] - '0');
            v.push_back(x);
          }
          if (key == "shape") ti.shape = v;
          else if (v.size() == 2) { ti.a = v[0]; ti.b = v[1]; }
        } else skipval();
      }
      if (ti.dtype != "F32") { err = "tensor " + name + " is " + ti.dtype + ", not F32"; return false; }
      if (base + ti.b > data.size() || ti.a > ti.b) { err = "tensor " + name + " outside the file"; return false; }
      t[name] = ti;
    }
    if (t.empty()) { err = "no tensors found"; return false; }
    return true;
  }
  bool has(const std::string& n) const { return t.count(n) != 0; }
  const TensorInfo& info(const std::string& n) const {
    auto it = t.find(n);
    if (it == t.end()) throw std::runtime_error("missing tensor in weight blob: " + n);
    return it->second;
  }
  std::vector<float> f32(const std::string& n) const {
    const TensorInfo& ti = info(n);
    std::vector<float> v((ti.b - ti.a) / 4);
    memcpy(v.data(), data.data() + base + ti.a, ti.b - ti.a);
    return v;
  }
};

// ------------------------------------------------------------ activations
struct Acts {
  size_t c = 0, h = 0, w = 0;
  std::vector<float> data;
  Acts() {}
  Acts(size_t c_, size_t h_, size_t w_) : c(c_), h(h_), w(w_), data(c_ * h_ * w_, 0.f) {}
  const float* plane(size_t ci) const { return data.data() + ci * h * w; }
};

// image.rs:159-169
static size_t reflect_index(long long i, size_t n) {
  if (n == 1) return 0;
  long long period = 2 * ((long long)n - 1);
  long long m = ((i % period) + period) % period;
  if (m >= (long long)n) m = period - m;
  return (size_t)m;
}

// ------------------------------------------------------------ layers
struct Bn {  // cpu.rs:39-77
  std::vector<float> scale, shift;
  void load(const Store& s, const std::string& p, size_t channels) {
    auto w = s.f32(p + ".weight"), b = s.f32(p + ".bias");
    auto mean = s.f32(p + ".running_mean"), var = s.f32(p + ".running_var");
    if (w.size() != channels || b.size() != channels || mean.size() != channels || var.size() != channels)
      throw std::runtime_error("BatchNorm " + p + ": expected " + std::to_string(channels) + " channels");
    scale.resize(channels);
    shift.resize(channels);
    for (size_t i = 0; i < channels; i++) {
      float sd = std::sqrt(var[i] + 1e-5f);
      float sc = w[i] / sd;
      scale[i] = sc;
      float ms = mean[i] * sc;
      shift[i] = b[i] - ms;
    }
  }
  void apply(Acts& a) const {
    size_t plane = a.h * a.w;
#pragma omp parallel for schedule(static)
    for (long long ci = 0; ci < (long long)a.c; ci++) {
      float s = scale[ci], t = shift[ci];
      float* p = a.data.data() + ci * plane;
      for (size_t i = 0; i < plane; i++) { float v = p[i] * s; p[i] = v + t; }
    }
  }
};

static void relu_inplace(Acts& a) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)a.data.size(); i++)
    if (a.data[i] < 0.f) a.data[i] = 0.f;
}

static void sigmoid_inplace(Acts& a) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)a.data.size(); i++) {
    float e = std::exp(-a.data[i]);
    float d = 1.0f + e;
    a.data[i] = 1.0f / d;
  }
}

static void add_inplace(Acts& dst, const Acts& src) {  // cpu.rs:702-708
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)dst.data.size(); i++) dst.data[i] = dst.data[i] + src.data[i];
}

struct Conv2dW {  // cpu.rs:80-192
  std::vector<float> w, bias;
  bool has_bias = false;
  size_t cin = 0, cout = 0, kh = 0, kw = 0;

  void load(const Store& s, const std::string& p) {
    const TensorInfo& ti = s.info(p + ".weight");
    w = s.f32(p + ".weight");
    cout = ti.shape[0]; cin = ti.shape[1]; kh = ti.shape[2]; kw = ti.shape[3];
    if (s.has(p + ".bias")) { bias = s.f32(p + ".bias"); has_bias = true; }
  }

  Acts forward_pad(const Acts& src, size_t pad, size_t stride, bool reflect) const {
    size_t h = src.h, wd = src.w;
    size_t oh = (h + 2 * pad - kh) / stride + 1;
    size_t ow = (wd + 2 * pad - kw) / stride + 1;
    Acts out(cout, oh, ow);
    size_t k = kh * kw;
#pragma omp parallel for schedule(dynamic, 4)
    for (long long row = 0; row < (long long)(cout * oh); row++) {
      size_t co = row / oh, oy = row % oh;
      float* dst = out.data.data() + row * ow;
      const float* wp = w.data() + co * cin * k;
      float b = has_bias ? bias[co] : 0.0f;
      for (size_t ox = 0; ox < ow; ox++) {
        float acc = b;
        for (size_t ci = 0; ci < cin; ci++) {
          const float* sp = src.data.data() + ci * h * wd;
          const float* kp = wp + ci * k;
          for (size_t ky = 0; ky < kh; ky++) {
            size_t iy = oy * stride + ky;
            size_t sy;
            if (iy < pad) {
              if (!reflect) continue;
              sy = reflect_index((long long)iy - (long long)pad, h);
            } else if (iy - pad >= h) {
              if (!reflect) continue;
              sy = reflect_index((long long)iy - (long long)pad, h);
            } else {
              sy = iy - pad;
            }
            const float* srow = sp + sy * wd;
            const float* krow = kp + ky * kw;
            for (size_t kx = 0; kx < kw; kx++) {
              size_t ix = ox * stride + kx;
              size_t sx;
              if (ix < pad || ix - pad >= wd) {
                if (!reflect) continue;
                sx = reflect_index((long long)ix - (long long)pad, wd);
              } else {
                sx = ix - pad;
              }
              float prod = krow[kx] * srow[sx];
              acc = acc + prod;
            }
          }
        }
        dst[ox] = acc;
      }
    }
    return out;
  }

  Acts forward_1x1(const Acts& src) const {
    size_t plane = src.h * src.w;
    Acts out(cout, src.h, src.w);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long co = 0; co < (long long)cout; co++) {
      const float* wp = w.data() + co * cin;
      float b = has_bias ? bias[co] : 0.0f;
      float* dst = out.data.data() + co * plane;
      for (size_t i = 0; i < plane; i++) {
        float acc = b;
        for (size_t ci = 0; ci < cin; ci++) {
          float prod = wp[ci] * src.data[ci * plane + i];
          acc = acc + prod;
        }
        dst[i] = acc;
      }
    }
    return out;
  }
};

// ------------------------------------------------------------ FFT (f64)
static void fft_radix2(double* re, double* im, size_t n, bool inverse) {  // cpu.rs:888-927
  size_t j = 0;
  for (size_t i = 1; i < n; i++) {
    size_t bit = n >> 1;
    while (j & bit) { j ^= bit; bit >>= 1; }
    j |= bit;
    if (i < j) { std::swap(re[i], re[j]); std::swap(im[i], im[j]); }
  }
  double sign = inverse ? 1.0 : -1.0;
  for (size_t len = 2; len <= n; len <<= 1) {
    double ang = sign * 2.0 * M_PI / (double)len;
    double wr = std::cos(ang), wi = std::sin(ang);
    for (size_t i = 0; i < n; i += len) {
      double cr = 1.0, ci = 0.0;
      for (size_t k = 0; k < len / 2; k++) {
        double ur = re[i + k], ui = im[i + k];
        double a = re[i + k + len / 2], b = im[i + k + len / 2];
        double vr = a * cr - b * ci;
        double vi = a * ci + b * cr;
        re[i + k] = ur + vr;
        im[i + k] = ui + vi;
        re[i + k + len / 2] = ur - vr;
        im[i + k + len / 2] = ui - vi;
        double ncr = cr * wr - ci * wi;
        ci = cr * wi + ci * wr;
        cr = ncr;
      }
    }
  }
}

struct Bluestein {
  size_t m = 0;
  std::vector<double> wr, wi, br, bi;
};

static size_t next_pow2(size_t v) { size_t p = 1; while (p < v) p <<= 1; return p; }

static const Bluestein& bluestein_tables(size_t n, bool inverse) {  // cpu.rs:947-980
  static thread_local std::map<std::pair<size_t, bool>, std::unique_ptr<Bluestein>> cache;
  auto key = std::make_pair(n, inverse);
  auto it = cache.find(key);
  if (it != cache.end()) return *it->second;
  auto t = std::make_unique<Bluestein>();
  double sign = inverse ? 1.0 : -1.0;
  t->wr.resize(n);
  t->wi.resize(n);
  for (size_t j = 0; j < n; j++) {
    double jm = (double)(((long long)j * (long long)j) % (2 * (long long)n));
    double ang = sign * M_PI * jm / (double)n;
    t->wr[j] = std::cos(ang);
    t->wi[j] = std::sin(ang);
  }
  size_t m = next_pow2(2 * n - 1);
  t->m = m;
  t->br.assign(m, 0.0);
  t->bi.assign(m, 0.0);
  t->br[0] = t->wr[0];
  t->bi[0] = t->wi[0];
  for (size_t j = 1; j < n; j++) {
    t->br[j] = t->wr[j]; t->bi[j] = t->wi[j];
    t->br[m - j] = t->wr[j]; t->bi[m - j] = t->wi[j];
  }
  fft_radix2(t->br.data(), t->bi.data(), m, false);
  auto& ref = *t;
  cache[key] = std::move(t);
  return ref;
}

static void fft_bluestein(double* re, double* im, size_t n, bool inverse) {  // cpu.rs:984-1011
  const Bluestein& t = bluestein_tables(n, inverse);
  size_t m = t.m;
  std::vector<double> ar(m, 0.0), ai(m, 0.0);
  for (size_t j = 0; j < n; j++) {
    double p1 = re[j] * t.wr[j], p2 = im[j] * t.wi[j];
    ar[j] = p1 + p2;
    double p3 = im[j] * t.wr[j], p4 = re[j] * t.wi[j];
    ai[j] = p3 - p4;
  }
  fft_radix2(ar.data(), ai.data(), m, false);
  for (size_t i = 0; i < m; i++) {
    double xr = ar[i] * t.br[i] - ai[i] * t.bi[i];
    double xi = ar[i] * t.bi[i] + ai[i] * t.br[i];
    ar[i] = xr;
    ai[i] = xi;
  }
  fft_radix2(ar.data(), ai.data(), m, true);
  double inv_m = 1.0 / (double)m;
  for (size_t j = 0; j < n; j++) {
    double cr = ar[j] * inv_m, ci = ai[j] * inv_m;
    re[j] = cr * t.wr[j] + ci * t.wi[j];
    im[j] = ci * t.wr[j] - cr * t.wi[j];
  }
}

static void fft1(double* re, double* im, size_t n, bool inverse) {  // cpu.rs:875-885
  if (n <= 1) return;
  if ((n & (n - 1)) == 0) fft_radix2(re, im, n, inverse);
  else fft_bluestein(re, im, n, inverse);
}

static void fft2(double* re, double* im, size_t h, size_t w, bool inverse) {  // cpu.rs:846-871
  std::vector<double> rr(w), ii(w);
  for (size_t y = 0; y < h; y++) {
    memcpy(rr.data(), re + y * w, w * 8);
    memcpy(ii.data(), im + y * w, w * 8);
    fft1(rr.data(), ii.data(), w, inverse);
    memcpy(re + y * w, rr.data(), w * 8);
    memcpy(im + y * w, ii.data(), w * 8);
  }
  std::vector<double> cr(h), ci(h);
  for (size_t x = 0; x < w; x++) {
    for (size_t y = 0; y < h; y++) { cr[y] = re[y * w + x]; ci[y] = im[y * w + x]; }
    fft1(cr.data(), ci.data(), h, inverse);
    for (size_t y = 0; y < h; y++) { re[y * w + x] = cr[y]; im[y * w + x] = ci[y]; }
  }
}

// cpu.rs:769-783: writes [2][h][w/2+1] (real plane, then imaginary plane).
static void rfft2_ortho(const float* src, size_t h, size_t w, float* dst) {
  size_t hw = w / 2 + 1;
  std::vector<double> re(h * w, 0.0), im(h * w, 0.0);
  for (size_t i = 0; i < h * w; i++) re[i] = (double)src[i];
  fft2(re.data(), im.data(), h, w, false);
  double scale = 1.0 / std::sqrt((double)(h * w));
  for (size_t y = 0; y < h; y++)
    for (size_t x = 0; x < hw; x++) {
      dst[y * hw + x] = (float)(re[y * w + x] * scale);
      dst[h * hw + y * hw + x] = (float)(im[y * w + x] * scale);
    }
}

// cpu.rs:801-837
static void irfft2_ortho(const float* src, size_t h, size_t w, float* dst) {
  size_t hw = w / 2 + 1;
  std::vector<double> re(h * w, 0.0), im(h * w, 0.0);
  for (size_t y = 0; y < h; y++)
    for (size_t x = 0; x < hw; x++) {
      re[y * w + x] = (double)src[y * hw + x];
      im[y * w + x] = (double)src[h * hw + y * hw + x];
    }
  for (size_t y = 0; y < h; y++)
    for (size_t x = hw; x < w; x++) {
      size_t xm = w - x;
      if (xm >= hw) continue;
      size_t ym = (h - y) % h;
      re[y * w + x] = re[ym * w + xm];
      im[y * w + x] = -im[ym * w + xm];
    }
  fft2(re.data(), im.data(), h, w, true);
  double scale = 1.0 / std::sqrt((double)(h * w));
  for (size_t i = 0; i < h * w; i++) dst[i] = (float)(re[i] * scale);
}

struct FourierUnit {  // cpu.rs:210-309
  Conv2dW conv;
  Bn bn;
  size_t half = 0;
  Acts forward(const Acts& x) const {
    size_t h = x.h, w = x.w, hw = w / 2 + 1;
    Acts s(2 * half, h, hw);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long c = 0; c < (long long)half; c++)
      rfft2_ortho(x.plane(c), h, w, s.data.data() + c * 2 * h * hw);
    Acts cv = conv.forward_1x1(s);
    bn.apply(cv);
    relu_inplace(cv);
    Acts out(half, h, w);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long c = 0; c < (long long)half; c++)
      irfft2_ortho(cv.data.data() + 2 * c * h * hw, h, w, out.data.data() + c * h * w);
    return out;
  }
};

struct Spectral {  // cpu.rs:197-266
  Conv2dW conv1, conv2;
  Bn bn1;
  FourierUnit fu;
  size_t half = 0;
  Acts forward(const Acts& x) const {
    Acts feat = conv1.forward_1x1(x);
    bn1.apply(feat);
    relu_inplace(feat);
    Acts f = fu.forward(feat);
    Acts sum(half, feat.h, feat.w);
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)sum.data.size(); i++) sum.data[i] = feat.data[i] + f.data[i];
    return conv2.forward_1x1(sum);
  }
};

struct ConvT {  // cpu.rs:313-374
  std::vector<float> w, bias;
  size_t cin = 0, cout = 0;
  void load(const Store& s, const std::string& p) {
    const TensorInfo& ti = s.info(p + ".weight");
    w = s.f32(p + ".weight");
    bias = s.f32(p + ".bias");
    cin = ti.shape[0];
    cout = ti.shape[1];
  }
  Acts forward(const Acts& src) const {
    size_t oh = src.h * 2, ow = src.w * 2;
    Acts out(cout, oh, ow);
#pragma omp parallel for schedule(dynamic, 1)
    for (long long co = 0; co < (long long)cout; co++) {
      float* dst = out.data.data() + co * oh * ow;
      float b = bias[co];
      for (size_t i = 0; i < oh * ow; i++) dst[i] = b;
      for (size_t ci = 0; ci < src.c; ci++) {
        const float* sp = src.plane(ci);
        const float* kp = w.data() + (ci * cout + co) * 9;
        for (size_t iy = 0; iy < src.h; iy++) {
          const float* row = sp + iy * src.w;
          for (size_t ix = 0; ix < src.w; ix++) {
            float v = row[ix];
            if (v == 0.0f) continue;
            for (size_t ky = 0; ky < 3; ky++) {
              size_t oy = iy * 2 + ky;
              if (oy == 0 || oy > oh) continue;
              float* drow = dst + (oy - 1) * ow;
              for (size_t kx = 0; kx < 3; kx++) {
                size_t ox = ix * 2 + kx;
                if (ox == 0 || ox > ow) continue;
                float prod = v * kp[ky * 3 + kx];
                drow[ox - 1] = drow[ox - 1] + prod;
              }
            }
          }
        }
      }
    }
    return out;
  }
};

// ------------------------------------------------------------ the net
struct FfcW {  // cpu.rs:417-432
  size_t kernel = 0, stride = 1, pad = 0;
  bool reflect = true;
  size_t in_local = 0, in_global = 0, out_local = 0, out_global = 0;
  std::unique_ptr<Conv2dW> l2l, l2g, g2l;
  std::unique_ptr<Spectral> spectral;
  std::unique_ptr<Bn> bn_l, bn_g;
  Acts conv(const Conv2dW& w, const Acts& src) const {
    if (kernel == 1) return w.forward_1x1(src);
    return w.forward_pad(src, pad, stride, reflect);
  }
};

enum StepKind { REFLECT_PAD, FFC, RES, CONCAT, UPSAMPLE, OUTCONV };
struct Step {
  StepKind kind;
  size_t pad = 0;
  std::unique_ptr<FfcW> ffc, res2;
  std::unique_ptr<ConvT> convt;
  std::unique_ptr<Bn> bn;
  std::unique_ptr<Conv2dW> out;
};

// model.rs:211-257
static std::unique_ptr<FfcW> load_ffc(const Store& s, size_t index, size_t sub, size_t cin, size_t cout,
                                      size_t kernel, size_t stride, float rgin, float rgout, bool pad0) {
  auto f = std::make_unique<FfcW>();
  f->in_global = (size_t)((float)cin * rgin);
  f->out_global = (size_t)((float)cout * rgout);
  f->in_local = cin - f->in_global;
  f->out_local = cout - f->out_global;
  f->kernel = kernel;
  f->stride = stride;
  f->pad = pad0 ? 0 : kernel / 2;
  f->reflect = true;
  std::string prefix = "model." + std::to_string(index);
  std::string fp = sub == 0 ? prefix + ".ffc" : sub == 1 ? prefix + ".conv1.ffc" : prefix + ".conv2.ffc";
  std::string partial = sub == 0 ? prefix : sub == 1 ? prefix + ".conv1" : prefix + ".conv2";
  if (f->in_local && f->out_local) { f->l2l = std::make_unique<Conv2dW>(); f->l2l->load(s, fp + ".convl2l"); }
  if (f->in_local && f->out_global) { f->l2g = std::make_unique<Conv2dW>(); f->l2g->load(s, fp + ".convl2g"); }
  if (f->in_global && f->out_local) { f->g2l = std::make_unique<Conv2dW>(); f->g2l->load(s, fp + ".convg2l"); }
  if (f->in_global && f->out_global) {
    auto sp = std::make_unique<Spectral>();
    std::string g = fp + ".convg2g";
    sp->half = f->out_global / 2;
    sp->conv1.load(s, g + ".conv1.0");
    sp->bn1.load(s, g + ".conv1.1", sp->half);
    sp->conv2.load(s, g + ".conv2");
    sp->fu.conv.load(s, g + ".fu.conv_layer");
    sp->fu.bn.load(s, g + ".fu.bn", 2 * sp->half);
    sp->fu.half = sp->half;
    f->spectral = std::move(sp);
  }
  if (f->out_local) { f->bn_l = std::make_unique<Bn>(); f->bn_l->load(s, partial + ".bn_l", f->out_local); }
  if (f->out_global) { f->bn_g = std::make_unique<Bn>(); f->bn_g->load(s, partial + ".bn_g", f->out_global); }
  return f;
}

// cpu.rs:635-688
static void run_ffc(const FfcW& w, const Acts& local, const Acts* global, Acts& out_l, Acts& out_g, bool& has_g) {
  out_l = Acts();
  if (w.out_local > 0) {
    Acts acc;
    bool have = false;
    if (w.l2l) { acc = w.conv(*w.l2l, local); have = true; }
    if (w.g2l) {
      Acts o = w.conv(*w.g2l, *global);
      if (!have) { acc = std::move(o); have = true; }
      else add_inplace(acc, o);
    }
    if (w.bn_l) { w.bn_l->apply(acc); relu_inplace(acc); }
    out_l = std::move(acc);
  }
  has_g = false;
  if (w.out_global > 0) {
    Acts acc;
    bool have = false;
    if (w.l2g) { acc = w.conv(*w.l2g, local); have = true; }
    if (w.spectral) {
      Acts o = w.spectral->forward(*global);
      if (!have) { acc = std::move(o); have = true; }
      else add_inplace(acc, o);
    }
    if (w.bn_g) { w.bn_g->apply(acc); relu_inplace(acc); }
    out_g = std::move(acc);
    has_g = true;
  }
}

static Acts reflect_pad_acts(const Acts& a, size_t pad) {  // cpu.rs:718-738
  if (pad == 0) return a;
  Acts out(a.c, a.h + 2 * pad, a.w + 2 * pad);
  size_t oh = out.h, ow = out.w;
#pragma omp parallel for schedule(static)
  for (long long c = 0; c < (long long)a.c; c++) {
    const float* sp = a.plane(c);
    float* dst = out.data.data() + c * oh * ow;
    for (size_t y = 0; y < oh; y++) {
      size_t sy = reflect_index((long long)y - (long long)pad, a.h);
      for (size_t x = 0; x < ow; x++) {
        size_t sx = reflect_index((long long)x - (long long)pad, a.w);
        dst[y * ow + x] = sp[sy * a.w + sx];
      }
    }
  }
  return out;
}

static Acts concat(const Acts& a, const Acts& b) {
  Acts out(a.c + b.c, a.h, a.w);
  memcpy(out.data.data(), a.data.data(), a.data.size() * 4);
  memcpy(out.data.data() + a.data.size(), b.data.data(), b.data.size() * 4);
  return out;
}

struct Net {
  std::vector<Step> steps;
  std::string err;

  void load(const Store& s) {  // model.rs:135-207 + cpu.rs:460-482
    auto push_pad = [&](size_t p) { Step st; st.kind = REFLECT_PAD; st.pad = p; steps.push_back(std::move(st)); };
    auto push_ffc = [&](std::unique_ptr<FfcW> f) { Step st; st.kind = FFC; st.ffc = std::move(f); steps.push_back(std::move(st)); };
    push_pad(3);
    push_ffc(load_ffc(s, 1, 0, 4, 64, 7, 1, 0.f, 0.f, true));
    push_ffc(load_ffc(s, 2, 0, 64, 128, 3, 2, 0.f, 0.f, false));
    push_ffc(load_ffc(s, 3, 0, 128, 256, 3, 2, 0.f, 0.f, false));
    push_ffc(load_ffc(s, 4, 0, 256, 512, 3, 2, 0.f, 0.75f, false));
    for (size_t i = 5; i <= 22; i++) {
      Step st;
      st.kind = RES;
      st.ffc = load_ffc(s, i, 1, 512, 512, 3, 1, 0.75f, 0.75f, false);
      st.res2 = load_ffc(s, i, 2, 512, 512, 3, 1, 0.75f, 0.75f, false);
      steps.push_back(std::move(st));
    }
    { Step st; st.kind = CONCAT; steps.push_back(std::move(st)); }
    const size_t ups[3][4] = {{24, 25, 512, 256}, {27, 28, 256, 128}, {30, 31, 128, 64}};
    for (auto& u : ups) {
      Step st;
      st.kind = UPSAMPLE;
      st.convt = std::make_unique<ConvT>();
      st.convt->load(s, "model." + std::to_string(u[0]));
      st.bn = std::make_unique<Bn>();
      st.bn->load(s, "model." + std::to_string(u[1]), u[3]);
      steps.push_back(std::move(st));
    }
    push_pad(3);
    Step st;
    st.kind = OUTCONV;
    st.out = std::make_unique<Conv2dW>();
    st.out->load(s, "model.34");
    steps.push_back(std::move(st));
  }

  // cpu.rs:485-558.  Steps [first, last) run; `local`/`global` are state in/out.
  void run_steps(size_t first, size_t last, Acts& local, Acts& global, bool& has_g,
                 long long dump_after = -1, std::vector<float>* dump = nullptr) const {
    for (size_t sn = first; sn < last && sn < steps.size(); sn++) {
      const Step& st = steps[sn];
      switch (st.kind) {
        case REFLECT_PAD:
          local = reflect_pad_acts(local, st.pad);
          if (has_g) global = reflect_pad_acts(global, st.pad);
          break;
        case FFC: {
          Acts nl, ng;
          bool hg;
          run_ffc(*st.ffc, local, has_g ? &global : nullptr, nl, ng, hg);
          local = std::move(nl);
          global = std::move(ng);
          has_g = hg;
          break;
        }
        case RES: {
          Acts nl, ng, nl2, ng2;
          bool hg, hg2;
          run_ffc(*st.ffc, local, has_g ? &global : nullptr, nl, ng, hg);
          run_ffc(*st.res2, nl, hg ? &ng : nullptr, nl2, ng2, hg2);
          add_inplace(local, nl2);
          if (has_g && hg2) add_inplace(global, ng2);
          else if (hg2) { global = std::move(ng2); has_g = true; }
          break;
        }
        case CONCAT:
          if (has_g) { local = concat(local, global); global = Acts(); has_g = false; }
          break;
        case UPSAMPLE: {
          Acts a = st.convt->forward(local);
          st.bn->apply(a);
          relu_inplace(a);
          local = std::move(a);
          global = Acts();
          has_g = false;
          break;
        }
        case OUTCONV:
          local = st.out->forward_pad(local, 0, 1, false);
          sigmoid_inplace(local);
          break;
      }
      if (dump && (long long)sn == dump_after) {
        dump->assign(local.data.begin(), local.data.end());
        if (has_g) dump->insert(dump->end(), global.data.begin(), global.data.end());
      }
    }
  }
};

struct Handle {
  Store store;
  Net net;
  std::string err;
};

}  // namespace

extern "C" {

// Open a weight file and resolve the network (cpu.rs:460-482).  NULL on error,
// with the message in `err`.
void* oracle_open(const char* path, char* err, int errlen) {
  auto h = std::make_unique<Handle>();
  std::string e;
  try {
    if (!h->store.open(path, e)) throw std::runtime_error(e);
    h->net.load(h->store);
  } catch (const std::exception& ex) {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", ex.what());
    return nullptr;
  }
  return h.release();
}

void oracle_close(void* p) { delete (Handle*)p; }

int oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

// Full forward: `in` is [4][h][w], `out` is [3][h][w] (cpu.rs:741-751).
int oracle_forward(void* p, const float* in, int h, int w, float* out) {
  auto* H = (Handle*)p;
  Acts local(4, (size_t)h, (size_t)w), global;
  memcpy(local.data.data(), in, sizeof(float) * 4 * (size_t)h * (size_t)w);
  bool has_g = false;
  H->net.run_steps(0, H->net.steps.size(), local, global, has_g);
  if (local.c != 3 || local.h != (size_t)h || local.w != (size_t)w) return -1;
  memcpy(out, local.data.data(), local.data.size() * 4);
  return 0;
}

// Forward with the LAMA_DUMP_STEP capture (cpu.rs:488-546): the local (+global)
// activation after step `step` is copied to `dump` (capacity in floats); the
// number of floats is returned through `n`.
int oracle_forward_dump(void* p, const float* in, int h, int w, int step, float* dump, long long cap,
                        long long* n) {
  auto* H = (Handle*)p;
  Acts local(4, (size_t)h, (size_t)w), global;
  memcpy(local.data.data(), in, sizeof(float) * 4 * (size_t)h * (size_t)w);
  bool has_g = false;
  std::vector<float> d;
  H->net.run_steps(0, (size_t)step + 1, local, global, has_g, step, &d);
  *n = (long long)d.size();
  if ((long long)d.size() > cap) return -1;
  memcpy(dump, d.data(), d.size() * 4);
  return 0;
}

// The 18-resblock stack alone (config 1): local [128][h][w] and global
// [384][h][w] are updated in place.  Runs plan steps 5 .. 5+nblocks.
int oracle_resblocks(void* p, float* local_io, float* global_io, int h, int w, int nblocks) {
  auto* H = (Handle*)p;
  Acts local(128, (size_t)h, (size_t)w), global(384, (size_t)h, (size_t)w);
  memcpy(local.data.data(), local_io, local.data.size() * 4);
  memcpy(global.data.data(), global_io, global.data.size() * 4);
  bool has_g = true;
  H->net.run_steps(5, 5 + (size_t)nblocks, local, global, has_g);
  memcpy(local_io, local.data.data(), local.data.size() * 4);
  memcpy(global_io, global.data.data(), global.data.size() * 4);
  return 0;
}

// Plane transforms (cpu.rs:769-837) for unit tests.
void oracle_rfft2(const float* src, int h, int w, float* dst) { rfft2_ortho(src, (size_t)h, (size_t)w, dst); }
void oracle_irfft2(const float* src, int h, int w, float* dst) { irfft2_ortho(src, (size_t)h, (size_t)w, dst); }

// build_input (lama-rs/src/main.rs:175-196): RGB premultiplied by (1-mask) and
// the mask, [4][h+pad_h][w+pad_w], reflect-extended to the padded size.
void oracle_build_input(const uint8_t* rgb, const uint8_t* mask, int h, int w, int pad_h, int pad_w,
                        float* out) {
  size_t oh = (size_t)(h + pad_h), ow = (size_t)(w + pad_w), plane = oh * ow;
  for (size_t y = 0; y < oh; y++) {
    size_t sy = reflect_index((long long)y, (size_t)h);
    for (size_t x = 0; x < ow; x++) {
      size_t sx = reflect_index((long long)x, (size_t)w);
      float m = (float)mask[sy * w + sx] / 255.0f;
      m = m > 0.0f ? 1.0f : 0.0f;
      size_t o = y * ow + x;
      for (size_t c = 0; c < 3; c++) {
        float v = (float)rgb[(sy * w + sx) * 3 + c] / 255.0f;
        float om = 1.0f - m;
        out[c * plane + o] = v * om;
      }
      out[3 * plane + o] = m;
    }
  }
}

// Composite + quantise (lama-rs/src/main.rs:272-307): masked pixels take the
// network output, clamped to [0,1], scaled by 255, +0.5, truncated; the rest
// copy the source bytes.  `out` is the [3][ph][pw] network output with
// ph/pw the padded size; the image is h x w.
void oracle_composite(const uint8_t* rgb, const uint8_t* mask, int h, int w, int ph, int pw,
                      const float* out, uint8_t* dst) {
  size_t plane = (size_t)ph * (size_t)pw;
  for (int y = 0; y < h; y++)
    for (int x = 0; x < w; x++) {
      size_t pi = (size_t)y * pw + x;
      size_t o = ((size_t)y * w + x) * 3;
      // mask_data at the padded index equals the source mask inside the image
      bool hole = mask[(size_t)y * w + x] > 0;
      if (!hole) { dst[o] = rgb[o]; dst[o + 1] = rgb[o + 1]; dst[o + 2] = rgb[o + 2]; continue; }
      for (int c = 0; c < 3; c++) {
        float v = out[c * plane + pi];
        v = std::min(std::max(v, 0.0f), 1.0f) * 255.0f;
        dst[o + c] = (uint8_t)(v + 0.5f);
      }
    }
}

}  // extern "C"
