// lama_rfft2_noalloc: the FourierUnit's forward transform (the two-pass rfft2
// of fft.cu) for callers that cannot allocate device memory.
//
// The two-pass transform needs an intermediate of batch*channels*(w/2+1)*h
// complex values plus two twiddle tables.  Here they live in one file-scope
// device array of fixed size, shared by every call in the process: nothing
// in it has to start at zero (the intermediate is fully written by the row
// pass before the column pass reads it, the tables are copied in by each
// call), and calls whose GPU work overlaps in time - on different streams,
// or from several host threads - race on it.  The entry point calls no
// cudaMalloc, cudaFree or other allocating routine.  Host code cannot use the
// array's name as a device pointer: the first call on each device, with that
// device current, looks up its address (cudaGetSymbolAddress) and sets the
// kernels' shared-memory limit; that first call belongs before any stream
// capture on the device.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "fft.cuh"
#include "lama_b200.h"

namespace lama {
namespace {

constexpr long long kScratchComplex = 1LL << 21;  // intermediate: 2,097,152 complex values (16 MiB)
constexpr int kMaxSide = 1024;                     // twiddle tables: h, w <= 1024
constexpr size_t kSmem = 160 * 1024;               // dynamic shared memory cap of the fft.cu kernels
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float2 g_scratch[kScratchComplex + 2 * kMaxSide];

struct DeviceSlot {
  std::once_flag once;
  cudaError_t status = cudaSuccess;
  float2* scratch = nullptr;
};
DeviceSlot g_slots[kMaxDevices];

// Once per device, with that device current: the array's device address and
// the kernels' shared-memory attribute.
cudaError_t setup(int device, float2** scratch) {
  DeviceSlot& s = g_slots[device];
  std::call_once(s.once, [&s] {
    s.status = cudaGetSymbolAddress((void**)&s.scratch, g_scratch);
    if (s.status == cudaSuccess) s.status = (cudaError_t)fft_prepare(kSmem);
  });
  *scratch = s.scratch;
  return s.status;
}

int fail(char* err, int err_len, int code, const char* fmt, ...) {
  if (err && err_len > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)err_len, fmt, ap);
    va_end(ap);
  }
  return code;
}

int log2_or_neg(int n) {
  if (n & (n - 1)) return -1;
  int l = 0;
  while ((1 << l) < n) l++;
  return l;
}

void fill_twiddles(float2* t, int n) {
  for (int k = 0; k < n; k++) {
    const double a = 2.0 * M_PI * (double)k / (double)n;
    t[k] = make_float2((float)std::cos(a), (float)std::sin(a));
  }
}

}  // namespace
}  // namespace lama

extern "C" int lama_rfft2_noalloc(int device, const float* d_feat, int batch, int channels, int h, int w,
                                  void* d_spec, void* stream, char* err, int err_len) {
  using namespace lama;
  if (err && err_len > 0) err[0] = 0;
  if (!d_feat || !d_spec) return fail(err, err_len, LAMA_EINVAL, "null input or output pointer");
  if (batch < 1 || channels < 1 || h < 1 || w < 1)
    return fail(err, err_len, LAMA_EINVAL, "batch, channels, h and w must be positive");
  if (channels > 65535) return fail(err, err_len, LAMA_EINVAL, "channels %d exceeds 65535", channels);
  if (h > kMaxSide || w > kMaxSide)
    return fail(err, err_len, LAMA_ESCRATCH, "plane %dx%d exceeds the fixed scratch limit of %d per side", h, w,
                kMaxSide);
  const int wh = w / 2 + 1;
  const long long need = (long long)batch * channels * wh * h;
  if (need > kScratchComplex)
    return fail(err, err_len, LAMA_ESCRATCH,
                "batch*channels*(w/2+1)*h = %lld complex values exceeds the fixed scratch of %lld", need,
                kScratchComplex);
  int ndev = 0;
  cudaError_t ce = cudaGetDeviceCount(&ndev);
  if (ce != cudaSuccess) return fail(err, err_len, LAMA_ECUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(ce));
  if (device < 0 || device >= ndev || device >= kMaxDevices)
    return fail(err, err_len, LAMA_EINVAL, "device %d not present (%d devices)", device, ndev);

  FftParams p{};
  p.batch = batch;
  p.c = channels;
  p.h = h;
  p.w = w;
  p.wh = wh;
  p.log2h = log2_or_neg(h);
  p.log2w = log2_or_neg(w);
  p.scale = (float)(1.0 / std::sqrt((double)h * (double)w));
  if (!fft_tiles(p, kSmem))
    return fail(err, err_len, LAMA_EUNSUPPORTED, "plane %dx%d needs more shared memory than the kernels have", h, w);

  int prev = -1;
  cudaGetDevice(&prev);
  if ((ce = cudaSetDevice(device)) != cudaSuccess)
    return fail(err, err_len, LAMA_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(ce));
  int rc = LAMA_OK;
  float2* scratch = nullptr;
  if ((ce = setup(device, &scratch)) != cudaSuccess) {
    rc = fail(err, err_len, LAMA_ECUDA, "scratch set-up on device %d: %s", device, cudaGetErrorString(ce));
  } else {
    const cudaStream_t st = (cudaStream_t)stream;
    float2 tw[2 * kMaxSide];
    fill_twiddles(tw, h);
    fill_twiddles(tw + kMaxSide, w);
    p.tmp = scratch;
    p.tw_h = scratch + kScratchComplex;
    p.tw_w = scratch + kScratchComplex + kMaxSide;
    p.feat = d_feat;
    p.spec = d_spec;
    p.spec_part = (long long)batch * h * wh * 2 * channels;
    // pageable source: each copy returns once tw has been consumed
    ce = cudaMemcpyAsync((void*)p.tw_h, tw, sizeof(float2) * (size_t)h, cudaMemcpyHostToDevice, st);
    if (ce == cudaSuccess)
      ce = cudaMemcpyAsync((void*)p.tw_w, tw + kMaxSide, sizeof(float2) * (size_t)w, cudaMemcpyHostToDevice, st);
    if (ce == cudaSuccess) ce = (cudaError_t)launch_rfft2(p, st);
    if (ce != cudaSuccess) rc = fail(err, err_len, LAMA_ECUDA, "rfft2 launch: %s", cudaGetErrorString(ce));
  }
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return rc;
}
