// lama_rfft2_noalloc: the FourierUnit's forward transform (the two-pass rfft2
// of fft.cu) for callers that cannot allocate device memory.
//
// The two-pass transform needs an intermediate of batch*channels*(w/2+1)*h
// complex values plus two twiddle tables.  Here they live in one file-scope
// device array of fixed size, shared by every call in the process: nothing
// in it has to start at zero (the intermediate is fully written by the row
// pass before the column pass reads it, and each call writes the twiddle
// tables it reads with a small kernel first), and calls whose GPU work
// overlaps in time - on different streams, or from several host threads -
// race on it.  The entry point calls no cudaMalloc, cudaFree or other
// allocating routine.  Host code cannot use the array's name as a device
// pointer: the first call on each device, with that device current, looks up
// its address (cudaGetSymbolAddress) and sets the kernels' shared-memory
// limit; that first call belongs before any stream capture on the device.
// With CUDA's lazy module loading (the default) the array's device memory is
// claimed by that first look-up, not when the library is loaded, so a caller
// that reserves the rest of the GPU for its own pool makes its first call
// before reserving it.  A set-up that failed (for example for lack of memory)
// is not remembered: the next call on that device tries again.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdint>
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
  bool ready = false;
  float2* scratch = nullptr;
};
DeviceSlot g_slots[kMaxDevices];
std::mutex g_setup_mutex;

// Per device, with that device current, until it succeeds once: the array's
// device address and the kernels' shared-memory attribute.
cudaError_t setup(int device, float2** scratch) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceSlot& s = g_slots[device];
  if (!s.ready) {
    float2* p = nullptr;
    cudaError_t st = cudaGetSymbolAddress((void**)&p, g_scratch);
    if (st == cudaSuccess) st = (cudaError_t)fft_prepare(kSmem);
    if (st != cudaSuccess) {
      cudaGetLastError();  // clear the (non-sticky) error so the caller's next CUDA call does not report it
      return st;
    }
    s.scratch = p;
    s.ready = true;
  }
  *scratch = s.scratch;
  return cudaSuccess;
}

// Twiddle tables t[k] = (cos, sin)(2 pi k / n) of both plane sides, computed
// in double and rounded to float (as the engine's host-built tables are).
__global__ void k_noalloc_twiddles(float2* tw_h, int h, float2* tw_w, int w) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < h) {
    double sn, cs;
    sincospi(2.0 * (double)i / (double)h, &sn, &cs);
    tw_h[i] = make_float2((float)cs, (float)sn);
  }
  if (i < w) {
    double sn, cs;
    sincospi(2.0 * (double)i / (double)w, &sn, &cs);
    tw_w[i] = make_float2((float)cs, (float)sn);
  }
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
  // the row pass reads feat as floats and the column pass stores the
  // spectrum as pairs of bf16 (4-byte words)
  if (((uintptr_t)d_feat & 3) || ((uintptr_t)d_spec & 3))
    return fail(err, err_len, LAMA_EINVAL, "d_feat and d_spec must be 4-byte aligned");
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
    p.tmp = scratch;
    p.tw_h = scratch + kScratchComplex;
    p.tw_w = scratch + kScratchComplex + kMaxSide;
    p.feat = d_feat;
    p.spec = d_spec;
    p.spec_part = (long long)batch * h * wh * 2 * channels;
    const int n = h > w ? h : w;
    k_noalloc_twiddles<<<(n + 255) / 256, 256, 0, st>>>((float2*)p.tw_h, h, (float2*)p.tw_w, w);
    ce = cudaGetLastError();
    if (ce == cudaSuccess) ce = (cudaError_t)launch_rfft2(p, st);
    if (ce != cudaSuccess) rc = fail(err, err_len, LAMA_ECUDA, "rfft2 launch: %s", cudaGetErrorString(ce));
  }
  if (prev >= 0 && prev != device) cudaSetDevice(prev);
  return rc;
}
