/*
 * lama_b200.h - C ABI of the B200 big-lama inpainting engine.
 *
 * The engine runs the big-lama FFC-ResNet generator forward pass on one
 * NVIDIA B200 (sm_100a).  It is the drop-in replacement for the reference
 * engine's operator boundary:
 *
 *   infer(store, plan, input: Vec<f32> [4][h][w], h, w, args) -> Result<Vec<f32> [3][h][w], String>
 *       lama-rs/src/main.rs:318-361
 *   cuda::run(store, model, &input, h, w) -> Result<Vec<f32>, String>
 *       lama-rs/src/cuda.rs:1542-1691
 *   WeightStore::open + cuda::load_steps
 *       lama-rs/src/weights.rs:80-106, lama-rs/src/cuda.rs:903-962
 *
 * Conventions (same as the reference):
 *   - buffers are owned by the caller; the engine never keeps a pointer past
 *     the call that received it;
 *   - the network input is [4][h][w] float, NCHW: RGB * (1 - mask), then the
 *     mask (0 or 1); h and w are multiples of 8 (main.rs:241-242);
 *   - the network output is [3][h][w] float, the sigmoid output before
 *     compositing;
 *   - every function returns 0 on success and a negative LAMA_E* code on
 *     failure; lama_last_error() gives the message (the reference's
 *     `Err(String)`).  There is no CPU fallback: a GPU failure is an error.
 *
 * Threading: an engine is bound to one device and is not thread-safe; engines
 * on different devices may be driven concurrently from different threads.
 *
 * Arithmetic: the reference is FP32.  Convolutions run on the tensor core as
 * three BF16 products of split operands (x = hi + lo) with FP32 accumulation,
 * which tracks FP32 to ~1e-5 relative per layer; transforms run in FP32.
 */
#ifndef LAMA_B200_H
#define LAMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lama_engine lama_engine;

enum {
  LAMA_OK = 0,
  LAMA_EINVAL = -1,   /* bad argument (size not a multiple of 8, null pointer, ...) */
  LAMA_EWEIGHTS = -2, /* weight file missing, truncated, not F32, wrong shape */
  LAMA_ECUDA = -3,    /* CUDA runtime / driver error */
  LAMA_EDEVICE = -4,  /* a kernel reported a device-side error (timeout, bad plan) */
  LAMA_ENOMEM = -5,   /* device allocation refused */
  LAMA_EUNSUPPORTED = -6,
  LAMA_ESCRATCH = -7  /* lama_rfft2_noalloc: request larger than its fixed scratch array */
};

/* Open the safetensors weight file and build the engine on CUDA device
 * `device`.  Replaces WeightStore::open (weights.rs:80-106: every tensor must
 * be F32 and inside the file) and cuda::load_steps (cuda.rs:903-962: BN
 * folding, weight upload).  On failure *out is still set when possible so
 * that lama_last_error() can report; close it with lama_close(). */
int lama_open(const char* weights_path, int device, lama_engine** out);

/* Forward pass on host buffers: in = [batch][4][h][w], out = [batch][3][h][w].
 * Replaces cuda::run (cuda.rs:1542-1691) / infer (main.rs:318-361); batch > 1
 * runs independent images in one pass. */
int lama_forward(lama_engine* e, const float* in, int batch, int h, int w, float* out);

/* Same with device pointers (inputs already in device memory), ordered on
 * the engine's stream; returns after the work is queued. */
int lama_forward_device(lama_engine* e, const float* d_in, int batch, int h, int w, float* d_out);

/* build_input + forward + composite on host u8 buffers: rgb [batch][h][w][3],
 * mask [batch][h][w] (non-zero = hole), out_rgb [batch][h][w][3].  Any h, w
 * >= 1: the network runs at the next multiple of 8 with reflect extension
 * (main.rs:175-196, 241-242); masked pixels take round(clamp(v,0,1)*255)
 * and every other byte is copied from rgb (main.rs:272-307). */
int lama_inpaint_u8(lama_engine* e, const uint8_t* rgb, const uint8_t* mask, int batch, int h, int w,
                    uint8_t* out_rgb);

/* lama_inpaint_u8 over n images from host memory, `chunk` images per pass,
 * with the host<->device copies of one chunk overlapping the pass of the
 * previous one (a copy stream and two staging sets; copies are asynchronous
 * when rgb, mask and out_rgb are page-locked).  Same bytes as lama_inpaint_u8
 * on each chunk.  No counterpart in the reference (its engine takes one image
 * per call); it is the serving form of `infer` + composite for many images. */
int lama_inpaint_u8_stream(lama_engine* e, const uint8_t* rgb, const uint8_t* mask, int n, int h, int w, int chunk,
                           uint8_t* out_rgb);

/* Same with device pointers, ordered on the engine's stream. */
int lama_inpaint_u8_device(lama_engine* e, const uint8_t* d_rgb, const uint8_t* d_mask, int batch, int h, int w,
                           uint8_t* d_out_rgb);

/* The FFC resblock stack alone (plan steps model.5 .. model.22,
 * cpu.rs:508-518 / cuda.rs:1590-1606): local [batch][128][h][w] and global
 * [batch][384][h][w] in, the same shapes out, host buffers. */
int lama_resblocks(lama_engine* e, const float* local_in, const float* global_in, int batch, int h, int w,
                   int nblocks, float* local_out, float* global_out);

/* Device-pointer variant of lama_resblocks. */
int lama_resblocks_device(lama_engine* e, const float* d_local_in, const float* d_global_in, int batch, int h,
                          int w, int nblocks, float* d_local_out, float* d_global_out);

/* Tile policy of the convolution GEMMs for plans built after this call
 * (cached plans are dropped): LAMA_TILING_AUTO uses pixel-major tiles,
 * shared by CTA pairs when a launch has at least two M tiles per SM or when a
 * small launch of 3x3-style taps can use the row union (with split K),
 * LAMA_TILING_SWAPPED uses channel-major tiles (M = 128 output channels,
 * N = 256 pixels) wherever they apply, LAMA_TILING_PIXEL uses single-CTA
 * pixel-major tiles only, LAMA_TILING_PAIRED uses pixel-major tiles shared by
 * CTA pairs (256 pixels x 128 channels over two SMs) wherever they apply.  All
 * policies compute the same function; tests use this to cover each kernel. */
enum { LAMA_TILING_AUTO = 0, LAMA_TILING_SWAPPED = 1, LAMA_TILING_PIXEL = 2, LAMA_TILING_PAIRED = 3 };
int lama_set_tiling(lama_engine* e, int policy);

/* Spectral-transform kernels for plans built after this call (cached plans
 * are dropped): LAMA_SPECTRAL_TWO_PASS always runs the two-pass kernels (any
 * plane size); LAMA_SPECTRAL_REGISTER runs the register-resident kernels
 * wherever the plane is a power of two with sides 8..64 (two-pass
 * elsewhere); LAMA_SPECTRAL_PREFETCH is REGISTER with the persistent
 * TMA-prefetching rfft2 for 64x64 planes; LAMA_SPECTRAL_TENSOR is PREFETCH
 * with the rfft2 of 64x64 planes as two DFT GEMMs on the tensor core;
 * LAMA_SPECTRAL_AUTO picks by plane size and batch (TENSOR for 64x64 planes
 * at 8 images or more, else PREFETCH).  All paths compute the same
 * function; tests use this to cover each. */
enum {
  LAMA_SPECTRAL_AUTO = 0,
  LAMA_SPECTRAL_TWO_PASS = 1,
  LAMA_SPECTRAL_REGISTER = 2,
  LAMA_SPECTRAL_PREFETCH = 3,
  LAMA_SPECTRAL_TENSOR = 4
};
int lama_set_spectral_path(lama_engine* e, int path);

/* Graph lanes of small-batch passes (no counterpart in the reference, which
 * runs one launch at a time on the default stream).  Where an FFC layer's
 * GEMM has fewer 128 x 128 output tiles than the GPU has SMs (e.g. a batch-1
 * 512x512 pass), the layer's spectral chain (conv1, rfft2, FourierUnit conv,
 * irfft2) runs on `chain_sms` SMs concurrently with the part of the FFC GEMM
 * that does not need it, on the others.  0 = one lane; -1 = the default (40).
 * Drops cached plans. */
int lama_set_lanes(lama_engine* e, int chain_sms);

/* Message of the last failure on this engine ("" if none). */
const char* lama_last_error(const lama_engine* e);

/* Wait for all work queued on the engine's stream; reports device errors. */
int lama_synchronize(lama_engine* e);

/* The engine's cudaStream_t, for ordering caller work with the engine's. */
void* lama_stream(lama_engine* e);

/* Kernel launches one forward pass issues at this shape (after the plan for
 * the shape exists; builds it if needed).  Returns < 0 on error. */
int lama_launch_count(lama_engine* e, int batch, int h, int w);

/* Capacity model (replaces mem.rs's estimated_bytes, lama-rs/src/mem.rs:13-36).
 * Device bytes one inpaint pass of `batch` w x h images (lama_inpaint_u8,
 * lama_inpaint_u8_device, one chunk of lama_inpaint_u8_stream; h and w are
 * padded to multiples of 8) allocates on a B200, beyond the engine's resident
 * weights (~0.2 GB): the pass's activations, spectral intermediates, split-K
 * workspaces and u8 buffers, computed by building the pass's plan without
 * allocating (no GPU or weight file needed).  Returns the byte count, or a
 * negative LAMA_E* code for non-positive sizes.  Every plan is checked the
 * same way before it allocates (mem.rs:49-73's guard, with its 10 % headroom
 * of free memory): a pass that does not fit returns LAMA_ENOMEM with the
 * needed and free amounts in lama_last_error(), before any allocation. */
long long lama_estimate_bytes(int batch, int h, int w);

/* The device bytes the engine's plan for that inpaint pass holds (building
 * it if needed); equals lama_estimate_bytes on a B200. */
int lama_plan_bytes(lama_engine* e, int batch, int h, int w, long long* bytes);

/* Per-kernel-class timing of one forward pass on device buffers: each launch
 * is bracketed by CUDA events on the engine's stream.  Fills up to
 * `max_stats` records; *n_stats is the number of classes. */
typedef struct {
  char name[32];
  int launches;
  double ms;       /* summed device time */
  double flops;    /* algorithmic FLOPs (2 x MACs over real taps) */
  double bytes;    /* algorithmic HBM bytes (operands + results, once) */
} lama_kernel_stat;

int lama_profile_forward(lama_engine* e, const float* d_in, int batch, int h, int w, float* d_out,
                         lama_kernel_stat* stats, int max_stats, int* n_stats);

/* Timeline of one forward pass as the captured graph runs it (both lanes):
 * per launch, in plan order, the time its inputs were ready (the latest
 * completion of the launches it follows) and its completion, in ms from the
 * start of the pass, read from timing events recorded inside a copy of the
 * pass's graph.  end_ms - ready_ms is the launch's exposed time (launch
 * latency included).  Fills up to `max_ops` records; *n_ops is the number of
 * launches. */
typedef struct {
  char name[32];
  int lane;        /* graph lane (0, or 1 for the spectral lane of small batches) */
  float ready_ms;
  float end_ms;
} lama_op_time;

int lama_profile_timeline(lama_engine* e, const float* d_in, int batch, int h, int w, float* d_out,
                          lama_op_time* times, int max_ops, int* n_ops);

/* Diagnostics (used by the layer-by-layer parity tests).
 * lama_debug_run: run only the first `n_ops` launches of the f32 forward plan
 * for this shape, eagerly, on host input [batch][4][h][w].
 * lama_debug_read: copy launch `op`'s output tensor to `out` as fp32 (split
 * pairs are summed); dims receives (batch, rows, cols, channels) of the
 * stored NHWC layout including any halo, or (batch, C, H, W) for NCHW
 * outputs; name receives the launch name (32 bytes).  With out == NULL only
 * dims and name are filled. */
int lama_debug_run(lama_engine* e, const float* in, int batch, int h, int w, int n_ops);
int lama_debug_read(lama_engine* e, int batch, int h, int w, int op, float* out, long long cap, int* dims,
                    char* name);

/* Diagnostic of the failure path (failure detection; the reference has no
 * counterpart): launches one CTA that waits on an mbarrier nothing
 * ever arrives on, with a limit of `limit_ms` milliseconds of SM clock
 * instead of the pass kernels' ~1 s.  The wait gives up, records its code in
 * the engine's device status word and returns, so the call reports
 * LAMA_EDEVICE ("a kernel wait timed out ...") and the engine stays usable;
 * no GPU fault or hang is involved.  limit_ms in 1..1000. */
int lama_debug_wait_timeout(lama_engine* e, int limit_ms);

/* --sections on the device (lama-rs/src/main.rs:465-566, the per-pass crop,
 * inference, composite and paste of the reference's loop): the w x h image
 * and mask go up once, then for each of the n rectangles rects[4i..4i+3] =
 * {x0, y0, x1, y1} (from lama_section_rects, rim first) one pass runs on the
 * side x side window centred on it (lama_window_origin), with the mask
 * restricted to the rectangle, and its fill is written into the
 * device-resident working image, which the next pass reads; the result comes
 * back once.  side = min(512, w, h) as in the reference.  n = 0 copies rgb.
 * Returns LAMA_EINVAL for a rectangle outside the image or its window. */
int lama_inpaint_sections_u8(lama_engine* e, const uint8_t* rgb, const uint8_t* mask, int w, int h,
                             const int* rects, int n, int side, uint8_t* out_rgb);

/* Host helpers of the CLI's --tile / --sections modes (no GPU needed).
 * They restate lama-rs/src/main.rs's geometry with the same constants
 * (window >= 512, sections of 256, multiples of 8) and ordering. */

/* Top-left of a `side`-long window centred on c, kept inside [0, extent-side]
 * (main.rs:722-727). */
int lama_window_origin(int c, int side, int extent);

/* The --tile window of a w x h mask (non-zero = hole): out = {x0, y0, side,
 * bbox_w, bbox_h}.  Returns 1, or 0 for an empty mask (main.rs:740-777). */
int lama_tile_rect(const uint8_t* mask, int w, int h, int* out);

/* Distance of every masked pixel to the rim of the hole (4-neighbour BFS);
 * UINT32_MAX for unmasked pixels (main.rs:664-717). */
int lama_mask_depth(const uint8_t* mask, int w, int h, uint32_t* depth);

/* The --sections pieces, rim first: up to `cap` rectangles {x0, y0, x1, y1}
 * (exclusive ends) written to `out`; returns their count (main.rs:597-659). */
int lama_section_rects(const uint8_t* mask, int w, int h, int* out, int cap);

/* No counterpart in the reference: the FourierUnit's forward transform
 * (rfft2, norm='ortho', the reference's transform directions) on its own,
 * for callers that cannot allocate device memory (a host whose HBM is
 * already reserved by another framework's pool, or a pipeline that cannot
 * take the device-wide synchronisation of cudaMalloc / cudaFree between its
 * launches).  It runs the two-pass kernels with their intermediate in a fixed
 * 16 MiB device array compiled into the library (held by every GPU that
 * loads the library, until exit) and calls no cudaMalloc / cudaFree.  The
 * first call on a device does that device's one-time set-up (it looks up the
 * array's device address and sets the kernels' shared-memory limit), so make
 * it before any stream capture on that device.  With CUDA's default lazy
 * module loading the array's memory is claimed by that first call, not when
 * the library is loaded: a caller that reserves the rest of the GPU for its
 * own pool makes its first call before reserving it.  A failed set-up is not
 * cached; the next call tries again.
 *   d_feat: [batch][channels][h][w] fp32 (device, 4-byte aligned);
 *   d_spec: [2][batch][h][w/2+1][2*channels] bf16 (device, 4-byte aligned;
 *           a misaligned pointer returns LAMA_EINVAL), value = part 0 +
 *           part 1, channel 2c = real and 2c+1 = imaginary part of channel c
 *           (the engine's own spectrum layout).
 * Limits: h, w <= 1024 and batch*channels*(w/2+1)*h <= 2,097,152 (16 MiB of
 * complex fp32); larger requests return LAMA_ESCRATCH.  Work is queued on
 * `stream` (a cudaStream_t, null = legacy default stream) of CUDA device
 * `device`; the caller's current device is restored.  Every call shares the
 * one array and leaves its contents behind; nothing in it needs to start at
 * zero (each call overwrites what it reads), but calls whose GPU work
 * overlaps in time race.  On failure a message is written to err (err_len
 * bytes, may be null). */
int lama_rfft2_noalloc(int device, const float* d_feat, int batch, int channels, int h, int w, void* d_spec,
                       void* stream, char* err, int err_len);

/* Free every device buffer and the engine. */
void lama_close(lama_engine* e);

/* ABI version of this header. */
int lama_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LAMA_B200_H */
