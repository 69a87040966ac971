// lama-inpaint: the command-line host over the B200 engine.
//
// Keeps the reference CLI's surface (lama-rs/src/main.rs): the flags of
// parse_args (:49-101), the default weight search (:142-171), the whole-image
// path (:212-313), --tile (:378-443) and --sections (:465-566), exit code 2
// for usage errors and 1 for run errors (:198-210), diagnostics on stderr,
// `-` for stdin/stdout.  The network pass, the input build and the composite
// run on the GPU through the C ABI (lama_inpaint_u8); --tile and --sections
// crop windows here and paste back exactly the pixels the reference pastes.
//
// Differences, on purpose: there is no CPU engine in this build, so --cpu is
// an error (the reference's CPU-only build rejects --gpu the same way) and a
// GPU failure is fatal (no silent fallback).
#include <unistd.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "lama_b200.h"
#include "png.h"

using lama_host::Rgb8;

namespace {

constexpr int kTileMin = 512;
constexpr int kPadMod = 8;

struct Args {
  std::string image, mask, output, weights;
  bool force_cpu = false, force_gpu = false, tile = false, sections = false;
};

const char* kUsage =
    "usage: lama-inpaint --image IN.png --mask MASK.png --output OUT.png\n"
    "                    [--weights big-lama.safetensors] [--cpu | --gpu]\n"
    "                    [--tile | --sections]\n"
    "\n"
    "Inpaints the pixels of IN.png that MASK.png marks (any non-black pixel is a\n"
    "hole) with the big-lama generator on an NVIDIA B200 and writes OUT.png at the\n"
    "input size.  '-' reads a PNG from stdin (for one of the inputs) or writes the\n"
    "result to stdout.  Only masked pixels come from the network.\n"
    "\n"
    "--tile      run on a square window around the mask (twice the mask's bounding\n"
    "            box, at least 512x512, clamped inside the image); images at or\n"
    "            below 512px on the short side run whole\n"
    "--sections  fill a large mask in 256x256 sections, one 512x512 window per\n"
    "            section, from the rim of the hole inward\n"
    "--gpu       accepted for compatibility (the GPU is always used)\n"
    "--cpu       not available: this build has no CPU engine\n";

void log(const std::string& s) { fprintf(stderr, "%s\n", s.c_str()); }

double secs(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

bool exists(const std::string& p) { return access(p.c_str(), F_OK) == 0; }

std::string dirname_of(const std::string& p) {
  const size_t k = p.find_last_of('/');
  return k == std::string::npos ? "." : p.substr(0, k == 0 ? 1 : k);
}

// main.rs:142-171: beside the executable, then models/, then up the tree, then cwd.
std::string default_weights(const std::string& rel) {
  char buf[4096];
  const ssize_t n = readlink("/proc/self/exe", buf, sizeof(buf) - 1);
  if (n > 0) {
    buf[n] = 0;
    std::string dir = dirname_of(buf);
    if (exists(dir + "/" + rel)) return dir + "/" + rel;
    if (exists(dir + "/models/" + rel)) return dir + "/models/" + rel;
    std::string base = dir;
    for (int i = 0; i < 6; i++) {
      if (exists(base + "/" + rel)) return base + "/" + rel;
      if (exists(base + "/models/" + rel)) return base + "/models/" + rel;
      if (base == "/" || base.empty()) break;
      base = dirname_of(base);
    }
  }
  return rel;
}

int parse_args(int argc, char** argv, Args& a, std::string& err) {
  for (int i = 1; i < argc; i++) {
    const std::string s = argv[i];
    auto val = [&](std::string& dst) {
      if (i + 1 >= argc) { err = s + " needs a value"; return false; }
      dst = argv[++i];
      return true;
    };
    if (s == "--image") { if (!val(a.image)) return 1; }
    else if (s == "--mask") { if (!val(a.mask)) return 1; }
    else if (s == "--output") { if (!val(a.output)) return 1; }
    else if (s == "--weights") { if (!val(a.weights)) return 1; }
    else if (s == "--cpu") a.force_cpu = true;
    else if (s == "--gpu") a.force_gpu = true;
    else if (s == "--tile") a.tile = true;
    else if (s == "--sections") a.sections = true;
    else if (s == "-h" || s == "--help") { printf("%s", kUsage); return -1; }
    else { err = "unknown argument " + s; return 1; }
  }
  if (a.image.empty()) { err = "--image is required"; return 1; }
  if (a.mask.empty()) { err = "--mask is required"; return 1; }
  if (a.output.empty()) { err = "--output is required"; return 1; }
  if (a.image == "-" && a.mask == "-") {
    err = "--image and --mask cannot both be '-' (stdin has only one stream)";
    return 1;
  }
  if (a.tile && a.sections) { err = "--tile and --sections are mutually exclusive"; return 1; }
  if (a.weights.empty()) a.weights = default_weights("big-lama.safetensors");
  return 0;
}

bool read_file(const std::string& path, std::vector<uint8_t>& out, std::string& err) {
  FILE* f = path == "-" ? stdin : fopen(path.c_str(), "rb");
  if (!f) { err = path + ": cannot open"; return false; }
  uint8_t buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out.insert(out.end(), buf, buf + n);
  if (f != stdin) fclose(f);
  return true;
}

bool read_rgb(const std::string& path, Rgb8& img, std::string& err) {
  std::vector<uint8_t> data;
  if (!read_file(path, data, err)) return false;
  return lama_host::png_decode(data, path == "-" ? "stdin" : path, img, err);
}

// image.rs:123-130: the mask is the red channel of any PNG.
bool read_gray(const std::string& path, std::vector<uint8_t>& g, int& w, int& h, std::string& err) {
  Rgb8 img;
  if (!read_rgb(path, img, err)) return false;
  w = img.width;
  h = img.height;
  g.resize((size_t)w * h);
  for (size_t i = 0; i < g.size(); i++) g[i] = img.data[i * 3];
  return true;
}

bool write_rgb(const std::string& path, const Rgb8& img, std::string& err) {
  std::vector<uint8_t> png;
  if (!lama_host::png_encode(img, png, err)) return false;
  FILE* f = path == "-" ? stdout : fopen(path.c_str(), "wb");
  if (!f) { err = path + ": cannot create"; return false; }
  const bool ok = fwrite(png.data(), 1, png.size(), f) == png.size();
  if (f == stdout) fflush(f);
  else fclose(f);
  if (!ok) err = path + ": write failed";
  return ok;
}

struct Engine {
  lama_engine* e = nullptr;
  ~Engine() { if (e) lama_close(e); }
};

// One window through the engine: build_input + forward + composite on the GPU.
// `oom_hint` names the mode that caps the pass's size; it is added to the
// message when the engine's capacity guard refuses the pass (as mem.rs:48-73
// does, before anything is allocated: the engine compares the pass's exact
// footprint with the device's free memory less 10 %).
bool inpaint(Engine& eng, const Rgb8& src, const std::vector<uint8_t>& mask, Rgb8& out, std::string& err,
             const char* oom_hint) {
  out.width = src.width;
  out.height = src.height;
  out.data.resize(src.data.size());
  const int rc = lama_inpaint_u8(eng.e, src.data.data(), mask.data(), 1, src.height, src.width, out.data.data());
  if (rc != 0) {
    err = std::string("gpu inference failed: ") + lama_last_error(eng.e);
    if (rc == LAMA_ENOMEM) err += std::string(". ") + oom_hint;
    return false;
  }
  return true;
}

Rgb8 crop_rgb(const Rgb8& img, int x0, int y0, int side) {
  Rgb8 o;
  o.width = o.height = side;
  o.data.resize((size_t)side * side * 3);
  for (int y = 0; y < side; y++)
    memcpy(&o.data[(size_t)y * side * 3], &img.data[(((size_t)(y0 + y)) * img.width + x0) * 3], (size_t)side * 3);
  return o;
}

std::vector<uint8_t> crop_gray(const std::vector<uint8_t>& m, int w, int x0, int y0, int side) {
  std::vector<uint8_t> o((size_t)side * side);
  for (int y = 0; y < side; y++) memcpy(&o[(size_t)y * side], &m[(size_t)(y0 + y) * w + x0], side);
  return o;
}

int run(const Args& a) {
  const auto t_start = std::chrono::steady_clock::now();
  std::string err;
  Rgb8 src;
  std::vector<uint8_t> mask;
  int mw = 0, mh = 0;
  if (!read_rgb(a.image, src, err) || !read_gray(a.mask, mask, mw, mh, err)) {
    log("error: " + err);
    return 1;
  }
  if (mw != src.width || mh != src.height) {
    log("error: mask is " + std::to_string(mw) + "x" + std::to_string(mh) + " but image is " +
        std::to_string(src.width) + "x" + std::to_string(src.height));
    return 1;
  }
  const int W = src.width, H = src.height;
  char msg[256];
  snprintf(msg, sizeof(msg), "loaded %dx%d image + mask in %.2fs", W, H, secs(t_start));
  log(msg);
  if (a.force_cpu) {
    log("error: --cpu: this build has no CPU engine (the B200 engine has no CPU fallback)");
    return 1;
  }

  Engine eng;
  const int rc = lama_open(a.weights.c_str(), 0, &eng.e);
  if (rc != 0) {
    log(std::string("error: ") + (eng.e ? lama_last_error(eng.e) : "cannot open the engine"));
    return 1;
  }
  log("weights: " + a.weights);

  Rgb8 out;
  bool sections = a.sections;
  if (sections && std::min(W, H) <= kTileMin) {
    snprintf(msg, sizeof(msg), "--sections: %dx%d is at or below %dpx on its short side; running the whole image", W,
             H, kTileMin);
    log(msg);
    sections = false;
  }
  if (sections) {
    // main.rs:465-566
    const int n = lama_section_rects(mask.data(), W, H, nullptr, 0);
    if (n == 0) {
      log("--sections: mask is empty; copying the input to the output");
      out = src;
    } else {
      std::vector<int> rects((size_t)n * 4);
      lama_section_rects(mask.data(), W, H, rects.data(), n);
      const int side = std::max(1, std::min(kTileMin, std::min(W, H)));
      snprintf(msg, sizeof(msg), "sections: %d passes, %dx%d window each, rim inward", n, side, side);
      log(msg);
      for (int i = 0; i < n; i++) {
        const int sx0 = rects[4 * i], sy0 = rects[4 * i + 1], sx1 = rects[4 * i + 2], sy1 = rects[4 * i + 3];
        snprintf(msg, sizeof(msg), "  pass %d/%d: %dx%d window at (%d,%d)", i + 1, n, side, side,
                 lama_window_origin((sx0 + sx1) / 2, side, W), lama_window_origin((sy0 + sy1) / 2, side, H));
        log(msg);
      }
      // every pass on the GPU: the working image (original plus the fills of
      // earlier passes) stays on the device between passes
      const auto t0 = std::chrono::steady_clock::now();
      out.width = W;
      out.height = H;
      out.data.resize(src.data.size());
      if (lama_inpaint_sections_u8(eng.e, src.data.data(), mask.data(), W, H, rects.data(), n, side,
                                   out.data.data()) != 0) {
        log(std::string("error: gpu inference failed: ") + lama_last_error(eng.e));
        return 1;
      }
      snprintf(msg, sizeof(msg), "inference: %d passes in %.2fs", n, secs(t0));
      log(msg);
    }
  } else if (a.tile) {
    // main.rs:378-443
    int t[5];
    if (lama_tile_rect(mask.data(), W, H, t) == 0) {
      log("--tile: mask is empty; copying the input to the output");
      out = src;
    } else {
      const int x0 = t[0], y0 = t[1], side = t[2];
      snprintf(msg, sizeof(msg), "tile: %dx%d window at (%d,%d) covering a %dx%d mask", side, side, x0, y0, t[3], t[4]);
      log(msg);
      Rgb8 sub = crop_rgb(src, x0, y0, side);
      std::vector<uint8_t> sub_mask = crop_gray(mask, W, x0, y0, side);
      const auto t0 = std::chrono::steady_clock::now();
      Rgb8 filled;
      if (!inpaint(eng, sub, sub_mask, filled, err,
                   "The device cannot hold this window: --sections fills the mask in 512x512 passes.")) {
        log("error: " + err);
        return 1;
      }
      snprintf(msg, sizeof(msg), "inference %dx%d in %.2fs", side, side, secs(t0));
      log(msg);
      out = src;
      for (int y = 0; y < side; y++)
        for (int x = 0; x < side; x++) {
          if (!sub_mask[(size_t)y * side + x]) continue;
          memcpy(&out.data[(((size_t)(y0 + y)) * W + x0 + x) * 3], &filled.data[((size_t)y * side + x) * 3], 3);
        }
    }
  } else {
    const auto t0 = std::chrono::steady_clock::now();
    if (!inpaint(eng, src, mask, out, err,
                 "The device cannot hold this image: --tile runs on a window around the mask, and "
                 "--sections fills a large mask in 512x512 passes.")) {
      log("error: " + err);
      return 1;
    }
    snprintf(msg, sizeof(msg), "inference %dx%d in %.2fs", W, H, secs(t0));
    log(msg);
  }
  if (!write_rgb(a.output, out, err)) { log("error: " + err); return 1; }
  log("wrote " + a.output);
  snprintf(msg, sizeof(msg), "total %.2fs", secs(t_start));
  log(msg);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  Args a;
  std::string err;
  // Diagnostic: decode a PNG the way --image does and write it back as 8-bit RGB.
  if (argc == 4 && std::string(argv[1]) == "--decode-png") {
    Rgb8 img;
    if (!read_rgb(argv[2], img, err) || !write_rgb(argv[3], img, err)) {
      fprintf(stderr, "error: %s\n", err.c_str());
      return 1;
    }
    return 0;
  }
  const int pr = parse_args(argc, argv, a, err);
  if (pr < 0) return 0;
  if (pr > 0) {
    fprintf(stderr, "error: %s\n\n%s", err.c_str(), kUsage);
    return 2;
  }
  return run(a);
}
