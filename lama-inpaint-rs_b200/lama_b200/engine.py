"""ctypes binding of the B200 engine (liblama_b200.so, include/lama_b200.h).

This is the Python face of the reference's operator boundary:

* `Engine(weights, device)`  ~ `WeightStore::open` + `cuda::load_steps`
  (lama-rs/src/weights.rs:80-106, lama-rs/src/cuda.rs:903-962);
* `Engine.forward(x)`        ~ `cuda::run` / `infer` (lama-rs/src/cuda.rs:1542-1691,
  lama-rs/src/main.rs:318-361): [4,h,w] or [B,4,h,w] f32 in, [3,h,w] / [B,3,h,w] out;
* `Engine.inpaint_u8(rgb, mask)` ~ `build_input` + `infer` + composite
  (lama-rs/src/main.rs:175-196, 272-307).

Errors raise `LamaError` carrying the engine's message (the reference's
`Err(String)`).  There is no CPU fallback: if the native library cannot be
loaded, importing the engine raises.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("LAMA_B200_LIB", os.path.join(PKG_ROOT, "liblama_b200.so"))

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_vp = ctypes.c_void_p

LAMA_ERRORS = {-1: "EINVAL", -2: "EWEIGHTS", -3: "ECUDA", -4: "EDEVICE", -5: "ENOMEM", -6: "EUNSUPPORTED"}


class LamaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{LAMA_ERRORS.get(code, code)}: {msg}")
        self.code = code
        self.msg = msg


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int), ("ms", ctypes.c_double),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


class OpTime(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("lane", ctypes.c_int), ("ready_ms", ctypes.c_float),
                ("end_ms", ctypes.c_float)]


_lib = None

# Every symbol include/lama_b200.h declares: (name, restype, argtypes).
SIGNATURES = [
    ("lama_abi_version", ctypes.c_int, []),
    ("lama_open", ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(_vp)]),
    ("lama_forward", ctypes.c_int, [_vp, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
    ("lama_forward_device", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("lama_inpaint_u8", ctypes.c_int, [_vp, _u8p, _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u8p]),
    ("lama_inpaint_u8_device", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("lama_inpaint_u8_stream", ctypes.c_int, [_vp, _u8p, _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, _u8p]),
    ("lama_inpaint_sections_u8", ctypes.c_int, [_vp, _u8p, _u8p, ctypes.c_int, ctypes.c_int,
                                                ctypes.POINTER(ctypes.c_int), ctypes.c_int, ctypes.c_int, _u8p]),
    ("lama_resblocks", ctypes.c_int, [_vp, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      _f32p, _f32p]),
    ("lama_resblocks_device", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, _vp, _vp]),
    ("lama_set_tiling", ctypes.c_int, [_vp, ctypes.c_int]),
    ("lama_set_spectral_path", ctypes.c_int, [_vp, ctypes.c_int]),
    ("lama_set_lanes", ctypes.c_int, [_vp, ctypes.c_int]),
    ("lama_debug_wait_timeout", ctypes.c_int, [_vp, ctypes.c_int]),
    ("lama_rfft2_noalloc", ctypes.c_int, [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          _vp, _vp, ctypes.c_char_p, ctypes.c_int]),
    ("lama_last_error", ctypes.c_char_p, [_vp]),
    ("lama_synchronize", ctypes.c_int, [_vp]),
    ("lama_stream", _vp, [_vp]),
    ("lama_launch_count", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("lama_estimate_bytes", ctypes.c_longlong, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("lama_plan_bytes", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_longlong)]),
    ("lama_profile_forward", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp,
                                            ctypes.POINTER(KernelStat), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    ("lama_profile_timeline", ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp,
                                             ctypes.POINTER(OpTime), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    ("lama_debug_run", ctypes.c_int, [_vp, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("lama_debug_read", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                       ctypes.c_longlong, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p]),
    ("lama_window_origin", ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("lama_tile_rect", ctypes.c_int, [_u8p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    ("lama_mask_depth", ctypes.c_int, [_u8p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]),
    ("lama_section_rects", ctypes.c_int, [_u8p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                          ctypes.c_int]),
    ("lama_close", None, [_vp]),
]
CLI_PATH = os.path.join(PKG_ROOT, "lama-inpaint")


def lib():
    """Load liblama_b200.so (raises OSError if it is missing: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `make -C lama-inpaint-rs_b200/csrc` "
                          "(the engine has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _fp(a):
    return a.ctypes.data_as(_f32p)


def _up(a):
    return a.ctypes.data_as(_u8p)


# ------------------------------------------------------------ host geometry (no GPU)

def estimate_bytes(batch: int, h: int, w: int) -> int:
    """Device bytes one inpaint pass of `batch` w x h images allocates on a B200
    (the capacity model behind the engine's guard; lama-rs/src/mem.rs:13-36)."""
    v = lib().lama_estimate_bytes(batch, h, w)
    if v < 0:
        raise LamaError(int(v), "batch, h and w must be positive")
    return int(v)


def window_origin(c: int, side: int, extent: int) -> int:
    return lib().lama_window_origin(c, side, extent)


def tile_rect(mask: np.ndarray):
    """--tile window (x0, y0, side, bbox_w, bbox_h) or None for an empty mask."""
    m = np.ascontiguousarray(mask, np.uint8)
    out = (ctypes.c_int * 5)()
    r = lib().lama_tile_rect(_up(m), m.shape[1], m.shape[0], out)
    return tuple(out) if r == 1 else None


def mask_depth(mask: np.ndarray) -> np.ndarray:
    m = np.ascontiguousarray(mask, np.uint8)
    d = np.empty(m.shape, np.uint32)
    lib().lama_mask_depth(_up(m), m.shape[1], m.shape[0], d.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return d


def section_rects(mask: np.ndarray):
    """--sections pieces [(x0, y0, x1, y1)], rim first."""
    m = np.ascontiguousarray(mask, np.uint8)
    n = lib().lama_section_rects(_up(m), m.shape[1], m.shape[0], None, 0)
    out = (ctypes.c_int * (4 * max(n, 1)))()
    lib().lama_section_rects(_up(m), m.shape[1], m.shape[0], out, n)
    return [tuple(out[4 * i: 4 * i + 4]) for i in range(n)]


class Engine:
    def __init__(self, weights_path: str, device: int = 0):
        L = lib()
        h = _vp()
        rc = L.lama_open(os.fsencode(weights_path), device, ctypes.byref(h))
        self._h = h
        if rc != 0:
            msg = L.lama_last_error(h).decode() if h else ""
            L.lama_close(h)
            self._h = None
            raise LamaError(rc, msg)

    def close(self):
        if getattr(self, "_h", None):
            lib().lama_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, rc):
        if rc != 0:
            raise LamaError(rc, lib().lama_last_error(self._h).decode())

    @property
    def handle(self):
        return self._h

    def stream(self) -> int:
        return lib().lama_stream(self._h) or 0

    TILING_AUTO, TILING_SWAPPED, TILING_PIXEL, TILING_PAIRED = 0, 1, 2, 3

    def set_tiling(self, policy: int):
        """Tile policy for plans built from now on (see include/lama_b200.h)."""
        self._check(lib().lama_set_tiling(self._h, policy))

    SPECTRAL_AUTO, SPECTRAL_TWO_PASS, SPECTRAL_REGISTER, SPECTRAL_PREFETCH, SPECTRAL_TENSOR = 0, 1, 2, 3, 4

    def set_spectral_path(self, path: int):
        """Spectral-transform kernels for plans built from now on (see include/lama_b200.h)."""
        self._check(lib().lama_set_spectral_path(self._h, path))

    def set_lanes(self, chain_sms: int):
        """SMs of the spectral graph lane at small batches (0 = one lane, -1 = default)."""
        self._check(lib().lama_set_lanes(self._h, chain_sms))

    def synchronize(self):
        self._check(lib().lama_synchronize(self._h))

    # -------------------------------------------------------------- forward
    def forward(self, x: np.ndarray) -> np.ndarray:
        """x: [4,h,w] or [B,4,h,w] f32 -> sigmoid output [3,h,w] / [B,3,h,w]."""
        x = np.ascontiguousarray(x, np.float32)
        single = x.ndim == 3
        if single:
            x = x[None]
        if x.ndim != 4 or x.shape[1] != 4:
            raise LamaError(-1, f"input must be [4,h,w] or [B,4,h,w] f32, got shape {x.shape}")
        b, _, h, w = x.shape
        out = np.empty((b, 3, h, w), np.float32)
        self._check(lib().lama_forward(self._h, _fp(x), b, h, w, _fp(out)))
        return out[0] if single else out

    def forward_device(self, d_in: int, d_out: int, batch: int, h: int, w: int):
        """Device pointers (e.g. torch data_ptr()); queued on the engine stream."""
        self._check(lib().lama_forward_device(self._h, d_in, batch, h, w, d_out))

    def inpaint_u8(self, rgb: np.ndarray, mask: np.ndarray) -> np.ndarray:
        """rgb [h,w,3] / [B,h,w,3] u8, mask [h,w] / [B,h,w] u8 -> composited u8 RGB."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        mask = np.ascontiguousarray(mask, np.uint8)
        single = rgb.ndim == 3
        if single:
            rgb, mask = rgb[None], mask[None]
        if rgb.ndim != 4 or rgb.shape[-1] != 3:
            raise LamaError(-1, f"rgb must be [h,w,3] or [B,h,w,3] u8, got shape {rgb.shape}")
        b, h, w, _ = rgb.shape
        if mask.shape != (b, h, w):
            raise LamaError(-1, f"mask is {mask.shape[-1]}x{mask.shape[-2]} but image is {w}x{h}")
        out = np.empty_like(rgb)
        self._check(lib().lama_inpaint_u8(self._h, _up(rgb), _up(mask), b, h, w, _up(out)))
        return out[0] if single else out

    def inpaint_u8_stream(self, rgb: np.ndarray, mask: np.ndarray, chunk: int) -> np.ndarray:
        """rgb [n,h,w,3] u8, mask [n,h,w] u8 -> composited u8 RGB, `chunk` images per pass with
        the host<->device copies of one chunk overlapping the pass of the previous one."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        mask = np.ascontiguousarray(mask, np.uint8)
        if rgb.ndim != 4 or rgb.shape[-1] != 3:
            raise LamaError(-1, f"rgb must be [n,h,w,3] u8, got shape {rgb.shape}")
        n, h, w, _ = rgb.shape
        if mask.shape != (n, h, w):
            raise LamaError(-1, f"mask is {mask.shape} but image is {rgb.shape}")
        out = np.empty_like(rgb)
        self._check(lib().lama_inpaint_u8_stream(self._h, _up(rgb), _up(mask), n, h, w, chunk, _up(out)))
        return out

    def inpaint_sections_u8(self, rgb: np.ndarray, mask: np.ndarray, rects, side: int) -> np.ndarray:
        """--sections on the device: rgb [h,w,3] u8, mask [h,w] u8, rects [(x0, y0, x1, y1), ...]
        (lama_section_rects order), one side x side window per rectangle."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        mask = np.ascontiguousarray(mask, np.uint8)
        if rgb.ndim != 3 or rgb.shape[-1] != 3:
            raise LamaError(-1, f"rgb must be [h,w,3] u8, got shape {rgb.shape}")
        h, w, _ = rgb.shape
        if mask.shape != (h, w):
            raise LamaError(-1, f"mask is {mask.shape[-1]}x{mask.shape[-2]} but image is {w}x{h}")
        r = np.ascontiguousarray(np.asarray(rects, np.int32).reshape(-1, 4))
        out = np.empty_like(rgb)
        self._check(lib().lama_inpaint_sections_u8(self._h, _up(rgb), _up(mask), w, h,
                                                   r.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(r), side,
                                                   _up(out)))
        return out

    def inpaint_u8_device(self, d_rgb: int, d_mask: int, d_out: int, batch: int, h: int, w: int):
        self._check(lib().lama_inpaint_u8_device(self._h, d_rgb, d_mask, batch, h, w, d_out))

    def resblocks(self, local: np.ndarray, glob: np.ndarray, nblocks: int = 18):
        """The 18-block FFC stack: local [B,128,h,w], global [B,384,h,w] f32."""
        l = np.ascontiguousarray(local, np.float32)
        g = np.ascontiguousarray(glob, np.float32)
        single = l.ndim == 3
        if single:
            l, g = l[None], g[None]
        if l.ndim != 4 or l.shape[1] != 128:
            raise LamaError(-1, f"local must be [128,h,w] or [B,128,h,w] f32, got shape {l.shape}")
        b, _, h, w = l.shape
        if g.shape != (b, 384, h, w):
            raise LamaError(-1, f"global must be {(b, 384, h, w)} to match local, got {g.shape}")
        lo = np.empty_like(l)
        go = np.empty_like(g)
        self._check(lib().lama_resblocks(self._h, _fp(l), _fp(g), b, h, w, nblocks, _fp(lo), _fp(go)))
        return (lo[0], go[0]) if single else (lo, go)

    def resblocks_device(self, d_l, d_g, d_lo, d_go, batch, h, w, nblocks=18):
        self._check(lib().lama_resblocks_device(self._h, d_l, d_g, batch, h, w, nblocks, d_lo, d_go))

    def plan_bytes(self, batch: int, h: int, w: int) -> int:
        """Device bytes the engine's inpaint plan for this shape holds (builds it)."""
        v = ctypes.c_longlong(0)
        self._check(lib().lama_plan_bytes(self._h, batch, h, w, ctypes.byref(v)))
        return v.value

    def launch_count(self, batch: int, h: int, w: int) -> int:
        n = lib().lama_launch_count(self._h, batch, h, w)
        if n < 0:
            self._check(n)
        return n

    def profile_forward(self, d_in: int, d_out: int, batch: int, h: int, w: int):
        stats = (KernelStat * 64)()
        n = ctypes.c_int(0)
        self._check(lib().lama_profile_forward(self._h, d_in, batch, h, w, d_out, stats, 64, ctypes.byref(n)))
        return [dict(name=s.name.decode(), launches=s.launches, ms=s.ms, flops=s.flops, bytes=s.bytes)
                for s in stats[: n.value]]

    def profile_timeline(self, d_in: int, d_out: int, batch: int, h: int, w: int):
        """Per-launch (name, lane, ready_ms, end_ms) of one graph replay of the forward pass."""
        cap = 1024
        ts = (OpTime * cap)()
        n = ctypes.c_int(0)
        self._check(lib().lama_profile_timeline(self._h, d_in, batch, h, w, d_out, ts, cap, ctypes.byref(n)))
        return [dict(name=t.name.decode(), lane=t.lane, ready_ms=t.ready_ms, end_ms=t.end_ms)
                for t in ts[: min(n.value, cap)]]

    # -------------------------------------------------------------- diagnostics
    def debug_run(self, x: np.ndarray, n_ops: int):
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 3:
            x = x[None]
        b, _, h, w = x.shape
        self._check(lib().lama_debug_run(self._h, _fp(x), b, h, w, n_ops))

    def debug_wait_timeout(self, limit_ms: int):
        """Run the bounded-wait probe (include/lama_b200.h); raises LamaError(EDEVICE)."""
        self._check(lib().lama_debug_wait_timeout(self._h, limit_ms))

    def op_names(self, batch: int, h: int, w: int):
        """Launch names of the f32 forward plan at this shape, in order."""
        names = []
        for i in range(self.launch_count(batch, h, w)):
            dims = (ctypes.c_int * 4)()
            name = ctypes.create_string_buffer(32)
            self._check(lib().lama_debug_read(self._h, batch, h, w, i, None, 0, dims, name))
            names.append(name.value.decode())
        return names

    def debug_read(self, batch: int, h: int, w: int, op: int):
        dims = (ctypes.c_int * 4)()
        name = ctypes.create_string_buffer(32)
        self._check(lib().lama_debug_read(self._h, batch, h, w, op, None, 0, dims, name))
        n = dims[0] * dims[1] * dims[2] * dims[3]
        out = np.empty(n, np.float32)
        self._check(lib().lama_debug_read(self._h, batch, h, w, op, _fp(out), n, dims, name))
        return name.value.decode(), out.reshape(tuple(dims))
