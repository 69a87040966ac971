"""ctypes wrapper over the CPU oracle (liblama_oracle.so).

TEST INFRASTRUCTURE ONLY: the checker the parity tests, the smoke check and
bench.py's CPU-baseline / reference legs use.  The product path never imports
this module.  The library restates the reference CPU engine
(lama-rs/src/cpu.rs); see lama_oracle.cpp for the arithmetic contract.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblama_oracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)


def build() -> str:
    """Compile the oracle with its Makefile (g++, -ffp-contract=off, OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_open.restype = ctypes.c_void_p
        L.oracle_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
        L.oracle_close.argtypes = [ctypes.c_void_p]
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_forward.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_forward_dump.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          _f32p, ctypes.c_longlong, ctypes.POINTER(ctypes.c_longlong)]
        L.oracle_resblocks.argtypes = [ctypes.c_void_p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_rfft2.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_irfft2.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_build_input.argtypes = [_u8p, _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_composite.argtypes = [_u8p, _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _f32p, _u8p]
        _lib = L
    return _lib


def _p(a, t=_f32p):
    return a.ctypes.data_as(t)


def set_threads(n: int) -> int:
    return lib().oracle_set_threads(n)


class Oracle:
    """The reference CPU engine restated: `Net::load` + `Net::forward`."""

    def __init__(self, weights_path: str):
        err = ctypes.create_string_buffer(512)
        self.h = lib().oracle_open(weights_path.encode(), err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def close(self):
        if self.h:
            lib().oracle_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x: np.ndarray) -> np.ndarray:
        """x: [4, h, w] f32 -> [3, h, w] f32 (sigmoid output)."""
        x = np.ascontiguousarray(x, np.float32)
        _, h, w = x.shape
        out = np.empty((3, h, w), np.float32)
        if lib().oracle_forward(self.h, _p(x), h, w, _p(out)) != 0:
            raise RuntimeError("oracle forward failed")
        return out

    def forward_dump(self, x: np.ndarray, step: int) -> np.ndarray:
        """Activation (local then global, NCHW) after plan step `step`."""
        x = np.ascontiguousarray(x, np.float32)
        _, h, w = x.shape
        cap = 64 * 4 * (h + 6) * (w + 6) + 16
        buf = np.empty(cap, np.float32)
        n = ctypes.c_longlong(0)
        if lib().oracle_forward_dump(self.h, _p(x), h, w, step, _p(buf), cap, ctypes.byref(n)) != 0:
            raise RuntimeError("dump buffer too small")
        return buf[: n.value].copy()

    def resblocks(self, local: np.ndarray, glob: np.ndarray, nblocks: int = 18):
        l = np.ascontiguousarray(local, np.float32).copy()
        g = np.ascontiguousarray(glob, np.float32).copy()
        _, h, w = l.shape
        lib().oracle_resblocks(self.h, _p(l), _p(g), h, w, nblocks)
        return l, g


def rfft2(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    h, w = x.shape
    out = np.empty((2, h, w // 2 + 1), np.float32)
    lib().oracle_rfft2(_p(x), h, w, _p(out))
    return out


def irfft2(spec: np.ndarray, w: int) -> np.ndarray:
    spec = np.ascontiguousarray(spec, np.float32)
    h = spec.shape[1]
    out = np.empty((h, w), np.float32)
    lib().oracle_irfft2(_p(spec), h, w, _p(out))
    return out


def build_input(rgb: np.ndarray, mask: np.ndarray, pad_h: int, pad_w: int) -> np.ndarray:
    rgb = np.ascontiguousarray(rgb, np.uint8)
    mask = np.ascontiguousarray(mask, np.uint8)
    h, w = mask.shape
    out = np.empty((4, h + pad_h, w + pad_w), np.float32)
    lib().oracle_build_input(_p(rgb, _u8p), _p(mask, _u8p), h, w, pad_h, pad_w, _p(out))
    return out


def composite(rgb: np.ndarray, mask: np.ndarray, out: np.ndarray) -> np.ndarray:
    rgb = np.ascontiguousarray(rgb, np.uint8)
    mask = np.ascontiguousarray(mask, np.uint8)
    out = np.ascontiguousarray(out, np.float32)
    h, w = mask.shape
    ph, pw = out.shape[1], out.shape[2]
    dst = np.empty((h, w, 3), np.uint8)
    lib().oracle_composite(_p(rgb, _u8p), _p(mask, _u8p), h, w, ph, pw, _p(out), _p(dst, _u8p))
    return dst
