"""lama_rfft2_noalloc (no counterpart in the reference): the two-pass rfft2
with its intermediate in a fixed device array, called through the C ABI.

Some callers cannot allocate device memory: a host whose HBM is already held
by another framework's memory pool, or a pipeline that cannot afford the
device-wide synchronisation of cudaMalloc / cudaFree between its launches.
The GPU test checks, for two calls issued back to back on one stream with
different plane sizes (one of them not a power of two):
  * the output against float64 torch.fft (norm='ortho', in the reference's
    transform directions: lama-rs/src/cpu.rs:769-1011), an independent check;
  * the output against the engine's own rfft2 launch (the existing entry
    point, lama_debug_run / lama_debug_read on the two-pass spectral path)
    on the same input;
  * that the device's free memory is the same before and after the calls.
This file is collected last on purpose: it must pass alone in a fresh process
and after every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import make_input
from lama_b200 import engine as E

LAMA_OK, LAMA_EINVAL, LAMA_ESCRATCH = 0, -1, -7
FFT_TOL = 1e-4  # max |diff| <= FFT_TOL * max |expected|, as for the engine's own spectral tests


def call(feat, batch, channels, h, w, spec, stream=0):
    err = ctypes.create_string_buffer(256)
    rc = E.lib().lama_rfft2_noalloc(0, feat, batch, channels, h, w, spec, stream, err, 256)
    return rc, err.value.decode()


# Size and alignment checks return before any CUDA call, so the placeholder
# (non-null, never dereferenced) pointers below are safe on a machine without
# a GPU.
@pytest.mark.parametrize("args,code,msg", [
    ((1, 192, 1025, 64), LAMA_ESCRATCH, "limit of 1024 per side"),
    ((1, 192, 64, 2048), LAMA_ESCRATCH, "limit of 1024 per side"),
    ((64, 192, 64, 64), LAMA_ESCRATCH, "exceeds the fixed scratch of 2097152"),
    ((1, 192, 256, 256), LAMA_ESCRATCH, "exceeds the fixed scratch"),
    ((0, 192, 64, 64), LAMA_EINVAL, "must be positive"),
])
def test_rejects_requests_beyond_the_fixed_scratch(args, code, msg):
    rc, text = call(16, *args, 16)
    assert rc == code and msg in text


def test_rejects_null_pointers():
    rc, text = call(None, 1, 192, 64, 64, None)
    assert rc == LAMA_EINVAL and "null" in text


@pytest.mark.parametrize("feat,spec", [(18, 16), (16, 18), (17, 16), (16, 4099)])
def test_rejects_misaligned_pointers(feat, spec):
    rc, text = call(feat, 1, 192, 64, 64, spec)
    assert rc == LAMA_EINVAL and "4-byte aligned" in text


def _torch_spectrum(feat):
    """float64 rfft2 (ortho, reference directions) in the engine's spectrum
    layout [h][w/2+1][2c] with (2c, 2c+1) = (re, im)."""
    from torch_ref import rfft2_ortho
    sp = rfft2_ortho(feat.double())
    _, c, h, wh = sp.shape
    return torch.stack((sp.real, sp.imag), -1).permute(0, 2, 3, 1, 4).reshape(1, h, wh, 2 * c).numpy()


@pytest.mark.gpu
def test_noalloc_rfft2_matches_torch_and_the_engine_on_two_calls_in_a_row(engine_tamed):
    cases = [(256, 320, 91), (600, 520, 92)]  # latents 32x40 and 75x65
    feats, from_engine = [], []
    try:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_TWO_PASS)
        for h, w, seed in cases:
            _, _, x = make_input(h, w, seed)
            engine_tamed.debug_run(x, 7)
            name5, feat = engine_tamed.debug_read(1, h, w, 5)
            name6, spec = engine_tamed.debug_read(1, h, w, 6)
            assert (name5, name6) == ("spectral_conv1", "rfft2")
            feats.append(torch.from_numpy(np.ascontiguousarray(feat.reshape(1, 192, h // 8, w // 8))))
            from_engine.append(spec.reshape(1, h // 8, w // 16 + 1, 384))
    finally:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_AUTO)
    expected = [_torch_spectrum(f) for f in feats]
    d_feats = [f.cuda() for f in feats]
    outs = [torch.full((2,) + e.shape, float("nan"), dtype=torch.bfloat16, device="cuda") for e in expected]
    # a first call does the one-time set-up (and claims the fixed array);
    # after it, calls must leave the device's free memory as it was
    rc, msg = call(d_feats[0].data_ptr(), 1, 192, cases[0][0] // 8, cases[0][1] // 8, outs[0].data_ptr())
    assert rc == LAMA_OK, msg
    torch.cuda.synchronize()
    for o in outs:
        o.fill_(float("nan"))
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for (h, w, _), f, o in zip(cases, d_feats, outs):  # back to back on the default stream, one sync after
        rc, msg = call(f.data_ptr(), 1, 192, h // 8, w // 8, o.data_ptr())
        assert rc == LAMA_OK, msg
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    for o, e, eng in zip(outs, expected, from_engine):
        got = (o[0].float() + o[1].float()).cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - e).max() <= FFT_TOL * np.abs(e).max()
        assert np.abs(got - eng).max() <= FFT_TOL * np.abs(eng).max()
