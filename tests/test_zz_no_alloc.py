"""lama_rfft2_noalloc (no counterpart in the reference): the two-pass rfft2
with its intermediate in a fixed device array, called through the C ABI.

The GPU test feeds it the engine's own conv1 output and compares with the
engine's rfft2 launch on the same data (lama_debug_run / lama_debug_read on
the two-pass spectral path), for two calls issued back to back on one stream
with different plane sizes.  This file is collected last on purpose: it must
pass alone in a fresh process and after every other test.
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


# Size checks return before any CUDA call, so the placeholder (non-null,
# never dereferenced) pointers below are safe on a machine without a GPU.
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


@pytest.mark.gpu
def test_noalloc_rfft2_matches_the_engine_on_two_calls_in_a_row(engine_tamed):
    cases = [(256, 320, 91), (600, 520, 92)]  # latents 32x40 and 75x65
    feats, expected = [], []
    try:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_TWO_PASS)
        for h, w, seed in cases:
            _, _, x = make_input(h, w, seed)
            engine_tamed.debug_run(x, 7)
            name5, feat = engine_tamed.debug_read(1, h, w, 5)
            name6, spec = engine_tamed.debug_read(1, h, w, 6)
            assert (name5, name6) == ("spectral_conv1", "rfft2")
            feats.append(torch.from_numpy(np.ascontiguousarray(feat.reshape(1, 192, h // 8, w // 8))).cuda())
            expected.append(spec.reshape(1, h // 8, w // 16 + 1, 384))
    finally:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_AUTO)
    outs = [torch.full((2,) + e.shape, float("nan"), dtype=torch.bfloat16, device="cuda") for e in expected]
    torch.cuda.synchronize()
    for (h, w, _), f, o in zip(cases, feats, outs):  # back to back on the default stream, one sync after
        rc, msg = call(f.data_ptr(), 1, 192, h // 8, w // 8, o.data_ptr())
        assert rc == LAMA_OK, msg
    torch.cuda.synchronize()
    for o, e in zip(outs, expected):
        got = (o[0].float() + o[1].float()).cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - e).max() <= FFT_TOL * np.abs(e).max()
