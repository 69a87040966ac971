"""The CPU oracle against the reference's own CUDA kernels.

`oracle/_ref/ref_cuda_bench` (built by `build()` where the reference checkout is
present) compiles the reference's `lama-rs/cuda/lama.cu` and drives it in the
launch order of the reference's `cuda::run`, with the checkpoint's weights.
Apart from the five kernels of the reference's absent toolkit dependency
(stand-ins there: cuFFT for the 2-D transforms, one-line elementwise kernels),
every number it produces comes from the reference's own device code, so its
agreement with the oracle pins the oracle to the reference beyond the
restatement itself.  Tolerance: the engine's own, max |diff| <= 1e-4 on the
sigmoid output.
"""

import os
import subprocess

import numpy as np
import pytest

from conftest import make_input

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "ref_cuda_bench")
TOL = 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("h,w,seed", [(64, 64, 81), (128, 128, 82)])
def test_oracle_agrees_with_the_reference_cuda_kernels(tmp_path, weights_tamed, oracle_tamed, h, w, seed):
    if not os.path.exists(BIN):
        pytest.skip("reference CUDA harness not built (no reference checkout where build() ran)")
    _, _, x = make_input(h, w, seed)
    src, dst = tmp_path / "in.f32", tmp_path / "out.f32"
    np.ascontiguousarray(x, np.float32).tofile(src)
    r = subprocess.run([BIN, "--run", weights_tamed, str(src), str(dst), str(h), str(w)], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(dst, np.float32).reshape(3, h, w)
    exp = oracle_tamed.forward(x)
    assert np.isfinite(got).all()
    err = float(np.abs(got - exp).max())
    assert err <= TOL, f"reference CUDA kernels differ from the oracle by {err}"
