"""Shared fixtures: seeded weight files, the CPU oracle, the B200 engine.

`-m "not gpu"` runs everything that needs no GPU (oracle pinning, weight
container, host logic, ABI exports); `-m gpu` runs the parity tests through
the C ABI on a B200.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "lama-inpaint-rs_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the engine's C ABI)")


def have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def weights_tamed(tmp_path_factory):
    """Seeded weights with resblock convs scaled so the output is unsaturated."""
    from lama_b200 import seeded
    p = tmp_path_factory.mktemp("w") / "tamed.safetensors"
    seeded.write_weights(str(p), res_scale=seeded.TAMED_RES_SCALE)
    return str(p)


@pytest.fixture(scope="session")
def weights_baseline(tmp_path_factory):
    """Seeded weights exactly as the benchmark configuration specifies."""
    from lama_b200 import seeded
    p = tmp_path_factory.mktemp("w") / "baseline.safetensors"
    seeded.write_weights(str(p))
    return str(p)


@pytest.fixture(scope="session")
def oracle_tamed(weights_tamed):
    import oracle as O
    return O.Oracle(weights_tamed)


@pytest.fixture(scope="session")
def oracle_baseline(weights_baseline):
    import oracle as O
    return O.Oracle(weights_baseline)


@pytest.fixture(scope="session")
def engine_tamed(weights_tamed):
    if not have_gpu():
        pytest.skip("no GPU")
    from lama_b200 import Engine
    e = Engine(weights_tamed, 0)
    yield e
    e.close()


@pytest.fixture(scope="session")
def engine_baseline(weights_baseline):
    if not have_gpu():
        pytest.skip("no GPU")
    from lama_b200 import Engine
    e = Engine(weights_baseline, 0)
    yield e
    e.close()


def make_input(h, w, seed, rect=None):
    """u8 image, u8 mask and the [4,h,w] network input built by the oracle's build_input."""
    import oracle as O
    from lama_b200 import seeded
    img = seeded.value_noise(h, w, seed)
    if rect is None:
        m = seeded.brush_mask(h, w, seed)
    else:
        m = seeded.rect_mask(h, w, *rect)
    ph, pw = (8 - h % 8) % 8, (8 - w % 8) % 8
    return img, m, O.build_input(img, m, ph, pw)
