"""Pin the CPU oracle (oracle/lama_oracle.cpp, a restatement of lama-rs/src/cpu.rs).

The reference ships no golden outputs for the network and its Rust engine
cannot be built offline, so the oracle is checked against an independent
PyTorch restatement (oracle/torch_ref.py: F.conv2d on reflect-padded input,
F.conv_transpose2d, torch FFTs) and its transforms against torch.fft.
"""

import numpy as np
import pytest
import torch

from conftest import make_input

import oracle as O
from torch_ref import TorchRef, irfft2_ortho, rfft2_ortho


def _pow2(n):
    return n & (n - 1) == 0


@pytest.mark.parametrize("h,w", [(64, 64), (32, 16), (8, 8), (16, 32), (4, 4)])
def test_rfft2_matches_torch_for_powers_of_two(h, w):
    a = np.random.default_rng(h * 100 + w).standard_normal((h, w)).astype(np.float32)
    s = O.rfft2(a)
    t = torch.fft.rfftn(torch.from_numpy(a).double(), norm="ortho")
    np.testing.assert_allclose(s[0], t.real.numpy(), atol=2e-6)
    np.testing.assert_allclose(s[1], t.imag.numpy(), atol=2e-6)


@pytest.mark.parametrize("h,w", [(64, 64), (16, 32), (8, 8)])
def test_irfft2_matches_torch_for_powers_of_two(h, w):
    sp = np.random.default_rng(h + w).standard_normal((2, h, w // 2 + 1)).astype(np.float32)
    got = O.irfft2(sp, w)
    exp = torch.fft.irfftn(torch.complex(torch.from_numpy(sp[0]).double(), torch.from_numpy(sp[1]).double()),
                           s=(h, w), norm="ortho").numpy()
    np.testing.assert_allclose(got, exp, atol=2e-6)


@pytest.mark.parametrize("h,w", [(75, 75), (9, 7), (8, 6), (6, 8), (25, 40), (1, 5)])
def test_non_power_of_two_transforms_run_the_opposite_direction(h, w):
    """cpu.rs:984-1011 (Bluestein) computes sum x_j e^{+2 pi i jk/n} when asked
    for the forward transform; the oracle must reproduce that, not torch.fft."""
    a = np.random.default_rng(1).standard_normal((h, w)).astype(np.float32)
    got = O.rfft2(a)
    exp = rfft2_ortho(torch.from_numpy(a).double(), reference_semantics=True)
    np.testing.assert_allclose(got[0], exp.real.numpy(), atol=3e-6)
    np.testing.assert_allclose(got[1], exp.imag.numpy(), atol=3e-6)
    sp = np.random.default_rng(2).standard_normal((2, h, w // 2 + 1)).astype(np.float32)
    inv = O.irfft2(sp, w)
    exp = irfft2_ortho(torch.complex(torch.from_numpy(sp[0]).double(), torch.from_numpy(sp[1]).double()), h, w,
                       reference_semantics=True)
    np.testing.assert_allclose(inv, exp.numpy(), atol=3e-6)
    if not (_pow2(h) and _pow2(w)):
        torch_sem = torch.fft.rfftn(torch.from_numpy(a).double(), norm="ortho")
        assert np.abs(got[1] - torch_sem.imag.numpy()).max() > 1e-2


def test_irfft2_inverts_rfft2():
    a = np.random.default_rng(3).standard_normal((64, 64)).astype(np.float32)
    np.testing.assert_allclose(O.irfft2(O.rfft2(a), 64), a, atol=2e-6)


@pytest.mark.parametrize("h,w,seed", [(64, 64, 1), (72, 56, 2), (40, 48, 3)])
def test_oracle_forward_matches_torch(weights_tamed, oracle_tamed, h, w, seed):
    from lama_b200 import seeded
    _, _, x = make_input(h, w, seed)
    got = oracle_tamed.forward(x)
    ref = TorchRef(dict(seeded.make_weights(res_scale=seeded.TAMED_RES_SCALE)))
    exp = ref.forward(x)[0]
    assert 0.0 < got.min() and got.max() < 1.0  # unsaturated: a sensitive comparison
    np.testing.assert_allclose(got, exp, atol=5e-6)


def test_oracle_step_dump_matches_the_encoder(weights_tamed, oracle_tamed):
    """LAMA_DUMP_STEP semantics (cpu.rs:488-546): after step 4 (model.4) the dump
    is local [128] then global [384] planes."""
    from lama_b200 import seeded
    _, _, x = make_input(32, 32, 4)
    d = oracle_tamed.forward_dump(x, 4)
    ref = TorchRef(dict(seeded.make_weights(res_scale=seeded.TAMED_RES_SCALE)))
    xl, xg = ref.encode(torch.from_numpy(x).double()[None])
    exp = np.concatenate([xl.numpy().ravel(), xg.numpy().ravel()])
    np.testing.assert_allclose(d, exp, atol=2e-5)


def test_build_input_and_composite_follow_main_rs():
    from lama_b200 import seeded
    rgb = seeded.value_noise(13, 11, 9)
    m = seeded.rect_mask(13, 11, 2, 3, 5, 6)
    x = O.build_input(rgb, m, 3, 5)
    assert x.shape == (4, 16, 16)
    # reflect extension (image.rs:159-169): padded row 13 reads row 11
    np.testing.assert_array_equal(x[:, 13, :11], x[:, 11, :11])
    mm = (m > 0).astype(np.float32)
    exp = (rgb.astype(np.float32) / np.float32(255.0)) * (np.float32(1.0) - mm)[..., None]
    np.testing.assert_array_equal(x[:3, :13, :11], exp.transpose(2, 0, 1))
    np.testing.assert_array_equal(x[3, :13, :11], mm)
    out = np.random.default_rng(0).uniform(-0.2, 1.2, (3, 16, 16)).astype(np.float32)
    c = O.composite(rgb, m, out)
    np.testing.assert_array_equal(c[m == 0], rgb[m == 0])
    q = (np.clip(out[:, :13, :11], 0, 1) * np.float32(255.0) + np.float32(0.5)).astype(np.uint8).transpose(1, 2, 0)
    np.testing.assert_array_equal(c[m > 0], q[m > 0])
