"""Parity of the B200 engine with the CPU oracle (a restatement of lama-rs/src/cpu.rs).

Tolerances (the reference is FP32; the engine computes convolutions as three
BF16 products of split operands with FP32 accumulation):
  * sigmoid output (pre-quantisation float): max |diff| <= 1e-4;
  * intermediate activations: max |diff| <= 1e-4 x max |expected| per layer,
    and <= 2e-3 x max |expected| after the 18-block stack with the BASELINE
    init, whose activations grow to ~1e10;
  * u8 composite: <= 1 level per pixel, mean <= 0.1 levels over masked
    pixels, unmasked pixels bit-exact (lama-rs/src/main.rs:272-307).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import make_input

import oracle as O

pytestmark = pytest.mark.gpu

FLOAT_TOL = 1e-4


def _interior(a, halo):
    if halo:
        a = a[:, halo:-halo, halo:-halo, :]
    return a.transpose(0, 3, 1, 2)


def test_encoder_and_first_block_layer_by_layer(engine_tamed):
    """Every launch of the encoder and of resblock model.5 against float64 torch."""
    from lama_b200 import plan, seeded
    from torch_ref import TorchRef, irfft2_ortho, rfft2_ortho
    h = w = 64
    _, _, x = make_input(h, w, 11)
    ref = TorchRef(dict(seeded.make_weights(res_scale=seeded.TAMED_RES_SCALE)))
    xt = F.pad(torch.from_numpy(x).double()[None], (3, 3, 3, 3), mode="reflect")
    exp = []
    xl, xg = xt, None
    with torch.no_grad():
        for b in plan.encoder():
            xl, xg = ref.ffc(b, xl, xg)
            exp.append(xl if xg is None else torch.cat([xl, xg], 1))
        XA = exp[-1]
        b1, b2 = plan.resblocks()[0]
        p = b1.ffc_prefix + ".convg2g"
        xl, xg = XA[:, :128], XA[:, 128:]
        feat = ref.bn(F.conv2d(xg, ref.t[p + ".conv1.0.weight"]), p + ".conv1.1")
        sp = rfft2_ortho(feat)
        st = torch.stack((sp.real, sp.imag), -1).permute(0, 1, 4, 2, 3).reshape(1, 384, 8, 5)
        fu = ref.bn(F.conv2d(st, ref.t[p + ".fu.conv_layer.weight"]), p + ".fu.bn")
        y = fu.reshape(1, 192, 2, 8, 5).permute(0, 1, 3, 4, 2)
        S = feat + irfft2_ortho(torch.complex(y[..., 0].contiguous(), y[..., 1].contiguous()), 8, 8)
        l1, g1 = ref.ffc(b1, xl, xg)
        l2, g2 = ref.ffc(b2, l1, g1)
    expected = {
        1: exp[0].numpy(), 2: exp[1].numpy(), 3: exp[2].numpy(), 4: exp[3].numpy(),
        5: feat.numpy(), 6: st.numpy().transpose(0, 2, 3, 1),
        7: fu.numpy().transpose(0, 2, 3, 1).reshape(1, 1, 40, 384), 8: S.numpy().transpose(0, 2, 3, 1),
        9: torch.cat([l1, g1], 1).numpy(), 14: torch.cat([xl + l2, xg + g2], 1).numpy(),
    }
    names = {1: "model1_7x7", 2: "model2_3x3s2", 3: "model3_3x3s2", 4: "model4_3x3s2", 5: "spectral_conv1",
             6: "rfft2", 7: "fourier_conv", 8: "irfft2", 9: "ffc_out", 14: "ffc_out"}
    for op, e in expected.items():
        engine_tamed.debug_run(x, op + 1)
        name, got = engine_tamed.debug_read(1, h, w, op)
        assert name == names[op]
        if op in (1, 2, 3, 4, 9, 14):
            got = _interior(got, 1)
        got = got.reshape(e.shape)
        err = np.abs(got - e).max() / np.abs(e).max()
        assert err < 1e-4, (name, err)


@pytest.mark.parametrize("h,w,seed", [(64, 64, 1), (72, 56, 2), (128, 128, 3), (48, 80, 4), (8, 8, 5), (24, 40, 6)])
def test_forward_matches_oracle(engine_tamed, oracle_tamed, h, w, seed):
    """Includes non-power-of-two latents (9x7, 6x10, 3x5: the reference's
    opposite-direction Bluestein transforms) and the 1x1 latent of an 8x8 input."""
    _, _, x = make_input(h, w, seed)
    got = engine_tamed.forward(x)
    exp = oracle_tamed.forward(x)
    assert np.abs(got - exp).max() <= FLOAT_TOL


def test_batch_equals_single_images(engine_tamed):
    xs = np.stack([make_input(64, 64, s)[2] for s in (21, 22, 23)])
    batch = engine_tamed.forward(xs)
    for i in range(3):
        np.testing.assert_array_equal(batch[i], engine_tamed.forward(xs[i]))


def test_forward_is_deterministic(engine_tamed):
    _, _, x = make_input(64, 64, 7)
    np.testing.assert_array_equal(engine_tamed.forward(x), engine_tamed.forward(x))


def test_streamed_inpaint_equals_per_chunk_calls(engine_tamed):
    """lama_inpaint_u8_stream (copies overlapping the passes, a ragged last
    chunk) gives the bytes of lama_inpaint_u8 chunk by chunk."""
    from lama_b200 import seeded
    n, h, w, chunk = 7, 72, 88, 3
    rgb = np.stack([seeded.value_noise(h, w, 70 + i) for i in range(n)])
    mask = np.stack([seeded.brush_mask(h, w, 70 + i) for i in range(n)])
    got = engine_tamed.inpaint_u8_stream(rgb, mask, chunk)
    exp = np.concatenate([engine_tamed.inpaint_u8(rgb[i:i + chunk], mask[i:i + chunk]) for i in range(0, n, chunk)])
    np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("h,w,seed", [(64, 64, 31), (61, 77, 32), (96, 40, 33)])
def test_inpaint_u8_matches_oracle_composite(engine_tamed, oracle_tamed, h, w, seed):
    img, m, x = make_input(h, w, seed)
    got = engine_tamed.inpaint_u8(img, m)
    exp = O.composite(img, m, oracle_tamed.forward(x))
    d = np.abs(got.astype(int) - exp.astype(int))
    assert d.max() <= 1
    assert d[m > 0].mean() <= 0.1
    np.testing.assert_array_equal(got[m == 0], img[m == 0])


def test_inpaint_u8_empty_and_full_masks(engine_tamed, oracle_tamed):
    img, _, _ = make_input(32, 32, 41)
    empty = np.zeros((32, 32), np.uint8)
    np.testing.assert_array_equal(engine_tamed.inpaint_u8(img, empty), img)
    full = np.full((32, 32), 255, np.uint8)
    got = engine_tamed.inpaint_u8(img, full)
    exp = O.composite(img, full, oracle_tamed.forward(O.build_input(img, full, 0, 0)))
    assert np.abs(got.astype(int) - exp.astype(int)).max() <= 1


def test_resblock_stack_with_baseline_init(engine_baseline, oracle_baseline):
    """Config 1 (the 18-block stack) with the BASELINE init, whose activations
    grow ~3.5x per block: relative error stays bounded."""
    rng = np.random.default_rng(5)
    l = rng.standard_normal((128, 16, 16)).astype(np.float32)
    g = rng.standard_normal((384, 16, 16)).astype(np.float32)
    gl, gg = engine_baseline.resblocks(l, g, 18)
    el, eg = oracle_baseline.resblocks(l, g, 18)
    scale = max(np.abs(el).max(), np.abs(eg).max())
    assert scale > 1e6
    assert np.abs(gl - el).max() / scale < 2e-3
    assert np.abs(gg - eg).max() / scale < 2e-3


def test_resblock_stack_tamed_and_partial_depth(engine_tamed, oracle_tamed):
    rng = np.random.default_rng(6)
    l = rng.standard_normal((128, 8, 8)).astype(np.float32)
    g = rng.standard_normal((384, 8, 8)).astype(np.float32)
    for nb in (0, 1, 18):
        gl, gg = engine_tamed.resblocks(l, g, nb)
        el, eg = oracle_tamed.resblocks(l, g, nb)
        scale = max(np.abs(el).max(), np.abs(eg).max())
        assert np.abs(gl - el).max() / scale < 1e-4, nb
        assert np.abs(gg - eg).max() / scale < 1e-4, nb


def test_baseline_init_full_pass(engine_baseline, oracle_baseline):
    """With the BASELINE init the sigmoid saturates; the saturated output and
    the last resblock's activations (~1e10) still match."""
    _, _, x = make_input(64, 64, 8)
    got = engine_baseline.forward(x)
    exp = oracle_baseline.forward(x)
    assert np.abs(got - exp).max() <= FLOAT_TOL
    names = engine_baseline.op_names(1, 64, 64)
    last = max(i for i, n in enumerate(names) if n == "ffc_out")
    engine_baseline.debug_run(x, last + 1)
    _, got_x = engine_baseline.debug_read(1, 64, 64, last)
    dump = oracle_baseline.forward_dump(x, 22)
    exp_x = np.concatenate([dump[: 128 * 64].reshape(128, 8, 8), dump[128 * 64:].reshape(384, 8, 8)])
    got_x = _interior(got_x, 1)[0]
    assert np.abs(got_x - exp_x).max() / np.abs(exp_x).max() < 2e-3


def test_invalid_sizes_are_errors(engine_tamed):
    from lama_b200 import LamaError
    with pytest.raises(LamaError) as ei:
        engine_tamed.forward(np.zeros((4, 60, 64), np.float32))
    assert ei.value.code == -1 and "multiples of 8" in ei.value.msg


def test_bad_device_is_an_error(weights_tamed):
    from lama_b200 import Engine, LamaError
    with pytest.raises(LamaError) as ei:
        Engine(weights_tamed, 4096)
    assert ei.value.code == -1


def test_full_size_512_batch_properties(engine_baseline):
    """Config 0 geometry at full size: finite, in [0,1], deterministic, and
    identical inputs in a batch give identical outputs."""
    _, _, x = make_input(512, 512, 0)
    xs = np.stack([x, x])
    a = engine_baseline.forward(xs)
    assert np.isfinite(a).all() and a.min() >= 0 and a.max() <= 1
    np.testing.assert_array_equal(a[0], a[1])
    np.testing.assert_array_equal(a, engine_baseline.forward(xs))


@pytest.mark.parametrize("policy", [1, 2, 3])
def test_tiling_policies_compute_the_same_pass(engine_tamed, oracle_tamed, policy):
    """Channel-major (swapped), pixel-major and CTA-pair GEMM tiles all match
    the oracle (odd tile counts give CTA pairs a dummy second tile)."""
    try:
        engine_tamed.set_tiling(policy)
        for h, w, seed in [(64, 64, 61), (72, 56, 62), (128, 96, 63)]:
            _, _, x = make_input(h, w, seed)
            got = engine_tamed.forward(x)
            assert np.abs(got - oracle_tamed.forward(x)).max() <= FLOAT_TOL, (policy, h, w)
        xs = np.stack([make_input(64, 64, s)[2] for s in (64, 65)])
        np.testing.assert_array_equal(engine_tamed.forward(xs)[1], engine_tamed.forward(xs[1]))
    finally:
        engine_tamed.set_tiling(0)


@pytest.mark.parametrize("path", [1, 2])
def test_spectral_paths_compute_the_same_pass(engine_tamed, oracle_tamed, path):
    """Two-pass and register-resident spectral kernels both match the oracle,
    single images and a batch (the automatic choice depends on the batch)."""
    try:
        engine_tamed.set_spectral_path(path)
        for h, w, seed in [(64, 64, 71), (128, 128, 72), (72, 56, 73)]:
            _, _, x = make_input(h, w, seed)
            assert np.abs(engine_tamed.forward(x) - oracle_tamed.forward(x)).max() <= FLOAT_TOL, (path, h, w)
        xs = np.stack([make_input(64, 64, s)[2] for s in (74, 75)])
        got = engine_tamed.forward(xs)
        for i in range(2):
            assert np.abs(got[i] - oracle_tamed.forward(xs[i])).max() <= FLOAT_TOL, (path, i)
    finally:
        engine_tamed.set_spectral_path(0)


@pytest.mark.parametrize("h,w,path", [(512, 512, 1), (512, 512, 2), (512, 512, 3), (256, 128, 2), (1024, 1024, 0),
                                      (2048, 2048, 0), (600, 600, 0), (520, 776, 0)])
def test_spectral_kernels_on_large_latents(engine_tamed, h, w, path):
    """rfft2 and irfft2 (+ the FourierUnit residual) of the first resblock at
    latents 64^2 (both spectral paths), 32x16 (register path), 128^2, 256^2
    75^2 (the --tile window of config 2) and 65x97
    against float64 torch with the reference's transform directions, on the
    engine's own conv1 / FourierUnit-conv outputs."""
    from torch_ref import irfft2_ortho, rfft2_ortho
    _, _, x = make_input(h, w, 81)
    lh, lw = h // 8, w // 8
    try:
        engine_tamed.set_spectral_path(path)
        engine_tamed.debug_run(x, 9)
        reads = {op: engine_tamed.debug_read(1, h, w, op) for op in (5, 6, 7, 8)}
    finally:
        engine_tamed.set_spectral_path(0)
    assert [reads[op][0] for op in (5, 6, 7, 8)] == ["spectral_conv1", "rfft2", "fourier_conv", "irfft2"]
    feat = torch.from_numpy(reads[5][1].reshape(1, 192, lh, lw)).double()
    sp = rfft2_ortho(feat)
    exp_spec = torch.stack((sp.real, sp.imag), -1).permute(0, 2, 3, 1, 4).reshape(1, lh, lw // 2 + 1, 384).numpy()
    got_spec = reads[6][1].reshape(exp_spec.shape)
    assert np.abs(got_spec - exp_spec).max() <= 1e-4 * np.abs(exp_spec).max()
    fu = torch.from_numpy(reads[7][1].reshape(1, lh, lw // 2 + 1, 192, 2)).double()
    fc = torch.complex(fu[..., 0], fu[..., 1]).permute(0, 3, 1, 2)
    exp_s = (feat + irfft2_ortho(fc, lh, lw)).permute(0, 2, 3, 1).numpy()
    got_s = reads[8][1].reshape(exp_s.shape)
    assert np.abs(got_s - exp_s).max() <= 1e-4 * np.abs(exp_s).max()


def test_swapped_tiles_match_pixel_tiles_on_the_baseline_stack(engine_baseline):
    rng = np.random.default_rng(9)
    l = rng.standard_normal((2, 128, 16, 16)).astype(np.float32)
    g = rng.standard_normal((2, 384, 16, 16)).astype(np.float32)
    try:
        engine_baseline.set_tiling(1)
        a = engine_baseline.resblocks(l, g, 18)
        engine_baseline.set_tiling(2)
        b = engine_baseline.resblocks(l, g, 18)
        engine_baseline.set_tiling(3)
        c = engine_baseline.resblocks(l, g, 18)
    finally:
        engine_baseline.set_tiling(0)
    scale = max(np.abs(b[0]).max(), np.abs(b[1]).max())
    assert np.abs(a[0] - b[0]).max() / scale < 1e-3 and np.abs(a[1] - b[1]).max() / scale < 1e-3
    assert np.abs(c[0] - b[0]).max() / scale < 1e-3 and np.abs(c[1] - b[1]).max() / scale < 1e-3


def test_a_device_wait_that_runs_out_is_reported_and_the_engine_recovers(engine_tamed, oracle_tamed):
    """Failure detection without a GPU fault: a kernel wait on a barrier that
    nothing arrives on gives up after its limit and records its code; the call
    reports EDEVICE and the next pass on the same engine is still correct."""
    from lama_b200.engine import LamaError
    with pytest.raises(LamaError) as ei:
        engine_tamed.debug_wait_timeout(20)
    assert ei.value.code == -4 and "timed out" in ei.value.msg and "code 6" in ei.value.msg
    _, _, x = make_input(64, 64, 91)
    assert np.abs(engine_tamed.forward(x) - oracle_tamed.forward(x)).max() <= FLOAT_TOL


def test_prefetching_rfft_matches_the_register_path_over_a_batch(engine_tamed):
    """The persistent prefetching rfft2 (64x64 planes) runs min(items, 2 x 148)
    CTAs; with 16 images x 48 channel groups = 768 items on 296 CTAs every CTA
    walks two or three items through its TMA landing zone, prefetching the
    next item's rows while it computes; the pass must match the register path."""
    base = [make_input(512, 512, s)[2] for s in (95, 96, 97, 98)]
    xs = np.stack([np.roll(base[i % 4], 29 * (i // 4), axis=2) for i in range(16)])
    try:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_REGISTER)
        ref = engine_tamed.forward(xs)
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_PREFETCH)
        got = engine_tamed.forward(xs)
        np.testing.assert_array_equal(got, engine_tamed.forward(xs))  # deterministic
    finally:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_AUTO)
    assert np.abs(got - ref).max() <= FLOAT_TOL


def test_small_batch_lanes_and_union_pairs_match_the_oracle(engine_tamed, oracle_tamed):
    """A batch-1 512x512 pass runs its FFC layers on two graph lanes (the
    spectral chain beside the FFC GEMM's local class and l2g parts, then a
    tail launch with conv2 that finishes the global class) with CTA-pair
    row-union tiles and split K; with one lane, and with single-CTA pixel
    tiles, the pass is the same function: all three against the oracle."""
    _, _, x = make_input(512, 512, 99)
    exp = oracle_tamed.forward(x)
    got = {}
    try:
        got["lanes"] = engine_tamed.forward(x)
        engine_tamed.set_lanes(0)
        got["one lane"] = engine_tamed.forward(x)
        engine_tamed.set_tiling(engine_tamed.TILING_PIXEL)
        got["pixel tiles"] = engine_tamed.forward(x)
    finally:
        engine_tamed.set_lanes(-1)
        engine_tamed.set_tiling(engine_tamed.TILING_AUTO)
    for k, v in got.items():
        assert np.abs(v - exp).max() <= FLOAT_TOL, k
    np.testing.assert_array_equal(got["lanes"], engine_tamed.forward(x))  # deterministic


def test_batched_transforms_at_batch_16_against_float64(engine_tamed):
    """At 16 images per pass the automatic path runs the 64x64 transforms as
    the tensor-core rfft2 (walking (image, 4 channels) items) and the
    16-channel parity-split irfft2; the spectrum and S = feat + irfft2(fu) of
    the first resblock against float64 torch for two images of the batch."""
    from torch_ref import irfft2_ortho, rfft2_ortho
    base = [make_input(512, 512, s)[2] for s in (111, 112, 113, 114)]
    xs = np.stack([np.roll(base[i % 4], 17 * (i // 4), axis=1) for i in range(16)])
    engine_tamed.debug_run(xs, 9)
    reads = {op: engine_tamed.debug_read(16, 512, 512, op) for op in (5, 6, 7, 8)}
    assert [reads[op][0] for op in (5, 6, 7, 8)] == ["spectral_conv1", "rfft2", "fourier_conv", "irfft2"]
    for i in (0, 13):
        feat = torch.from_numpy(reads[5][1][i].reshape(1, 192, 64, 64)).double()
        sp = rfft2_ortho(feat)
        exp_spec = torch.stack((sp.real, sp.imag), -1).permute(0, 2, 3, 1, 4).reshape(64, 33, 384).numpy()
        got_spec = reads[6][1][i].reshape(64, 33, 384)
        assert np.abs(got_spec - exp_spec).max() <= 1e-4 * np.abs(exp_spec).max()
        fu = torch.from_numpy(reads[7][1][i].reshape(1, 64, 33, 192, 2)).double()
        fc = torch.complex(fu[..., 0], fu[..., 1]).permute(0, 3, 1, 2)
        exp_s = (feat + irfft2_ortho(fc, 64, 64)).permute(0, 2, 3, 1).numpy()[0]
        got_s = reads[8][1][i].reshape(64, 64, 192)
        assert np.abs(got_s - exp_s).max() <= 1e-4 * np.abs(exp_s).max()


def test_tensor_core_rfft_against_float64_over_a_batch(engine_tamed, oracle_tamed):
    """The tensor-core rfft2 (two split-BF16 DFT GEMMs per (image, 4 channels)
    item, one persistent CTA per SM walking 768 items at 16 images): the
    spectrum of the first resblock against float64 torch on the engine's own
    conv1 output, and S = feat + irfft2(fu) after it, for two images of the
    batch; and a single-image pass with it against the oracle."""
    from torch_ref import irfft2_ortho, rfft2_ortho
    base = [make_input(512, 512, s)[2] for s in (121, 122, 123, 124)]
    xs = np.stack([np.roll(base[i % 4], 23 * (i // 4), axis=2) for i in range(16)])
    try:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_TENSOR)
        engine_tamed.debug_run(xs, 9)
        reads = {op: engine_tamed.debug_read(16, 512, 512, op) for op in (5, 6, 7, 8)}
        _, _, x = make_input(512, 512, 125)
        single = engine_tamed.forward(x)
    finally:
        engine_tamed.set_spectral_path(engine_tamed.SPECTRAL_AUTO)
    assert [reads[op][0] for op in (5, 6, 7, 8)] == ["spectral_conv1", "rfft2", "fourier_conv", "irfft2"]
    for i in (0, 13):
        feat = torch.from_numpy(reads[5][1][i].reshape(1, 192, 64, 64)).double()
        sp = rfft2_ortho(feat)
        exp_spec = torch.stack((sp.real, sp.imag), -1).permute(0, 2, 3, 1, 4).reshape(64, 33, 384).numpy()
        got_spec = reads[6][1][i].reshape(64, 33, 384)
        assert np.abs(got_spec - exp_spec).max() <= 1e-4 * np.abs(exp_spec).max(), i
        fu = torch.from_numpy(reads[7][1][i].reshape(1, 64, 33, 192, 2)).double()
        fc = torch.complex(fu[..., 0], fu[..., 1]).permute(0, 3, 1, 2)
        exp_s = (feat + irfft2_ortho(fc, 64, 64)).permute(0, 2, 3, 1).numpy()[0]
        got_s = reads[8][1][i].reshape(64, 64, 192)
        assert np.abs(got_s - exp_s).max() <= 1e-4 * np.abs(exp_s).max(), i
    assert np.abs(single - oracle_tamed.forward(x)).max() <= FLOAT_TOL
