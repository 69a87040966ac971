"""Parity of the configurations the benchmark and the north star quote, against
the CPU oracle (a restatement of lama-rs/src/cpu.rs).

* the bench's pass: one lama_inpaint_u8_device chunk of 64 pairs at 512x512
  (CTA-pair GEMM tiles, the tensor-core rfft2 walking ~21 (image, channel
  group) items per CTA, the parity-split irfft2, the composite fused into the
  OutConv), two images against the oracle composite and every image against
  a batch-1 call;
* the 18-block stack at the 64x64 latent with the BASELINE init, batch 8;
* the reference's own example inputs (testdata/in.png, mask.png) through the
  CLI;
* config 2: --tile on a 2048x2048 image with a 300x300 hole (600x600
  window, 75x75 latent: non-power-of-two transforms), the whole output image;
* a 1024x1024 whole-image pass, pre-quantisation floats;
* device --sections against the reference's loop (main.rs:465-566) written
  over the oracle.

Tolerances (as in test_gpu_parity.py): sigmoid output max |diff| <= 1e-4;
u8 composite <= 1 level, mean <= 0.1 levels over masked pixels, unmasked
pixels bit-exact (main.rs:272-307).
"""

import os
import subprocess

import numpy as np
import pytest
import torch
from PIL import Image

import oracle as O
from conftest import make_input
from lama_b200 import seeded
from lama_b200.engine import CLI_PATH, section_rects, tile_rect, window_origin

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
FLOAT_TOL = 1e-4


def _check_u8(got, img, m, exp, max_levels=1):
    d = np.abs(got.astype(int) - exp.astype(int))
    assert d.max() <= max_levels, d.max()
    assert d[m > 0].mean() <= 0.1, d[m > 0].mean()
    np.testing.assert_array_equal(got[m == 0], img[m == 0])


def _headline_inputs(n, size=512):
    """n distinct pairs: 16 seeded value-noise images and brush masks, each
    reused four times rolled by a different offset (cheap to make, and no two
    pairs of the chunk alike)."""
    base = [(seeded.value_noise(size, size, 3000 + i), seeded.brush_mask(size, size, 3000 + i)) for i in range(16)]
    rgb = np.stack([np.roll(base[i % 16][0], 37 * (i // 16), axis=1) for i in range(n)])
    mask = np.stack([np.roll(base[i % 16][1], -53 * (i // 16), axis=0) for i in range(n)])
    return rgb, mask


def test_bench_chunk_of_64_matches_the_oracle(engine_tamed, oracle_tamed):
    n = 64
    rgb, mask = _headline_inputs(n)
    d_rgb, d_mask = torch.from_numpy(rgb).cuda(), torch.from_numpy(mask).cuda()
    d_out = torch.empty_like(d_rgb)
    engine_tamed.inpaint_u8_device(d_rgb.data_ptr(), d_mask.data_ptr(), d_out.data_ptr(), n, 512, 512)
    engine_tamed.synchronize()
    got = d_out.cpu().numpy()
    for i in (0, 45):
        x = O.build_input(rgb[i], mask[i], 0, 0)
        _check_u8(got[i], rgb[i], mask[i], O.composite(rgb[i], mask[i], oracle_tamed.forward(x)))
    # every image of the chunk against the same image alone (batch 1 runs
    # split-K GEMM tiles and one transform item per CTA, so up to one level)
    for i in range(n):
        one = engine_tamed.inpaint_u8(rgb[i], mask[i])
        _check_u8(got[i], rgb[i], mask[i], one)
    # and the chunk is deterministic
    engine_tamed.inpaint_u8_device(d_rgb.data_ptr(), d_mask.data_ptr(), d_out.data_ptr(), n, 512, 512)
    engine_tamed.synchronize()
    np.testing.assert_array_equal(d_out.cpu().numpy(), got)


def test_stack_at_the_64x64_latent_with_the_baseline_init_batch_8(engine_baseline, oracle_baseline):
    """The FFC layers exactly as the 512x512 pass runs them (64x64 latent,
    512 channels), eight images per launch; activations grow to ~1e10."""
    rng = np.random.default_rng(12)
    l = rng.standard_normal((8, 128, 64, 64)).astype(np.float32)
    g = rng.standard_normal((8, 384, 64, 64)).astype(np.float32)
    gl, gg = engine_baseline.resblocks(l, g, 18)
    for i in (0, 5):
        el, eg = oracle_baseline.resblocks(l[i], g[i], 18)
        scale = max(np.abs(el).max(), np.abs(eg).max())
        assert scale > 1e6
        assert np.abs(gl[i] - el).max() / scale < 2e-3
        assert np.abs(gg[i] - eg).max() / scale < 2e-3


def _cli(tmp_path, weights, image, mask, *extra):
    out = tmp_path / "out.png"
    r = subprocess.run([CLI_PATH, "--image", str(image), "--mask", str(mask), "--output", str(out),
                        "--weights", weights, *extra], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr
    return np.asarray(Image.open(out))


def test_reference_testdata_through_the_cli(tmp_path, weights_tamed, oracle_tamed):
    """The reference's example pair (512x512, 14.5 % masked) end to end."""
    ip, mp = os.path.join(GOLDEN, "ref_testdata_in.png"), os.path.join(GOLDEN, "ref_testdata_mask.png")
    img = np.asarray(Image.open(ip).convert("RGB"))
    m = np.asarray(Image.open(mp).convert("L"))
    assert img.shape == (512, 512, 3) and int((m > 0).sum()) == 38000
    got = _cli(tmp_path, weights_tamed, ip, mp)
    exp = O.composite(img, m, oracle_tamed.forward(O.build_input(img, m, 0, 0)))
    _check_u8(got, img, m, exp)


def test_config2_tile_window_on_a_2048_image(tmp_path, weights_tamed, oracle_tamed):
    """a 300x300 hole in a 2048x2048 image gives a 600x600
    window (latent 75x75); the whole output image against the oracle."""
    h = w = 2048
    img = seeded.value_noise(h, w, 401)
    m = seeded.rect_mask(h, w, 911, 604, 300, 300)
    Image.fromarray(img).save(tmp_path / "in.png")
    Image.fromarray(m).save(tmp_path / "mask.png")
    got = _cli(tmp_path, weights_tamed, tmp_path / "in.png", tmp_path / "mask.png", "--tile")
    x0, y0, side, bw, bh = tile_rect(m)
    assert (side, bw, bh) == (600, 300, 300)
    sub, sm = img[y0:y0 + side, x0:x0 + side], m[y0:y0 + side, x0:x0 + side]
    win = O.composite(sub, sm, oracle_tamed.forward(O.build_input(sub, sm, 0, 0)))
    exp = img.copy()
    exp[y0:y0 + side, x0:x0 + side][sm > 0] = win[sm > 0]
    _check_u8(got, img, m, exp)


def test_1024_whole_pass_floats(engine_tamed, oracle_tamed):
    _, _, x = make_input(1024, 1024, 402)
    got = engine_tamed.forward(x)
    exp = oracle_tamed.forward(x)
    assert np.abs(got - exp).max() <= FLOAT_TOL


def _oracle_sections(orc, img, m):
    """The reference's --sections loop (lama-rs/src/main.rs:465-566) over the
    oracle: the working image accumulates each pass's fill, each pass masks
    only its own section inside its window, and writes back only that
    section's masked pixels."""
    h, w = m.shape
    working = img.copy()
    side = min(512, w, h)
    pad = (8 - side % 8) % 8
    for x0, y0, x1, y1 in section_rects(m):
        wx = window_origin((x0 + x1) // 2, side, w)
        wy = window_origin((y0 + y1) // 2, side, h)
        sub = working[wy:wy + side, wx:wx + side].copy()
        sm = m[wy:wy + side, wx:wx + side].copy()
        yy, xx = np.mgrid[wy:wy + side, wx:wx + side]
        sm[~((xx >= x0) & (xx < x1) & (yy >= y0) & (yy < y1))] = 0
        filled = O.composite(sub, sm, orc.forward(O.build_input(sub, sm, pad, pad)))
        blk = m[y0:y1, x0:x1] > 0
        working[y0:y1, x0:x1][blk] = filled[y0 - wy:y1 - wy, x0 - wx:x1 - wx][blk]
    return working


def test_device_sections_match_the_reference_loop_over_the_oracle(engine_tamed, oracle_tamed):
    """300x420 image, 300x300 windows, two sections.  A later pass reads the
    earlier passes' fills as context, so a one-level difference there can move
    a later pixel across a rounding boundary: two levels are allowed outside
    the first section, one inside it."""
    h, w = 300, 420
    img = seeded.value_noise(h, w, 403)
    m = seeded.rect_mask(h, w, 40, 50, 340, 200)
    rects = section_rects(m)
    assert len(rects) >= 2
    got = engine_tamed.inpaint_sections_u8(img, m, rects, min(512, w, h))
    exp = _oracle_sections(oracle_tamed, img, m)
    d = np.abs(got.astype(int) - exp.astype(int))
    x0, y0, x1, y1 = rects[0]
    assert d[y0:y1, x0:x1].max() <= 1
    assert d.max() <= 2 and d[m > 0].mean() <= 0.1
    np.testing.assert_array_equal(got[m == 0], img[m == 0])
