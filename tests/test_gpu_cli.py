"""End-to-end CLI runs on the GPU: whole image, --tile, --sections, stdin/stdout.

The whole-image and --tile outputs are checked against the oracle composite.
The --sections tests here are consistency checks, not parity: the CLI and the
device-resident driver (lama_inpaint_sections_u8) must give, bit for bit, the
bytes of the reference's orchestration (lama-rs/src/main.rs:465-566) written
in Python over the engine's per-window u8 entry point, which pins the section
geometry, window crops and write-back.  Parity of --sections with the oracle
is test_gpu_headline.py's.
"""

import os
import subprocess

import numpy as np
import pytest
from PIL import Image

import oracle as O
from lama_b200 import seeded
from lama_b200.engine import CLI_PATH, section_rects, tile_rect, window_origin

pytestmark = pytest.mark.gpu


def _write(tmp_path, img, mask):
    Image.fromarray(img).save(tmp_path / "in.png")
    Image.fromarray(mask).save(tmp_path / "mask.png")


def _cli(tmp_path, weights, *extra):
    r = subprocess.run([CLI_PATH, "--image", str(tmp_path / "in.png"), "--mask", str(tmp_path / "mask.png"),
                        "--output", str(tmp_path / "out.png"), "--weights", weights, *extra],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    return np.asarray(Image.open(tmp_path / "out.png"))


def test_cli_whole_image_matches_oracle(tmp_path, weights_tamed, oracle_tamed):
    img = seeded.value_noise(90, 70, 51)
    m = seeded.brush_mask(90, 70, 51)
    _write(tmp_path, img, m)
    got = _cli(tmp_path, weights_tamed)
    x = O.build_input(img, m, 6, 2)
    exp = O.composite(img, m, oracle_tamed.forward(x))
    d = np.abs(got.astype(int) - exp.astype(int))
    assert d.max() <= 1 and d[m > 0].mean() <= 0.1
    np.testing.assert_array_equal(got[m == 0], img[m == 0])


def test_cli_tile_matches_oracle(tmp_path, weights_tamed, oracle_tamed):
    h, w = 300, 360
    img = seeded.value_noise(h, w, 52)
    m = seeded.rect_mask(h, w, 200, 120, 40, 30)
    _write(tmp_path, img, m)
    got = _cli(tmp_path, weights_tamed, "--tile")
    x0, y0, side, _, _ = tile_rect(m)
    assert side == 296  # capped to the largest multiple of 8 inside the image
    sub, sm = img[y0:y0 + side, x0:x0 + side], m[y0:y0 + side, x0:x0 + side]
    win = O.composite(sub, sm, oracle_tamed.forward(O.build_input(sub, sm, 0, 0)))
    exp = img.copy()
    exp[y0:y0 + side, x0:x0 + side][sm > 0] = win[sm > 0]
    d = np.abs(got.astype(int) - exp.astype(int))
    assert d.max() <= 1
    np.testing.assert_array_equal(got[m == 0], img[m == 0])


def test_cli_sections_follow_the_reference_orchestration(tmp_path, weights_tamed, engine_tamed):
    h, w = 700, 760
    img = seeded.value_noise(h, w, 53)
    m = seeded.rect_mask(h, w, 100, 120, 520, 300)
    _write(tmp_path, img, m)
    got = _cli(tmp_path, weights_tamed, "--sections")
    working = img.copy()
    side = min(512, w, h)
    secs = section_rects(m)
    assert len(secs) > 1
    for x0, y0, x1, y1 in secs:
        wx = window_origin((x0 + x1) // 2, side, w)
        wy = window_origin((y0 + y1) // 2, side, h)
        sub = working[wy:wy + side, wx:wx + side].copy()
        sm = m[wy:wy + side, wx:wx + side].copy()
        yy, xx = np.mgrid[wy:wy + side, wx:wx + side]
        sm[~((xx >= x0) & (xx < x1) & (yy >= y0) & (yy < y1))] = 0
        filled = engine_tamed.inpaint_u8(sub, sm)
        blk = m[y0:y1, x0:x1] > 0
        working[y0:y1, x0:x1][blk] = filled[y0 - wy:y1 - wy, x0 - wx:x1 - wx][blk]
    np.testing.assert_array_equal(got, working)


def _host_sections(engine, img, m):
    """The reference's --sections loop (main.rs:465-566) written on the host:
    crop the working image, restrict the mask to the section, inpaint, paste."""
    h, w = m.shape
    working = img.copy()
    side = min(512, w, h)
    for x0, y0, x1, y1 in section_rects(m):
        wx = window_origin((x0 + x1) // 2, side, w)
        wy = window_origin((y0 + y1) // 2, side, h)
        sub = working[wy:wy + side, wx:wx + side].copy()
        sm = m[wy:wy + side, wx:wx + side].copy()
        yy, xx = np.mgrid[wy:wy + side, wx:wx + side]
        sm[~((xx >= x0) & (xx < x1) & (yy >= y0) & (yy < y1))] = 0
        filled = engine.inpaint_u8(sub, sm)
        blk = m[y0:y1, x0:x1] > 0
        working[y0:y1, x0:x1][blk] = filled[y0 - wy:y1 - wy, x0 - wx:x1 - wx][blk]
    return working


@pytest.mark.parametrize("h,w,kind,seed", [(700, 760, "rect", 61), (530, 610, "brush", 62), (300, 420, "rect", 63)])
def test_device_sections_match_the_host_loop(engine_tamed, h, w, kind, seed):
    """lama_inpaint_sections_u8 keeps the working image on the GPU between
    passes; it must give the host loop's bytes exactly."""
    img = seeded.value_noise(h, w, seed)
    if kind == "rect":
        m = seeded.rect_mask(h, w, w // 7, h // 6, w // 2 + 40, h // 2 + 30)  # x0, y0, width, height
    else:
        m = np.maximum(seeded.brush_mask(h, w, seed), seeded.rect_mask(h, w, 40, 50, w - 100, h - 90))
    rects = section_rects(m)
    side = min(512, w, h)
    got = engine_tamed.inpaint_sections_u8(img, m, rects, side)
    np.testing.assert_array_equal(got, _host_sections(engine_tamed, img, m))
    np.testing.assert_array_equal(got[m == 0], img[m == 0])


def test_device_sections_reject_a_rectangle_outside_its_window(engine_tamed):
    img = seeded.value_noise(600, 600, 64)
    m = seeded.rect_mask(600, 600, 10, 10, 580, 580)
    with pytest.raises(Exception, match="EINVAL"):
        engine_tamed.inpaint_sections_u8(img, m, [(0, 0, 600, 600)], 512)
    np.testing.assert_array_equal(engine_tamed.inpaint_sections_u8(img, m, [], 512), img)


def test_cli_stdin_and_stdout(tmp_path, weights_tamed, engine_tamed):
    img = seeded.value_noise(48, 56, 54)
    m = seeded.brush_mask(48, 56, 54)
    _write(tmp_path, img, m)
    with open(tmp_path / "in.png", "rb") as f:
        r = subprocess.run([CLI_PATH, "--image", "-", "--mask", str(tmp_path / "mask.png"), "--output", "-",
                            "--weights", weights_tamed], stdin=f, capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr
    import io
    got = np.asarray(Image.open(io.BytesIO(r.stdout)))
    np.testing.assert_array_equal(got, engine_tamed.inpaint_u8(img, m))


def test_cli_empty_mask_with_tile_copies_the_input(tmp_path, weights_tamed):
    img = seeded.value_noise(40, 40, 55)
    _write(tmp_path, img, np.zeros((40, 40), np.uint8))
    np.testing.assert_array_equal(_cli(tmp_path, weights_tamed, "--tile"), img)
