"""--tile / --sections geometry, through the C ABI (no GPU).

These restate, case for case, the reference CLI's own unit tests
(lama-rs/src/main.rs:801-1158) against this repo's implementation
(lama-inpaint-rs_b200/host/geometry.cpp): the expected windows, section
counts and orders below are the reference tests' known answers.  The one
reference test not restated here, crop_helpers_copy_the_requested_region, checks
CLI-internal crop helpers; their counterparts in host/main.cpp are exercised by
the GPU test of --tile (tests/test_gpu_cli.py), which compares the pasted window
with the oracle pixel by pixel (within one level).
"""

import numpy as np
import pytest

from lama_b200.engine import mask_depth, section_rects, tile_rect, window_origin

TILE_MIN, SECTION_BLOCK, PAD_MOD = 512, 256, 8
UMAX = np.iinfo(np.uint32).max


def mask_of(w, h, rect=None):
    """main.rs:805-815: inclusive rectangle (x0, y0, x1, y1)."""
    m = np.zeros((h, w), np.uint8)
    if rect is not None:
        x0, y0, x1, y1 = rect
        m[y0:y1 + 1, x0:x1 + 1] = 255
    return m


def assert_contains(t, m):
    x0, y0, side = t[:3]
    ys, xs = np.nonzero(m)
    assert (xs >= x0).all() and (xs < x0 + side).all() and (ys >= y0).all() and (ys < y0 + side).all()
    assert x0 + side <= m.shape[1] and y0 + side <= m.shape[0]
    if min(m.shape) >= PAD_MOD:
        assert side % PAD_MOD == 0


def test_empty_mask_has_no_window():
    assert tile_rect(mask_of(256, 256)) is None


def test_small_mask_gets_the_minimum_window():
    m = mask_of(1024, 1024, (500, 500, 515, 515))
    t = tile_rect(m)
    assert t[2] == TILE_MIN
    assert_contains(t, m)


def test_window_is_twice_the_bounding_box():
    m = mask_of(2048, 2048, (900, 800, 1199, 1099))
    t = tile_rect(m)
    assert t[2] == 600
    assert_contains(t, m)


def test_wider_than_tall_uses_the_longer_side():
    m = mask_of(2048, 2048, (100, 1000, 799, 1099))
    t = tile_rect(m)
    assert t[2] == 1400
    assert_contains(t, m)


@pytest.mark.parametrize("x0,y0", [(0, 0), (824, 0), (0, 824), (824, 924)])
def test_window_stays_inside_the_image_at_every_corner(x0, y0):
    m = mask_of(1024, 1024, (x0, y0, x0 + 199, y0 + 99))
    assert_contains(tile_rect(m), m)


def test_window_is_capped_at_the_image_size():
    t = tile_rect(mask_of(300, 500, (0, 0, 299, 499)))
    assert t[2] == 296
    assert (t[0], t[1]) == (2, 102)


def test_oversized_bounding_box_is_clamped_not_clipped():
    m = mask_of(2048, 2048, (1700, 1700, 1999, 1999))
    t = tile_rect(m)
    assert t[2] == 600 and (t[0], t[1]) == (1448, 1448)
    assert_contains(t, m)


@pytest.mark.parametrize("side", range(1, 9))
def test_tiny_images_do_not_fail(side):
    t = tile_rect(mask_of(side, side, (0, 0, side - 1, side - 1)))
    assert 1 <= t[2] <= side
    assert t[0] + t[2] <= side and t[1] + t[2] <= side


def assert_covers(sections, m):
    hits = np.zeros(m.shape, np.int32)
    for x0, y0, x1, y1 in sections:
        sub = m[y0:y1, x0:x1] > 0
        assert sub.any(), "empty section"
        assert x1 - x0 <= SECTION_BLOCK and y1 - y0 <= SECTION_BLOCK
        hits[y0:y1, x0:x1] += sub
    np.testing.assert_array_equal(hits, (m > 0).astype(np.int32))


def section_depth(s, m, depth):
    x0, y0, x1, y1 = s
    sub = m[y0:y1, x0:x1] > 0
    return depth[y0:y1, x0:x1][sub].min()


def test_sections_of_a_small_mask_are_single_and_cover_it():
    m = mask_of(1024, 1024, (500, 500, 700, 700))
    s = section_rects(m)
    assert s == [(500, 500, 701, 701)]
    assert_covers(s, m)


def test_a_300x300_mask_becomes_four_sections():
    m = mask_of(1024, 1024, (300, 300, 598, 598))
    s = section_rects(m)
    assert len(s) == 4
    assert_covers(s, m)
    for i, a in enumerate(s):
        for b in s[i + 1:]:
            assert a[2] <= b[0] or b[2] <= a[0] or a[3] <= b[1] or b[3] <= a[1]
    assert (s[0][0], s[0][2], s[2][0], s[2][2]) == (300, 556, 300, 556)


def test_the_rim_is_filled_before_the_interior():
    m = mask_of(2048, 2048, (500, 500, 1099, 1099))
    s = section_rects(m)
    assert_covers(s, m)
    d = mask_depth(m)
    assert section_depth(s[0], m, d) == 0
    assert section_depth(s[-1], m, d) > 0
    ds = [section_depth(x, m, d) for x in s]
    assert ds == sorted(ds)


def test_mask_depth_is_zero_on_the_rim_and_grows_inward():
    m = mask_of(512, 512, (100, 100, 299, 299))
    d = mask_depth(m)
    assert d[100, 100] == 0 and d[299, 299] == 0
    assert d[200, 200] >= 99
    assert d[0, 0] == UMAX


def test_order_is_deterministic():
    a = mask_of(2048, 2048, (100, 100, 699, 399))
    b = mask_of(2048, 2048, (100, 100, 699, 399))
    assert section_rects(a) == section_rects(b) and section_rects(a)


def test_a_wide_mask_is_sectioned_and_ordered_by_depth():
    m = mask_of(2048, 2048, (100, 100, 699, 399))
    s = section_rects(m)
    assert len(s) == 6
    assert_covers(s, m)
    d = mask_depth(m)
    ds = [section_depth(x, m, d) for x in s]
    assert ds == sorted(ds)


def test_empty_mask_has_no_sections():
    assert section_rects(mask_of(256, 256)) == []


def test_a_single_pixel_mask_is_one_small_piece():
    m = mask_of(1024, 1024, (800, 900, 800, 900))
    assert section_rects(m) == [(800, 900, 801, 901)]


def test_passes_fill_the_hole_monotonically_and_completely():
    m = mask_of(1024, 1024, (300, 300, 598, 598))
    s = section_rects(m)
    filled = np.zeros(m.shape, bool)
    total = int((m > 0).sum())
    remaining, seen = total, []
    for x0, y0, x1, y1 in s:
        new = (m[y0:y1, x0:x1] > 0) & ~filled[y0:y1, x0:x1]
        remaining -= int(new.sum())
        filled[y0:y1, x0:x1] |= m[y0:y1, x0:x1] > 0
        seen.append(remaining)
    assert remaining == 0 and seen[0] < total and seen == sorted(seen, reverse=True)
    d = mask_depth(m)
    x0, y0, x1, y1 = s[0]
    assert ((m[y0:y1, x0:x1] > 0) & (d[y0:y1, x0:x1] == 0)).any()


def test_window_origin_stays_inside():
    assert window_origin(0, 512, 1024) == 0
    assert window_origin(1023, 512, 1024) == 512
    assert window_origin(500, 512, 1024) == 244
    assert window_origin(600, 512, 300) == 0
    assert window_origin(0, 4096, 1024) == 0


def test_every_section_fits_in_a_512_window_inside_a_large_image():
    m = mask_of(1024, 1024, (0, 0, 1023, 1023))
    for x0, y0, x1, y1 in section_rects(m):
        wx = window_origin((x0 + x1) // 2, TILE_MIN, 1024)
        wy = window_origin((y0 + y1) // 2, TILE_MIN, 1024)
        assert wx <= x0 and x1 <= wx + TILE_MIN
        assert wy <= y0 and y1 <= wy + TILE_MIN
