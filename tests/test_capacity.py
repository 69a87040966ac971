"""Capacity guard refit (lama-rs/src/mem.rs:13-73).

The reference estimates a pass's device memory from a line fitted to GTX 1080
measurements (1170 B/px + 343 MiB, mem.rs:13-36) and refuses a forced GPU run
that will not fit, keeping 10 % of free memory as headroom (mem.rs:49-73).
This engine's estimate is the plan's exact footprint: `lama_estimate_bytes`
builds the pass's plan without allocating (no GPU, no weight file) and sums
what it would allocate.  The CPU tests pin that sum against the activation
layout restated here and check the properties the reference's own tests check
(monotone, a 512x512 pass small, the per-pixel slope); the GPU tests check it
against the bytes the engine's real plan holds and that an oversized pass is
refused before anything is allocated.
"""

import numpy as np
import pytest

from lama_b200 import engine as E


def layout_bytes(b, h, w):
    """Device buffers of one u8 inpaint pass as the engine lays them out:
    split-bf16 NHWC activations ([2][B][H+2halo][W+2halo][C] x 2 bytes), the
    spectral intermediates of 64x64-and-smaller power-of-two latents (register
    and prefetching transforms: no two-pass intermediate), u8 staging.
    Split-K workspaces (small batches only) are not included."""
    H, W = -(-h // 8) * 8, -(-w // 8) * 8

    def act(bb, hh, ww, c, halo):
        return 2 * 2 * bb * (hh + 2 * halo) * (ww + 2 * halo) * c

    h8, w8 = H // 8, W // 8
    wh = w8 // 2 + 1
    n = act(b, H + 6, W, 32, 0)                       # reflect-padded, x-tap-packed input
    n += b * h * w * 3 + b * h * w + b * h * w * 3    # rgb, mask, composited output
    n += act(b, H, W, 64, 1) + act(b, H // 2, W // 2, 128, 1) + act(b, H // 4, W // 4, 256, 1)
    n += 2 * act(b, h8, w8, 512, 1)                   # the resblock state, ping-pong
    n += b * h8 * w8 * 192 * 4                        # feat (fp32)
    n += act(b, 1, h8 * wh, 384, 0)                   # spectrum (split bf16)
    n += b * h8 * wh * 384 * 4                        # FourierUnit conv output (fp32)
    n += act(b, h8, w8, 192, 0)                       # S = feat + irfft2
    n += (h8 + w8) * 8                                # twiddle tables
    n += act(b, 2 * h8, 2 * w8, 256, 0) + act(b, 4 * h8, 4 * w8, 128, 0) + act(b, H, W, 64, 3)
    return n


@pytest.mark.parametrize("b,h,w", [(64, 512, 512), (16, 512, 512), (256, 512, 512), (8, 256, 512)])
def test_estimate_is_the_activation_layout_at_throughput_batches(b, h, w):
    """The layout plus the static tile schedules (one int per tile of the
    launches that have one: under 0.1 % of the activations)."""
    base = layout_bytes(b, h, w)
    extra = E.estimate_bytes(b, h, w) - base
    assert 0 <= extra < 1e-3 * base, extra


def test_small_batches_add_split_k_workspaces_only():
    """Batch-1 passes split the K loop of their GEMMs; the workspaces come on
    top of the layout and stay a fraction of it."""
    got, base = E.estimate_bytes(1, 512, 512), layout_bytes(1, 512, 512)
    assert base < got < 2 * base


def test_estimate_grows_with_area_and_batch():
    last = 0
    for side in (8, 64, 512, 1024, 2048, 4096):
        v = E.estimate_bytes(1, side, side)
        assert v > last
        last = v
    assert E.estimate_bytes(2, 512, 512) > E.estimate_bytes(1, 512, 512)


def test_per_pixel_slope_and_the_passes_the_guard_turns_on():
    """About 1.16 KB per input pixel at large sizes (the reference's GTX 1080
    fit is 1170 B/px for its own engine); a 512x512 pass is well under 1 GB,
    a 2048x2048 whole-image pass about 5 GB and a 16384x16384 pass beyond a
    B200's 180 GB, which the guard therefore refuses."""
    for side in (2048, 4096):
        slope = E.estimate_bytes(1, side, side) / side ** 2
        assert 1100 < slope < 1250, (side, slope)
    assert E.estimate_bytes(1, 512, 512) < 1 << 30
    assert 4 << 30 < E.estimate_bytes(1, 2048, 2048) < 6 << 30
    assert E.estimate_bytes(1, 16384, 16384) > 180 * 10 ** 9


def test_padding_to_multiples_of_eight():
    assert E.estimate_bytes(1, 600, 600) > 0
    assert E.estimate_bytes(1, 61, 77) >= E.estimate_bytes(1, 56, 72)


@pytest.mark.parametrize("b,h,w", [(0, 512, 512), (1, 0, 512), (1, 512, -8)])
def test_non_positive_sizes_are_refused(b, h, w):
    with pytest.raises(E.LamaError) as ei:
        E.estimate_bytes(b, h, w)
    assert ei.value.code == -1


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,w", [(1, 512, 512), (3, 64, 96), (1, 600, 600), (2, 1024, 1024), (16, 512, 512),
                                   (1, 61, 77)])
def test_estimate_equals_the_bytes_the_real_plan_holds(engine_tamed, b, h, w):
    assert engine_tamed.plan_bytes(b, h, w) == E.estimate_bytes(b, h, w)


@pytest.mark.gpu
def test_a_pass_beyond_the_device_is_refused_before_allocating(engine_tamed):
    """~600 images of 512x512 need ~183 GB: refused with the needed and free
    amounts, and nothing is allocated (free memory unchanged)."""
    import torch
    b = 600
    assert E.estimate_bytes(b, 512, 512) > 180 * 10 ** 9
    d = torch.zeros((b, 512, 512, 3), dtype=torch.uint8, device="cuda")
    m = torch.zeros((b, 512, 512), dtype=torch.uint8, device="cuda")
    o = torch.empty_like(d)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    with pytest.raises(E.LamaError) as ei:
        engine_tamed.inpaint_u8_device(d.data_ptr(), m.data_ptr(), o.data_ptr(), b, 512, 512)
    assert ei.value.code == -5
    assert "needs about" in ei.value.msg and "is free of" in ei.value.msg
    assert torch.cuda.mem_get_info()[0] == free0
