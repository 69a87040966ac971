"""Algorithmic work of a pass, from the topology mirror (lama_b200/plan.py).

The counts are 2 x MAC over real taps only (no im2col, padding or transposed-conv
zero taps), the figures the bench's roofline divides by time.  They are checked
against an independent count of the same topology (lama-rs/src/model.rs:135-257):
439.8 GFLOP per 512^2 pass, 370.3 for the 18-block stack at a 64^2 latent, 603.5
for a 600^2 tile window, ~1758 at 1024^2 and 7028.8 at 2048^2.
"""

import pytest

from lama_b200 import plan


@pytest.mark.parametrize("side,gflop", [(512, 439.8), (600, 603.5), (1024, 1758.0), (2048, 7028.8)])
def test_pass_flops_match_the_independent_count(side, gflop):
    got = plan.algorithmic_flops(side, side)["total"] / 1e9
    assert abs(got - gflop) <= 0.1 + 1e-4 * gflop, got


def test_resblock_stack_flops():
    f = plan.algorithmic_flops(512, 512)
    assert abs((f["ffc"] + f["spectral"]) / 1e9 - 370.3) < 0.05


def test_flops_by_part_at_512():
    """Shares by part: resblock 3x3 convs 69 %, spectral 1x1 15 %, encoder 8 %,
    decoder 7 %, OutConv 1 %."""
    f = plan.algorithmic_flops(512, 512)
    share = {k: v / f["total"] for k, v in f.items() if k != "total"}
    assert abs(share["ffc"] - 0.692) < 0.002
    assert abs(share["spectral"] - 0.150) < 0.002
    assert abs(share["encoder"] - 0.081) < 0.002
    assert abs(share["decoder"] - 0.066) < 0.002
    assert abs(share["outconv"] - 0.011) < 0.001
    # one FFC layer's 3x3 branches: 2 x 4096 x 9 x (128*128 + 384*128 + 128*384)
    assert f["ffc"] / 36 == 2 * 4096 * 9 * (128 * 128 + 384 * 128 + 128 * 384)


def test_flops_grow_with_area():
    a = plan.algorithmic_flops(256, 256)["total"]
    b = plan.algorithmic_flops(512, 512)["total"]
    assert 3.9 < b / a < 4.1
