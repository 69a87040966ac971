"""Independent PyTorch-CPU restatement of the big-lama generator forward.

TEST INFRASTRUCTURE ONLY: a second checker next to the C++ restatement of the
reference CPU engine (oracle/lama_oracle.cpp).  It is written with PyTorch's
own operators - `F.conv2d` on reflect-padded input, `F.conv_transpose2d`,
`torch.fft.rfftn/irfftn(norm='ortho')` - i.e. the upstream LaMa semantics the
reference claims parity with (README.md:28-29), not the reference's loops.

Topology: lama-rs/src/model.rs:135-207.  FFC: lama-rs/src/cpu.rs:635-688.
SpectralTransform / FourierUnit: lama-rs/src/cpu.rs:239-308.  ConvT + BN + ReLU:
lama-rs/src/cpu.rs:524-530.  OutConv + sigmoid: lama-rs/src/cpu.rs:531-534.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "lama-inpaint-rs_b200"))
from lama_b200 import plan  # noqa: E402


def _fft1(a, inverse: bool, dim: int, reference_semantics: bool):
    """Unnormalised 1-D complex DFT along `dim`.

    With `reference_semantics`, a length that is not a power of two runs the
    opposite direction, as the reference CPU engine's Bluestein path does
    (lama-rs/src/cpu.rs:984-1011 builds a_j = x_j*conj(w_j) and b = w, the
    conjugate of the chirp pair of the transform it is asked for, so
    `inverse=false` yields sum_j x_j exp(+2 pi i jk/n)).  Power-of-two lengths
    use radix-2 (cpu.rs:888-927) and agree with torch.fft.
    """
    n = a.shape[dim]
    forward = not inverse
    if reference_semantics and (n & (n - 1)) != 0:
        forward = not forward
    return torch.fft.fft(a, dim=dim) if forward else torch.fft.ifft(a, dim=dim) * n


def rfft2_ortho(x, reference_semantics=True):
    """[..., h, w] real -> [..., h, w//2+1] complex, norm='ortho'."""
    h, w = x.shape[-2:]
    f = _fft1(_fft1(x.to(torch.complex128), False, -1, reference_semantics), False, -2, reference_semantics)
    return f[..., : w // 2 + 1] / np.sqrt(h * w)


def irfft2_ortho(X, h, w, reference_semantics=True):
    """Inverse of the above with the 2-D Hermitian completion of cpu.rs:801-837."""
    hw = w // 2 + 1
    F = torch.zeros(X.shape[:-2] + (h, w), dtype=torch.complex128)
    F[..., :hw] = X
    if w - hw > 0:
        xs = torch.arange(hw, w)
        xm = w - xs
        keep = xm < hw
        xs, xm = xs[keep], xm[keep]
        ym = (h - torch.arange(h)) % h
        F[..., :, xs] = torch.conj(X[..., ym, :][..., :, xm])
    r = _fft1(_fft1(F, True, -1, reference_semantics), True, -2, reference_semantics)
    return (r.real / np.sqrt(h * w))


class TorchRef:
    """`reference_semantics=True` reproduces the reference's FFT direction for
    non-power-of-two planes; False gives upstream torch.fft semantics."""

    def __init__(self, tensors: dict[str, np.ndarray], dtype=torch.float64, reference_semantics=True):
        self.dtype = dtype
        self.refsem = reference_semantics
        self.t = {k: torch.from_numpy(np.asarray(v)).to(dtype) for k, v in tensors.items()}

    def bn(self, x, prefix, relu=True):
        w, b = self.t[prefix + ".weight"], self.t[prefix + ".bias"]
        m, v = self.t[prefix + ".running_mean"], self.t[prefix + ".running_var"]
        s = w / torch.sqrt(v + 1e-5)
        y = x * s[None, :, None, None] + (b - m * s)[None, :, None, None]
        return F.relu(y) if relu else y

    def conv(self, x, name, pad, stride):
        w = self.t[name]
        if pad:
            x = F.pad(x, (pad, pad, pad, pad), mode="reflect")
        return F.conv2d(x, w, stride=stride)

    def spectral(self, x, p):
        f = self.bn(F.conv2d(x, self.t[p + ".conv1.0.weight"]), p + ".conv1.1")
        n, c, h, w = f.shape
        sp = rfft2_ortho(f, self.refsem)
        st = torch.stack((sp.real.to(self.dtype), sp.imag.to(self.dtype)), dim=-1).permute(0, 1, 4, 2, 3).reshape(n, 2 * c, h, w // 2 + 1)
        y = self.bn(F.conv2d(st, self.t[p + ".fu.conv_layer.weight"]), p + ".fu.bn")
        y = y.reshape(n, c, 2, h, w // 2 + 1).permute(0, 1, 3, 4, 2)
        y = torch.complex(y[..., 0].contiguous(), y[..., 1].contiguous())
        fu = irfft2_ortho(y.to(torch.complex128), h, w, self.refsem).to(self.dtype)
        return F.conv2d(f + fu, self.t[p + ".conv2.weight"])

    def ffc(self, b: plan.Ffc, xl, xg):
        p = b.ffc_prefix
        ol = og = None
        if b.out_local > 0:
            ol = 0
            if b.has_l2l:
                ol = ol + self.conv(xl, p + ".convl2l.weight", b.pad, b.stride)
            if b.has_g2l:
                ol = ol + self.conv(xg, p + ".convg2l.weight", b.pad, b.stride)
            ol = self.bn(ol, b.partial + ".bn_l")
        if b.out_global > 0:
            og = 0
            if b.has_l2g:
                og = og + self.conv(xl, p + ".convl2g.weight", b.pad, b.stride)
            if b.has_g2g:
                og = og + self.spectral(xg, p + ".convg2g")
            og = self.bn(og, b.partial + ".bn_g")
        return ol, og

    def encode(self, x):
        """model.0..model.4: returns (local [N,128,h/8,w/8], global [N,384,...])."""
        x = F.pad(x, (3, 3, 3, 3), mode="reflect")
        xl, xg = x, None
        for b in plan.encoder():
            xl, xg = self.ffc(b, xl, xg)
        return xl, xg

    def resblocks(self, xl, xg, blocks=None):
        for i, (c1, c2) in enumerate(plan.resblocks()):
            if blocks is not None and i >= blocks:
                break
            l1, g1 = self.ffc(c1, xl, xg)
            l2, g2 = self.ffc(c2, l1, g1)
            xl, xg = xl + l2, xg + g2
        return xl, xg

    def decode(self, xl, xg, presigmoid=False):
        x = torch.cat([xl, xg], dim=1)
        for idx, bn_idx, _, _ in plan.UPSAMPLES:
            x = F.conv_transpose2d(x, self.t[f"model.{idx}.weight"], self.t[f"model.{idx}.bias"],
                                   stride=2, padding=1, output_padding=1)
            x = self.bn(x, f"model.{bn_idx}")
        x = F.pad(x, (3, 3, 3, 3), mode="reflect")
        y = F.conv2d(x, self.t[f"model.{plan.OUTCONV}.weight"], self.t[f"model.{plan.OUTCONV}.bias"])
        return y if presigmoid else torch.sigmoid(y)

    @torch.no_grad()
    def forward(self, x: np.ndarray, presigmoid=False) -> np.ndarray:
        xt = torch.from_numpy(np.asarray(x)).to(self.dtype)
        if xt.dim() == 3:
            xt = xt[None]
        xl, xg = self.encode(xt)
        xl, xg = self.resblocks(xl, xg)
        return self.decode(xl, xg, presigmoid).numpy()
