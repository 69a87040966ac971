"""The big-lama generator topology and its checkpoint tensor names.

Mirrors the reference plan `model::build` / `model::ffc`
(lama-rs/src/model.rs:135-257) and the parameter names its loaders read
(lama-rs/src/cpu.rs:561-616, lama-rs/src/cuda.rs:832-962).  The tensor list is
in `state_dict` order, which is the order the reference's exporter writes
(lama-rs/export_weights.py:34-45): module registration order of the upstream
LaMa `FFCResNetGenerator`.

Counts: 229 convolution tensors + 152 BatchNorms x 5 = 989 tensors.
"""

from __future__ import annotations

from dataclasses import dataclass, field

FFC_RESNET_RATIO = 0.75
N_RESBLOCKS = 18
FIRST_RES = 5          # model.5 .. model.22
CONCAT = 23
UPSAMPLES = ((24, 25, 512, 256), (27, 28, 256, 128), (30, 31, 128, 64))
OUTCONV = 34


@dataclass
class Ffc:
    """One FFC_BN_ACT, with the branch split derived as `model::ffc` does."""
    index: int
    sub: int
    cin: int
    cout: int
    kernel: int
    stride: int
    ratio_gin: float
    ratio_gout: float
    pad: int = field(init=False)
    in_global: int = field(init=False)
    out_global: int = field(init=False)
    in_local: int = field(init=False)
    out_local: int = field(init=False)

    def __post_init__(self):
        # model.rs:222-225: int(c * ratio) truncation, as `as usize` does.
        self.in_global = int(float(self.cin) * self.ratio_gin)
        self.out_global = int(float(self.cout) * self.ratio_gout)
        self.in_local = self.cin - self.in_global
        self.out_local = self.cout - self.out_global
        self.pad = self.kernel // 2

    @property
    def ffc_prefix(self) -> str:
        return {0: f"model.{self.index}.ffc", 1: f"model.{self.index}.conv1.ffc"}.get(
            self.sub, f"model.{self.index}.conv2.ffc")

    @property
    def partial(self) -> str:
        return {0: f"model.{self.index}", 1: f"model.{self.index}.conv1"}.get(
            self.sub, f"model.{self.index}.conv2")

    @property
    def has_l2l(self): return self.in_local > 0 and self.out_local > 0
    @property
    def has_l2g(self): return self.in_local > 0 and self.out_global > 0
    @property
    def has_g2l(self): return self.in_global > 0 and self.out_local > 0
    @property
    def has_g2g(self): return self.in_global > 0 and self.out_global > 0


def encoder() -> list[Ffc]:
    """model.1 .. model.4 (model.rs:141-160).  model.1 is a valid 7x7 (pad 0)."""
    m1 = Ffc(1, 0, 4, 64, 7, 1, 0.0, 0.0)
    m1.pad = 0
    return [m1,
            Ffc(2, 0, 64, 128, 3, 2, 0.0, 0.0),
            Ffc(3, 0, 128, 256, 3, 2, 0.0, 0.0),
            Ffc(4, 0, 256, 512, 3, 2, 0.0, FFC_RESNET_RATIO)]


def resblocks() -> list[tuple[Ffc, Ffc]]:
    """model.5 .. model.22, each two FFC 512->512 (model.rs:162-172)."""
    out = []
    for i in range(FIRST_RES, FIRST_RES + N_RESBLOCKS):
        out.append((Ffc(i, 1, 512, 512, 3, 1, FFC_RESNET_RATIO, FFC_RESNET_RATIO),
                    Ffc(i, 2, 512, 512, 3, 1, FFC_RESNET_RATIO, FFC_RESNET_RATIO)))
    return out


def _bn(prefix: str, c: int) -> list[tuple[str, tuple]]:
    return [(f"{prefix}.weight", (c,)), (f"{prefix}.bias", (c,)),
            (f"{prefix}.running_mean", (c,)), (f"{prefix}.running_var", (c,)),
            (f"{prefix}.num_batches_tracked", ())]


def _ffc_tensors(b: Ffc) -> list[tuple[str, tuple]]:
    p, k = b.ffc_prefix, b.kernel
    t: list[tuple[str, tuple]] = []
    if b.has_l2l:
        t.append((f"{p}.convl2l.weight", (b.out_local, b.in_local, k, k)))
    if b.has_l2g:
        t.append((f"{p}.convl2g.weight", (b.out_global, b.in_local, k, k)))
    if b.has_g2l:
        t.append((f"{p}.convg2l.weight", (b.out_local, b.in_global, k, k)))
    if b.has_g2g:
        half = b.out_global // 2
        g = f"{p}.convg2g"
        t.append((f"{g}.conv1.0.weight", (half, b.in_global, 1, 1)))
        t += _bn(f"{g}.conv1.1", half)
        t.append((f"{g}.fu.conv_layer.weight", (2 * half, 2 * half, 1, 1)))
        t += _bn(f"{g}.fu.bn", 2 * half)
        t.append((f"{g}.conv2.weight", (b.out_global, half, 1, 1)))
    if b.out_local > 0:
        t += _bn(f"{b.partial}.bn_l", b.out_local)
    if b.out_global > 0:
        t += _bn(f"{b.partial}.bn_g", b.out_global)
    return t


def tensor_list() -> list[tuple[str, tuple]]:
    """All 989 checkpoint tensors `(name, shape)` in state_dict order."""
    t: list[tuple[str, tuple]] = []
    for b in encoder():
        t += _ffc_tensors(b)
    for c1, c2 in resblocks():
        t += _ffc_tensors(c1)
        t += _ffc_tensors(c2)
    for idx, bn_idx, cin, cout in UPSAMPLES:
        t.append((f"model.{idx}.weight", (cin, cout, 3, 3)))
        t.append((f"model.{idx}.bias", (cout,)))
        t += _bn(f"model.{bn_idx}", cout)
    t.append((f"model.{OUTCONV}.weight", (3, 64, 7, 7)))
    t.append((f"model.{OUTCONV}.bias", (3,)))
    return t


def algorithmic_flops(h: int, w: int) -> dict[str, float]:
    """FLOPs of one h x w pass (h, w multiples of 8), 2 x MAC over real taps only:
    no im2col, padding or transposed-conv zero taps.  Keys: encoder, ffc (the 36
    FFC layers' 3x3 branches), spectral (their 1x1 convs and FourierUnit convs),
    decoder (the three ConvTranspose2d), outconv, total."""
    h8, w8 = h // 8, w // 8
    f = {}
    enc = 0
    ho, wo = h, w  # model.1 is a valid 7x7 over the pad-3 input: output h x w
    for b in encoder():
        ho, wo = ho // b.stride, wo // b.stride
        enc += ho * wo * b.cout * b.cin * b.kernel * b.kernel
    f["encoder"] = 2.0 * enc
    ffc = spec = 0
    for pair in resblocks():
        for b in pair:
            taps = b.kernel * b.kernel
            ffc += h8 * w8 * taps * (b.out_local * b.in_local + b.out_global * b.in_local + b.out_local * b.in_global)
            half = b.out_global // 2
            spec += h8 * w8 * (half * b.in_global + b.out_global * half)       # conv1, conv2
            spec += h8 * (w8 // 2 + 1) * (2 * half) * (2 * half)                # FourierUnit 1x1
    f["ffc"] = 2.0 * ffc
    f["spectral"] = 2.0 * spec
    dec = 0
    hin, win = h8, w8
    for _, _, cin, cout in UPSAMPLES:
        dec += cin * cout * 9 * hin * win
        hin, win = 2 * hin, 2 * win
    f["decoder"] = 2.0 * dec
    f["outconv"] = 2.0 * h * w * 3 * 64 * 49
    f["total"] = f["encoder"] + f["ffc"] + f["spectral"] + f["decoder"] + f["outconv"]
    return f
