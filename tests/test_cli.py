"""The C++ CLI (lama-inpaint-rs_b200/lama-inpaint): argument contract and PNG codec.

Usage errors exit 2 and run errors exit 1 (lama-rs/src/main.rs:198-210); the
PNG reader accepts what the reference's reader accepts (lama-rs/src/image.rs:80-130),
checked against PIL.  End-to-end inpainting through the CLI is a GPU test.
"""

import os
import subprocess

import numpy as np
import pytest
from PIL import Image

from lama_b200.engine import CLI_PATH

pytestmark = pytest.mark.skipif(not os.path.exists(CLI_PATH), reason="CLI not built")


def run(*args, **kw):
    return subprocess.run([CLI_PATH, *args], capture_output=True, text=True, **kw)


def test_help_exits_zero():
    r = run("--help")
    assert r.returncode == 0 and "--tile" in r.stdout and "--sections" in r.stdout


@pytest.mark.parametrize("args,msg", [
    ([], "--image is required"),
    (["--image", "a.png"], "--mask is required"),
    (["--image", "a.png", "--mask", "b.png"], "--output is required"),
    (["--image", "-", "--mask", "-", "--output", "o.png"], "cannot both be '-'"),
    (["--image", "a", "--mask", "b", "--output", "o", "--tile", "--sections"], "mutually exclusive"),
    (["--bogus"], "unknown argument --bogus"),
    (["--image"], "--image needs a value"),
])
def test_usage_errors_exit_2(args, msg):
    r = run(*args)
    assert r.returncode == 2 and msg in r.stderr


def test_size_mismatch_is_a_run_error(tmp_path):
    Image.fromarray(np.zeros((8, 8, 3), np.uint8)).save(tmp_path / "a.png")
    Image.fromarray(np.zeros((8, 9), np.uint8)).save(tmp_path / "m.png")
    r = run("--image", str(tmp_path / "a.png"), "--mask", str(tmp_path / "m.png"), "--output", str(tmp_path / "o.png"))
    assert r.returncode == 1 and "mask is 9x8 but image is 8x8" in r.stderr


def test_cpu_flag_is_refused(tmp_path):
    Image.fromarray(np.zeros((8, 8, 3), np.uint8)).save(tmp_path / "a.png")
    Image.fromarray(np.zeros((8, 8), np.uint8)).save(tmp_path / "m.png")
    r = run("--image", str(tmp_path / "a.png"), "--mask", str(tmp_path / "m.png"), "--output",
            str(tmp_path / "o.png"), "--cpu")
    assert r.returncode == 1 and "no CPU engine" in r.stderr


def _rgb_expected(im: Image.Image) -> np.ndarray:
    """What image.rs:80-120 produces: RGB8 (16-bit high byte, alpha dropped)."""
    if im.mode == "P":
        return np.asarray(im.convert("RGB"))
    if im.mode in ("I;16", "I;16B", "I"):
        a = np.asarray(im).astype(np.uint32) >> 8
        return np.repeat(a.astype(np.uint8)[..., None], 3, axis=2)
    return np.asarray(im.convert("RGB"))


@pytest.mark.parametrize("mode", ["RGB", "RGBA", "L", "LA", "P", "I;16"])
@pytest.mark.parametrize("interlace", [False, True])
def test_png_decode_matches_pil(tmp_path, mode, interlace):
    rng = np.random.default_rng(3)
    h, w = 37, 53
    if mode == "I;16":
        im = Image.fromarray(rng.integers(0, 65535, (h, w), dtype=np.uint16))
    else:
        im = Image.fromarray(rng.integers(0, 255, (h, w, 3), dtype=np.uint8)).convert(mode)
    src = tmp_path / "in.png"
    im.save(src, interlace=interlace) if not interlace else im.save(src, optimize=False, interlace=1)
    dst = tmp_path / "out.png"
    r = run("--decode-png", str(src), str(dst))
    assert r.returncode == 0, r.stderr
    got = np.asarray(Image.open(dst))
    np.testing.assert_array_equal(got, _rgb_expected(Image.open(src)))


def test_png_rejects_garbage(tmp_path):
    p = tmp_path / "bad.png"
    p.write_bytes(b"not a png at all")
    r = run("--decode-png", str(p), str(tmp_path / "o.png"))
    assert r.returncode == 1 and "not a PNG" in r.stderr


def test_png_rejects_low_bit_depth(tmp_path):
    Image.fromarray(np.zeros((4, 4), bool)).save(tmp_path / "b.png")  # 1-bit
    r = run("--decode-png", str(tmp_path / "b.png"), str(tmp_path / "o.png"))
    assert r.returncode == 1 and "bit depth" in r.stderr


def _rechunk_idat(png: bytes, piece: int, cut: int = 0) -> bytes:
    """The same PNG with its compressed stream split into IDAT chunks of `piece`
    bytes (less its last `cut` bytes), CRCs recomputed."""
    import struct
    import zlib

    pos, head, stream, tail = 8, [png[:8]], b"", []
    while pos < len(png):
        n = struct.unpack(">I", png[pos:pos + 4])[0]
        kind, data = png[pos + 4:pos + 8], png[pos + 8:pos + 8 + n]
        pos += 12 + n
        if kind == b"IDAT":
            stream += data
        else:
            (tail if stream else head).append(png[pos - 12 - n:pos])
    stream = stream[:len(stream) - cut]
    chunks = [stream[i:i + piece] for i in range(0, len(stream), piece)]
    body = b"".join(struct.pack(">I", len(c)) + b"IDAT" + c + struct.pack(">I", zlib.crc32(b"IDAT" + c))
                    for c in chunks)
    return b"".join(head) + body + b"".join(tail)


def test_png_stream_split_over_many_idat_chunks(tmp_path):
    rng = np.random.default_rng(4)
    im = Image.fromarray(rng.integers(0, 255, (29, 41, 3), dtype=np.uint8))
    src = tmp_path / "in.png"
    im.save(src)
    split = tmp_path / "split.png"
    split.write_bytes(_rechunk_idat(src.read_bytes(), 97))
    r = run("--decode-png", str(split), str(tmp_path / "o.png"))
    assert r.returncode == 0, r.stderr
    np.testing.assert_array_equal(np.asarray(Image.open(tmp_path / "o.png")), np.asarray(im))


def test_png_truncated_stream_is_a_run_error(tmp_path):
    rng = np.random.default_rng(5)
    im = Image.fromarray(rng.integers(0, 255, (29, 41, 3), dtype=np.uint8))
    src = tmp_path / "in.png"
    im.save(src)
    bad = tmp_path / "cut.png"
    bad.write_bytes(_rechunk_idat(src.read_bytes(), 1 << 20, cut=200))
    r = run("--decode-png", str(bad), str(tmp_path / "o.png"))
    assert r.returncode == 1 and "corrupt image data" in r.stderr


def test_png_writer_splits_a_large_stream_into_idat_chunks(tmp_path):
    """Noise does not compress: a 700x700 image leaves more than one 1 MiB IDAT chunk."""
    rng = np.random.default_rng(6)
    im = Image.fromarray(rng.integers(0, 255, (700, 700, 3), dtype=np.uint8))
    src, dst = tmp_path / "in.png", tmp_path / "out.png"
    im.save(src)
    r = run("--decode-png", str(src), str(dst))
    assert r.returncode == 0, r.stderr
    assert dst.read_bytes().count(b"IDAT") >= 2
    np.testing.assert_array_equal(np.asarray(Image.open(dst)), np.asarray(im))


def _png16(samples: np.ndarray, ctype: int) -> bytes:
    """A 16-bit PNG written by hand: samples [h, w, channels] uint16, filter 0."""
    import struct
    import zlib

    h, w, _ = samples.shape
    rows = b"".join(b"\0" + samples[y].astype(">u2").tobytes() for y in range(h))

    def chunk(kind, data):
        return struct.pack(">I", len(data)) + kind + data + struct.pack(">I", zlib.crc32(kind + data))

    ihdr = struct.pack(">IIBBBBB", w, h, 16, ctype, 0, 0, 0)
    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", zlib.compress(rows)) +
            chunk(b"IEND", b""))


@pytest.mark.parametrize("ctype,channels", [(2, 3), (6, 4), (4, 2)])
def test_sixteen_bit_colour_keeps_the_high_byte(tmp_path, ctype, channels):
    """image.rs:80-120 reads 16-bit samples through their high byte; grey (and
    grey+alpha) spreads to all three channels, alpha is dropped."""
    rng = np.random.default_rng(7 + ctype)
    s = rng.integers(0, 65536, (13, 17, channels), dtype=np.uint16)
    src = tmp_path / "in16.png"
    src.write_bytes(_png16(s, ctype))
    r = run("--decode-png", str(src), str(tmp_path / "o.png"))
    assert r.returncode == 0, r.stderr
    hi = (s >> 8).astype(np.uint8)
    exp = hi[..., :3] if channels >= 3 else np.repeat(hi[..., :1], 3, axis=2)
    np.testing.assert_array_equal(np.asarray(Image.open(tmp_path / "o.png")), exp)


def test_palette_index_past_the_palette_takes_its_last_entry(tmp_path):
    """image.rs:103-110: an index beyond the palette is clamped to its last entry."""
    import struct
    import zlib

    idx = np.array([[0, 1, 2, 5], [5, 1, 0, 3]], np.uint8)
    pal = bytes([10, 20, 30, 200, 100, 50])  # two entries
    rows = b"".join(b"\0" + idx[y].tobytes() for y in range(idx.shape[0]))

    def chunk(kind, data):
        return struct.pack(">I", len(data)) + kind + data + struct.pack(">I", zlib.crc32(kind + data))

    png = (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", 4, 2, 8, 3, 0, 0, 0)) +
           chunk(b"PLTE", pal) + chunk(b"IDAT", zlib.compress(rows)) + chunk(b"IEND", b""))
    src = tmp_path / "pal.png"
    src.write_bytes(png)
    r = run("--decode-png", str(src), str(tmp_path / "o.png"))
    assert r.returncode == 0, r.stderr
    table = np.array([[10, 20, 30], [200, 100, 50]], np.uint8)
    np.testing.assert_array_equal(np.asarray(Image.open(tmp_path / "o.png")), table[np.minimum(idx, 1)])
