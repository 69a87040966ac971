"""The `.safetensors` container: a little-endian u64 header length, that many
bytes of JSON (`{name: {dtype, shape, data_offsets}}` plus an optional
`__metadata__`), then the payloads.

The writer keeps the layout of the reference's dependency-free writer
(lama-rs/safetensors_light.py:21-65): payloads in the given order, each padded
to start on an `align`-byte boundary, the JSON header padded with spaces so the
payload section starts aligned too, and `__metadata__` leading the header.  The
reader applies the checks the reference's weight store applies
(lama-rs/src/weights.rs:80-106): F32 only, every tensor inside the file.
"""

from __future__ import annotations

import io
import json
import struct

import numpy as np


def write_safetensors(path, tensors, metadata=None, align=8) -> int:
    """Write `(name, dtype, shape, raw_bytes)` tuples; returns payload bytes."""
    payload = io.BytesIO()
    header: dict = {}
    for name, dtype, shape, raw in tensors:
        if payload.tell() % align:
            payload.write(b"\x00" * (align - payload.tell() % align))
        start = payload.tell()
        payload.write(raw)
        header[name] = {"dtype": dtype, "shape": list(shape),
                        "data_offsets": [start, payload.tell()]}
    if metadata:
        header = {"__metadata__": {str(k): str(v) for k, v in metadata.items()}, **header}
    blob = json.dumps(header, separators=(",", ":")).encode("utf-8")
    pad = (-(8 + len(blob))) % align
    blob += b" " * pad
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(blob)))
        fh.write(blob)
        fh.write(payload.getvalue())
    return payload.tell()


class SafeTensors:
    """Read-only view of a container: `names()` in file order, `f32(name)`."""

    def __init__(self, path):
        with open(path, "rb") as fh:
            data = fh.read()
        if len(data) < 8:
            raise ValueError(f"{path}: too short for a safetensors header")
        (hlen,) = struct.unpack("<Q", data[:8])
        if 8 + hlen > len(data):
            raise ValueError(f"{path}: header length {hlen} past end of file")
        header = json.loads(data[8:8 + hlen].decode("utf-8"))
        self.metadata = header.pop("__metadata__", {})
        self._base = 8 + hlen
        self._data = data
        self._info = {}
        for name, t in header.items():
            if t["dtype"] != "F32":
                raise ValueError(f"tensor {name} is {t['dtype']}, not F32 - is this a big-lama checkpoint?")
            a, b = t["data_offsets"]
            if not (0 <= a <= b and self._base + b <= len(data)):
                raise ValueError(f"tensor {name}: data_offsets {a}..{b} outside the file")
            n = int(np.prod(t["shape"])) if t["shape"] else 1
            if b - a != 4 * n:
                raise ValueError(f"tensor {name}: {b - a} bytes for shape {t['shape']}")
            self._info[name] = (tuple(t["shape"]), a, b)
        # JSON object order is the file's tensor order (json keeps insertion order).
        self._order = list(self._info)
        if not self._order:
            raise ValueError(f"no tensors found in {path}")

    def names(self):
        return list(self._order)

    def shape(self, name):
        return self._info[name][0]

    def f32(self, name) -> np.ndarray:
        if name not in self._info:
            raise KeyError(f"missing tensor in weight blob: {name}")
        shape, a, b = self._info[name]
        return np.frombuffer(self._data, dtype="<f4", count=(b - a) // 4,
                             offset=self._base + a).reshape(shape).copy()
