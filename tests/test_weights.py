"""The checkpoint container and the engine's load-time checks.

Golden fixture: tests/golden/container_ref.safetensors was written by the
reference's own writer (lama-rs/safetensors_light.py).  The load-time checks
follow lama-rs/src/weights.rs:80-106 (F32 only, payload inside the file) and
the loaders' "missing tensor in weight blob" error; the engine validates the
whole file on the host before it touches the GPU, so these run on CPU.
"""

import json
import os
import struct

import numpy as np
import pytest

from lama_b200 import plan, seeded
from lama_b200.safetensors_io import SafeTensors, write_safetensors

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_tensor_inventory_is_the_big_lama_checkpoint():
    tl = plan.tensor_list()
    assert len(tl) == 989
    conv = [n for n, s in tl if len(s) == 4 or n.endswith(".bias") and not any(
        b in n for b in (".bn_l", ".bn_g", ".conv1.1", ".fu.bn", "model.25", "model.28", "model.31"))]
    assert len(conv) == 229
    assert sum(1 for n, _ in tl if n.endswith("running_var")) == 152
    nparams = sum(int(np.prod(s)) if s else 1 for _, s in tl)
    assert 50.9e6 < nparams < 51.1e6
    d = dict(tl)
    assert d["model.5.conv1.ffc.convl2l.weight"] == (128, 128, 3, 3)
    assert d["model.5.conv1.ffc.convg2g.fu.conv_layer.weight"] == (384, 384, 1, 1)
    assert d["model.24.weight"] == (512, 256, 3, 3)
    assert d["model.34.weight"] == (3, 64, 7, 7)
    assert d["model.22.conv2.bn_g.num_batches_tracked"] == ()


def test_writer_matches_the_reference_writer_byte_for_byte():
    meta = json.load(open(os.path.join(GOLD, "container_ref.json")))
    tensors = [(n, "F32", list(v.shape), v.astype("<f4").tobytes())
               for n, v in seeded.make_weights(meta["seed"])[: meta["tensors"]]]
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "mine.safetensors")
        write_safetensors(p, tensors)
        assert open(p, "rb").read() == open(os.path.join(GOLD, "container_ref.safetensors"), "rb").read()


def test_reader_parses_the_reference_container():
    st = SafeTensors(os.path.join(GOLD, "container_ref.safetensors"))
    ws = seeded.make_weights()[:12]
    assert st.names() == [n for n, _ in ws]
    for n, v in ws:
        np.testing.assert_array_equal(st.f32(n), v)


def test_seeded_weights_are_reproducible_and_follow_the_init_rules():
    a = dict(seeded.make_weights())
    b = dict(seeded.make_weights())
    for k in ("model.5.conv1.ffc.convl2l.weight", "model.25.running_var", "model.34.bias"):
        np.testing.assert_array_equal(a[k], b[k])
    g = a["model.5.conv1.bn_l.weight"]
    assert g.min() >= 0.8 and g.max() <= 1.2
    v = a["model.5.conv1.bn_l.running_var"]
    assert v.min() >= 0.5 and v.max() <= 1.5
    assert np.all(a["model.5.conv1.bn_l.running_mean"] == 0)
    w = a["model.2.ffc.convl2l.weight"]
    assert abs(w.std() - np.sqrt(2.0 / (64 * 9))) < 0.01 * np.sqrt(2.0 / (64 * 9)) * 10


# ------------------------------------------------------------ engine load checks (CPU)

def _engine_error(path):
    from lama_b200 import Engine, LamaError
    with pytest.raises(LamaError) as ei:
        Engine(path, 0)
    return ei.value


def _rewrite(tmp_path, mutate):
    tl = seeded.make_weights()
    tensors = [(n, "F32", list(v.shape), v.astype("<f4").tobytes()) for n, v in tl]
    tensors = mutate(tensors)
    p = str(tmp_path / "w.safetensors")
    write_safetensors(p, tensors)
    return p


def test_missing_weight_file_is_a_weights_error(tmp_path):
    e = _engine_error(str(tmp_path / "nope.safetensors"))
    assert e.code == -2 and "cannot open" in e.msg


def test_non_f32_tensor_is_rejected(tmp_path):
    def mut(ts):
        n, _, s, raw = ts[3]
        ts[3] = (n, "F16", s, raw[: len(raw) // 2])
        return ts
    e = _engine_error(_rewrite(tmp_path, mut))
    assert e.code == -2 and "not F32" in e.msg


def test_missing_tensor_names_the_tensor(tmp_path):
    e = _engine_error(_rewrite(tmp_path, lambda ts: [t for t in ts if t[0] != "model.7.conv2.ffc.convg2l.weight"]))
    assert e.code == -2 and "missing tensor in weight blob: model.7.conv2.ffc.convg2l.weight" in e.msg


def test_wrong_shape_is_rejected(tmp_path):
    def mut(ts):
        return [(n, d, [s[1], s[0]] + s[2:] if n == "model.3.ffc.convl2l.weight" else s, r) for n, d, s, r in ts]
    e = _engine_error(_rewrite(tmp_path, mut))
    assert e.code == -2 and "model.3.ffc.convl2l.weight" in e.msg and "shape" in e.msg


def test_truncated_file_is_rejected(tmp_path, weights_baseline):
    data = open(weights_baseline, "rb").read()
    p = tmp_path / "trunc.safetensors"
    p.write_bytes(data[: len(data) // 2])
    e = _engine_error(str(p))
    assert e.code == -2 and ("outside the file" in e.msg or "truncated" in e.msg)


def test_header_length_past_end_is_rejected(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    e = _engine_error(str(p))
    assert e.code == -2


def _raw_container(tmp_path, shape_json, offsets=(0, 16)):
    import json as _json
    header = '{"t": {"dtype": "F32", "shape": %s, "data_offsets": [%d, %d]}}' % (shape_json, *offsets)
    _json.loads(header)  # well-formed JSON; only the numbers are hostile
    p = tmp_path / "hostile.safetensors"
    p.write_bytes(struct.pack("<Q", len(header)) + header.encode() + b"\0" * offsets[1])
    return str(p)


@pytest.mark.parametrize("shape_json,msg", [
    ("[99999999999999999999999]", "bad shape"),           # does not fit int64
    ("[-1, -4]", "negative or oversized dimension"),       # product 4 matches the payload
    ("[4611686018427387904, 4]", "negative or oversized dimension"),  # product overflows
])
def test_hostile_shapes_are_rejected_without_overflow(tmp_path, shape_json, msg):
    e = _engine_error(_raw_container(tmp_path, shape_json))
    assert e.code == -2 and msg in e.msg


def test_a_valid_checkpoint_passes_every_weight_check_before_the_device(weights_baseline):
    """Parsing, name/shape checks, BN folding and repacking all run on the host
    before any CUDA call, so without a GPU the first error is the device's."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the engine would open")
    e = _engine_error(weights_baseline)
    assert e.code == -3, e.msg


def test_engines_open_from_several_threads_at_once(weights_baseline):
    """Engines on different devices may be opened and driven from different
    threads: the host side of lama_open keeps no process-wide state, so four
    concurrent opens each get their own engine and their own error text
    (ctypes releases the GIL around the call)."""
    import threading

    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the engines would open")
    errs = [None] * 4

    def one(i):
        try:
            errs[i] = _engine_error(weights_baseline)
        except BaseException as x:  # recorded and checked below
            errs[i] = x

    ts = [threading.Thread(target=one, args=(i,)) for i in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert all(getattr(e, "code", None) == -3 for e in errs), errs
