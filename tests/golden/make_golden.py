"""Regenerate the committed golden fixtures (run in a container that has the
reference checkout; the fixtures themselves travel with the repo).

container_ref.safetensors
    A small safetensors file written by the reference's OWN dependency-free
    writer (lama-rs/safetensors_light.py, imported from the reference tree)
    from the first 12 seeded big-lama tensors.  The tests check that this
    repo's writer produces the same bytes from the same tensors and that both
    readers (the Python one and the engine's C++ one) parse it.

ref_testdata_in.png, ref_testdata_mask.png
    The reference's own example inputs (testdata/in.png, 512x512 RGB, and
    testdata/mask.png, 512x512 grey, 38,000 masked pixels), copied byte for
    byte; their SHA-256 digests are recorded in ref_testdata.json.  The GPU
    tests run them through the CLI and compare with the oracle.

Usage: python tests/golden/make_golden.py /path/to/reference
"""

import hashlib
import importlib.util
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "lama-inpaint-rs_b200"))

from lama_b200 import seeded  # noqa: E402

N_TENSORS = 12


def fixture_tensors():
    return [(n, "F32", list(v.shape), v.astype("<f4").tobytes()) for n, v in seeded.make_weights()[:N_TENSORS]]


def main():
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference checkout (holds lama-rs/safetensors_light.py)>")
    ref = sys.argv[1]
    spec = importlib.util.spec_from_file_location("safetensors_light", os.path.join(ref, "lama-rs", "safetensors_light.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = os.path.join(HERE, "container_ref.safetensors")
    mod.write_safetensors(out, fixture_tensors())
    with open(os.path.join(HERE, "container_ref.json"), "w") as f:
        json.dump({"writer": "lama-rs/safetensors_light.py:21-65", "tensors": N_TENSORS,
                   "seed": seeded.WEIGHT_SEED, "bytes": os.path.getsize(out)}, f, indent=1)
    print("wrote", out, os.path.getsize(out), "bytes")
    digests = {}
    for name in ("in.png", "mask.png"):
        dst = os.path.join(HERE, "ref_testdata_" + name)
        shutil.copyfile(os.path.join(ref, "testdata", name), dst)
        digests["ref_testdata_" + name] = hashlib.sha256(open(dst, "rb").read()).hexdigest()
    with open(os.path.join(HERE, "ref_testdata.json"), "w") as f:
        json.dump({"source": "reference testdata/in.png and testdata/mask.png", "sha256": digests}, f, indent=1)
    print("copied the reference's testdata PNGs")


if __name__ == "__main__":
    main()
