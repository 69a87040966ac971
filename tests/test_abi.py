"""The C-ABI library loads and exports every symbol include/lama_b200.h declares.

No compute calls: this runs on a machine without a GPU.
"""

import ctypes
import os
import re

from lama_b200 import engine

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "lama_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lama_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_operator_surface():
    names = declared_functions()
    for n in ("lama_open", "lama_forward", "lama_inpaint_u8", "lama_last_error", "lama_close"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(engine.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    bound = {n for n, _, _ in engine.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_abi_version_is_callable_without_a_gpu():
    assert engine.lib().lama_abi_version() == 1


def test_last_error_on_null_engine():
    assert engine.lib().lama_last_error(None) == b"null engine"


def test_entry_points_refuse_a_null_engine_without_touching_the_gpu():
    """Every engine entry point returns LAMA_EINVAL (-1) for a null engine
    before any CUDA call, including the streamed and --sections drivers."""
    L = engine.lib()
    u8 = ctypes.c_uint8 * 16
    buf = u8()
    p = ctypes.cast(buf, ctypes.POINTER(ctypes.c_uint8))
    rects = (ctypes.c_int * 4)(0, 0, 2, 2)
    assert L.lama_inpaint_u8(None, p, p, 1, 2, 2, p) == -1
    assert L.lama_inpaint_u8_stream(None, p, p, 1, 2, 2, 1, p) == -1
    assert L.lama_inpaint_sections_u8(None, p, p, 2, 2, rects, 1, 2, p) == -1
    assert L.lama_synchronize(None) == -1


def test_binding_rejects_mismatched_shapes_before_calling_the_library():
    """Wrong shapes would make the library read or write past a host buffer; the
    binding refuses them first (an engine without a handle: no GPU needed)."""
    import numpy as np
    import pytest

    eng = engine.Engine.__new__(engine.Engine)
    eng._h = None
    bad = [
        (eng.forward, (np.zeros((3, 8, 8), np.float32),)),
        (eng.forward, (np.zeros((8, 8), np.float32),)),
        (eng.inpaint_u8, (np.zeros((8, 8, 4), np.uint8), np.zeros((8, 8), np.uint8))),
        (eng.inpaint_u8, (np.zeros((8, 8, 3), np.uint8), np.zeros((8, 9), np.uint8))),
        (eng.inpaint_u8_stream, (np.zeros((2, 8, 8, 4), np.uint8), np.zeros((2, 8, 8), np.uint8), 1)),
        (eng.inpaint_sections_u8, (np.zeros((8, 8), np.uint8), np.zeros((8, 8), np.uint8), [], 8)),
        (eng.resblocks, (np.zeros((128, 8, 8), np.float32), np.zeros((192, 8, 8), np.float32))),
        (eng.resblocks, (np.zeros((64, 8, 8), np.float32), np.zeros((384, 8, 8), np.float32))),
    ]
    for fn, args in bad:
        with pytest.raises(engine.LamaError) as ex:
            fn(*args)
        assert ex.value.code == -1, fn.__name__


def test_header_is_plain_c_and_links_against_the_library(tmp_path):
    """A C caller (the reference's FFI side is C-ABI) compiles against the header
    with a strict C99 compiler and links the library; the program calls an entry
    point that needs no GPU."""
    import shutil
    import subprocess
    import pytest

    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    inc = os.path.join(ROOT, "include")
    libdir = os.path.dirname(engine.LIB_PATH)
    src = tmp_path / "caller.c"
    src.write_text('#include "lama_b200.h"\n'
                   "int main(void) {\n"
                   "  lama_engine* e = 0;\n"
                   "  if (lama_open(0, 0, &e) != LAMA_EINVAL) return 2;\n"
                   "  lama_close(e);\n"
                   "  return lama_abi_version() == 1 ? 0 : 1;\n"
                   "}\n")
    exe = tmp_path / "caller"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", inc, str(src),
                        "-L", libdir, "-llama_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert subprocess.run([str(exe)]).returncode == 0


def test_a_missing_library_fails_loudly(tmp_path):
    """No silent fallback: without liblama_b200.so the binding raises at its
    first use instead of computing anything another way."""
    import subprocess
    import sys

    code = ("import sys; sys.path.insert(0, sys.argv[1])\n"
            "from lama_b200 import engine\n"
            "try:\n"
            "    engine.lib()\n"
            "except OSError as x:\n"
            "    print('raised:', x)\n"
            "    sys.exit(0)\n"
            "sys.exit(1)\n")
    env = dict(os.environ, LAMA_B200_LIB=str(tmp_path / "absent.so"))
    r = subprocess.run([sys.executable, "-c", code, os.path.join(ROOT, "lama-inpaint-rs_b200")], env=env,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "is missing" in r.stdout, r.stdout + r.stderr


def test_the_product_never_reaches_the_oracle():
    """The oracle is test infrastructure: nothing in the engine package (CUDA
    sources, C ABI, CLI, Python binding) imports, links or names it."""
    pkg = os.path.join(ROOT, "lama-inpaint-rs_b200")
    hits = []
    for d, _, files in os.walk(pkg):
        if "_build" in d:
            continue
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h", "Makefile")) or f == "Makefile":
                txt = open(os.path.join(d, f), errors="replace").read()
                if re.search(r"\boracle\b", txt):
                    hits.append(os.path.join(d, f))
    assert not hits, hits
