"""CPU tests of the C ABI boundary: libtmoe.so loads and exports every symbol include/tmoe.h
declares, and the host-side argument checks fail with codes (no compute without a GPU)."""
import ctypes as C
import os
import subprocess

import pytest

import tetraeder_b200 as tb
from tetraeder_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    names = _lib.header_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
    nm = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    assert set(names) <= exported
    # nothing else leaks out of the library but the ABI
    assert {n for n in exported if n.startswith("tmoe")} == set(names)


def test_version():
    assert _lib.load().tmoe_version() == 100


def test_create_rejects_bad_config_without_gpu():
    lib = _lib.load()
    cfg = _lib.Config(2048, 768, 128, 8, 12, 12, 14, 64, 0, 1e-6)
    bad = _lib.Config(2000, 768, 128, 8, 12, 12, 14, 64, 0, 1e-6)  # not a multiple of 256
    h = C.c_void_p()
    rc = lib.tmoe_create(C.byref(bad), C.byref(h))
    assert rc == -1 and not h.value
    assert b"256" in lib.tmoe_last_error(None)
    bad2 = _lib.Config(2048, 768, 128, 8, 2, 2, 14, 64, 0, 1e-6)  # Q4_0 is not a supported type
    assert lib.tmoe_create(C.byref(bad2), C.byref(h)) == -4
    assert lib.tmoe_create(None, C.byref(h)) == -1
    del cfg


def test_null_handle_calls_return_invalid():
    lib = _lib.load()
    assert lib.tmoe_route(None, None, None, 1, 0, None, None, None, None, None, None, None) == -1
    assert lib.tmoe_experts(None, None, None, 1, None, None, None, None) == -1
    assert lib.tmoe_check(None, None) == -1
    lib.tmoe_destroy(None)


def test_header_is_plain_c():
    """The header compiles as C (no C++ or torch types in the signatures)."""
    src = os.path.join(ROOT, "include", "tmoe.h")
    r = subprocess.run(["gcc", "-x", "c", "-std=c99", "-fsyntax-only", "-Wall", "-Werror", src],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_product_has_no_oracle_or_cpu_fallback():
    """The package never imports the oracle, and its ops need the CUDA library."""
    pkg = os.path.join(ROOT, "tetraeder_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "from oracle" not in text, f
                assert "tmoe_oracle" not in text, f


def test_moe_layer_requires_cuda():
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    with pytest.raises(RuntimeError, match="CUDA"):
        tb.MoeLayer(2048, 768, 128, 8)
