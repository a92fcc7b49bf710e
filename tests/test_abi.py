"""The C ABI library: it loads, exports every entry point include/lightx2v_cuda.h
declares, and reports host-side errors without touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from lightx2v_cuda import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "lightx2v_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^LX2V_API[^;(]*?\b(lx2v_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_binding():
    syms = declared_symbols()
    assert len(syms) >= 25
    assert set(syms) == set(L.SIGNATURES), set(syms) ^ set(L.SIGNATURES)


def test_integration_guide_binds_every_declared_symbol():
    # the Rust side of the boundary (the extern "C" block and the methods of
    # the crate written out in INTEGRATION.md) names every entry point
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    missing = [s for s in declared_symbols() if not re.search(r"\b" + s + r"\b", doc)]
    assert not missing, missing


def test_library_exports_every_declared_symbol():
    lib = L.load()
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for s in declared_symbols():
        assert s in exported, s
        assert getattr(lib, s) is not None
    # nothing but the ABI is exported
    assert {s for s in exported if s.startswith("lx2v")} == set(declared_symbols())


def test_null_and_bad_arguments_are_errors_not_crashes():
    lib = L.load()
    assert lib.lx2v_buf_len(None, None, None) == L.ERR_INVALID
    assert b"null context" in lib.lx2v_last_error(None)
    assert lib.lx2v_set_linear_path(None, 1) == L.ERR_INVALID
    assert lib.lx2v_init(0, None) == L.ERR_INVALID


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device path")
def test_init_without_a_device_is_no_device():
    lib = L.load()
    ctx = ctypes.c_void_p()
    st = lib.lx2v_init(0, ctypes.byref(ctx))
    assert st == L.ERR_NO_DEVICE
    assert not ctx.value
    from lightx2v_cuda import CudaBackend
    assert CudaBackend.try_new() is None
