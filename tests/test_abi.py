"""The C-ABI library without a GPU: it loads, exports every entry point include/*.h declares, and keeps the
reference driver's error behaviour for calls made before fpga_open() (driver/matvec_fpga.cpp:127-129,
174-176, 208-210). No compute call runs here."""
import ctypes as C
import subprocess
import sys

import pytest

from conftest import ROOT


def test_library_builds_and_loads(mvb):
    mvb.lib()


def test_exports_every_declared_symbol(mvb):
    names = mvb.declared_symbols()
    # the reference's six, then this library's additions
    for ref in ("fpga_open", "fpga_alloc", "fpga_alloc_try", "fpga_matvec", "fpga_matvec4", "fpga_close"):
        assert ref in names
    out = subprocess.run(["nm", "-D", "--defined-only", mvb.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_calls_before_open_fail(mvb):
    L = mvb.lib()
    L.fpga_close()  # safe when nothing is open (reference cpp:235-243)
    assert mvb.fpga_matvec4(0, 0, 0, 0, 0, 896, 896, 4) == -1
    assert "fpga_open() not called" in mvb.last_error()
    assert mvb.fpga_matvec(0, 0, 0, 0, 0, 288, 288, 32) == -1
    buf, phys = mvb.fpga_alloc_try(4096)
    assert buf is None and phys == 0
    buf, phys = mvb.fpga_alloc(4096)
    assert buf is None and "fpga_open() not called" in mvb.last_error()


def test_open_without_gpu_fails_loudly(mvb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert mvb.fpga_open() == -1
    assert mvb.last_error().startswith("fpga:")


def test_bad_memidx_rejected(mvb):
    # FPGA_MEMIDX is parsed like the reference (cpp:83-91) before any device is touched
    code = ("import sys; sys.path.insert(0, %r); from conftest import load_pkg; m = load_pkg(); "
            "rc = m.fpga_open(); print(rc, m.last_error())" % (ROOT + "/tests"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       env={"FPGA_MEMIDX": "x1", "PATH": "/usr/bin:/bin"})
    assert r.stdout.startswith("-1 fpga: bad FPGA_MEMIDX"), r.stdout + r.stderr


def test_header_is_plain_c():
    """include/*.h compile as C with no CUDA or torch types (what a cgo/ctypes/JNI binding sees)."""
    src = '#include "matvec_b200.h"\nint main(void){return 0;}\n'
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-x", "c", "-I", ROOT + "/include", "-", "-o",
                        "/dev/null"], input=src, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
