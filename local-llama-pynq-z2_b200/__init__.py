"""B200 group-quantized matvec behind the reference's driver/matvec_fpga.h C ABI.

Python mirror of the C ABI in include/matvec_fpga.h and include/matvec_b200.h, over ctypes. The names,
argument meanings and 0/-1 returns are the reference driver's (driver/matvec_fpga.h:12-33); ``check()`` turns a
-1 into an exception carrying the library's message.

    import mvb
    mvb.fpga_open()
    buf, phys = mvb.fpga_alloc(nbytes)       # numpy uint8 view of the pinned host buffer, device address
    ...write weights / activations into buf...
    mvb.fpga_matvec4(phys_w, phys_ws, phys_xq, phys_xs, phys_out, n, d, 4)
    ...read the result from buf...

The library is built in-tree (build.py) and must be present: there is no fallback of any kind.
"""
import ctypes as C
import os
import re

from . import qwb  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmatvec_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

_lib = None


class MatvecError(RuntimeError):
    pass


def lib():
    """The loaded libmatvec_b200.so; raises if it was not built (python build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MatvecError(f"{LIB_PATH} is missing: build it with python {os.path.join(HERE, 'build.py')}")
        L = C.CDLL(LIB_PATH)
        u64, i, vp = C.c_uint64, C.c_int, C.c_void_p
        L.fpga_open.restype = i
        L.fpga_alloc.restype = vp
        L.fpga_alloc.argtypes = [C.c_size_t, C.POINTER(u64)]
        L.fpga_alloc_try.restype = vp
        L.fpga_alloc_try.argtypes = [C.c_size_t, C.POINTER(u64)]
        L.fpga_matvec.restype = i
        L.fpga_matvec.argtypes = [u64] * 5 + [i] * 3
        L.fpga_matvec4.restype = i
        L.fpga_matvec4.argtypes = [u64] * 5 + [i] * 3
        L.fpga_close.restype = None
        L.mvb_last_error.restype = C.c_char_p
        for name in ("mvb_matvec4", "mvb_matvec"):
            f = getattr(L, name)
            f.restype = i
            f.argtypes = [vp] * 5 + [i] * 3 + [vp]
        for name in ("mvb_qmatvec4", "mvb_qmatvec"):
            f = getattr(L, name)
            f.restype = i
            f.argtypes = [vp] * 4 + [i] * 3 + [vp]
        L.mvb_rows_per_tile.restype = i
        L.mvb_rows_per_tile.argtypes = [i, i]
        _bind_extra(L)
        _lib = L
    return _lib


def _bind_extra(L):
    """Hook for entry points added by other modules of the package (set by them at import)."""
    for f in _extra_binders:
        f(L)


_extra_binders = []


def declared_symbols():
    """Every function name declared in include/*.h (the exported C ABI)."""
    names = []
    for h in sorted(os.listdir(INCLUDE)):
        if h.endswith(".h"):
            text = re.sub(r"/\*.*?\*/", "", open(os.path.join(INCLUDE, h)).read(), flags=re.S)
            names += re.findall(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\([^;{]*\)\s*;", text, flags=re.M)
    return names


def last_error():
    return lib().mvb_last_error().decode()


def check(rc, what="call"):
    if rc != 0:
        raise MatvecError(f"{what} failed: {last_error()}")
    return rc


# ---- the reference's six entry points (driver/matvec_fpga.h:15-33) ----

def fpga_open():
    return lib().fpga_open()


def _alloc(fn, nbytes):
    import numpy as np
    phys = C.c_uint64(0)
    p = fn(nbytes, C.byref(phys))
    if not p:
        return None, 0
    arr = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), (nbytes,))
    return arr, phys.value


def fpga_alloc(nbytes):
    """(numpy uint8 view of the pinned host buffer, device address) or (None, 0)."""
    return _alloc(lib().fpga_alloc, nbytes)


def fpga_alloc_try(nbytes):
    return _alloc(lib().fpga_alloc_try, nbytes)


def fpga_matvec(wq, ws, xq, xs, out, n, d, gs):
    return lib().fpga_matvec(wq, ws, xq, xs, out, n, d, gs)


def fpga_matvec4(w, ws, xq, xs, out, n, d, wbits):
    return lib().fpga_matvec4(w, ws, xq, xs, out, n, d, wbits)


def fpga_close():
    lib().fpga_close()


# ---- device-pointer entry points (include/matvec_b200.h), for torch CUDA tensors ----

def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def matvec4(w, ws, xq, xs, out, n, d, wbits, stream=None):
    """out = fpga_matvec4's computation on CUDA tensors (asynchronous on `stream`)."""
    return check(lib().mvb_matvec4(_ptr(w), _ptr(ws), _ptr(xq), _ptr(xs), _ptr(out), n, d, wbits, _stream(stream)),
                 "mvb_matvec4")


def matvec(wq, ws, xq, xs, out, n, d, gs, stream=None):
    """out = fpga_matvec's computation (runq, fp32 scales) on CUDA tensors."""
    return check(lib().mvb_matvec(_ptr(wq), _ptr(ws), _ptr(xq), _ptr(xs), _ptr(out), n, d, gs, _stream(stream)),
                 "mvb_matvec")


def qmatvec4(w, ws, x, out, n, d, wbits, stream=None):
    """matvec4 with qwen.c's activation quantization fused into the kernel (x: fp32 CUDA tensor)."""
    return check(lib().mvb_qmatvec4(_ptr(w), _ptr(ws), _ptr(x), _ptr(out), n, d, wbits, _stream(stream)),
                 "mvb_qmatvec4")


def qmatvec(wq, ws, x, out, n, d, gs, stream=None):
    """matvec with runq.c's activation quantization fused into the kernel."""
    return check(lib().mvb_qmatvec(_ptr(wq), _ptr(ws), _ptr(x), _ptr(out), n, d, gs, _stream(stream)),
                 "mvb_qmatvec")


def rows_per_tile(n, d):
    return lib().mvb_rows_per_tile(n, d)
