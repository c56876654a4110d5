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
        ip = C.POINTER(C.c_int)
        for name in ("mvb_qwen_load", "mvb_runq_load"):
            getattr(L, name).restype = vp
            getattr(L, name).argtypes = [vp, C.c_size_t, i]
        for name in ("mvb_qwen_load_file", "mvb_runq_load_file"):
            getattr(L, name).restype = vp
            getattr(L, name).argtypes = [C.c_char_p, i]
        L.mvb_qwen_config.restype = i
        L.mvb_qwen_config.argtypes = [vp, ip]
        L.mvb_qwen_stream.restype = vp
        L.mvb_qwen_stream.argtypes = [vp]
        L.mvb_qwen_forward.restype = i
        L.mvb_qwen_forward.argtypes = [vp, i, i, vp]
        L.mvb_qwen_prefill.restype = i
        L.mvb_qwen_prefill.argtypes = [vp, ip, i]
        L.mvb_qwen_prefill_tokenwise.restype = i
        L.mvb_qwen_prefill_tokenwise.argtypes = [vp, ip, i]
        L.mvb_qwen_cache.restype = i
        L.mvb_qwen_cache.argtypes = [vp, i, C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.mvb_qwen_decode.restype = i
        L.mvb_qwen_decode.argtypes = [vp, i, ip]
        for name in ("mvb_qwen_generate", "mvb_runq_generate"):
            getattr(L, name).restype = i
            getattr(L, name).argtypes = [vp, ip, i, i, ip]
        L.mvb_qwen_full_head.restype = i
        L.mvb_qwen_full_head.argtypes = [vp, i]
        L.mvb_qwen_rewind.restype = i
        L.mvb_qwen_rewind.argtypes = [vp, i, i, i]
        L.mvb_qwen_launch.restype = i
        L.mvb_qwen_launch.argtypes = [vp, i]
        L.mvb_qwen_free.restype = None
        L.mvb_qwen_free.argtypes = [vp]
        L.mvb_norm_matvec4_static.restype = i
        L.mvb_norm_matvec4_static.argtypes = [vp, vp, C.c_float, vp, vp, vp, i, i, i, vp]
        L.mvb_expf_eval.restype = i
        L.mvb_expf_eval.argtypes = [vp, vp, i, ip, C.POINTER(C.c_float), vp]
        L.mvb_qwen_trace.restype = i
        L.mvb_qwen_trace.argtypes = [vp, i, i, C.POINTER(C.c_float)]
        L.mvb_qwen_profile.restype = i
        L.mvb_qwen_profile.argtypes = [vp, C.POINTER(C.c_float), i]
        L.mvb_qwen_stamps.restype = i
        L.mvb_qwen_stamps.argtypes = [vp, C.POINTER(C.c_double), i]
        L.mvb_qwen_kernel_info.restype = i
        L.mvb_qwen_kernel_info.argtypes = [vp, i, i, C.c_char_p, i, ip, C.POINTER(C.c_double)]
        L.mvb_gemm4.restype = i
        L.mvb_gemm4.argtypes = [vp] * 5 + [i] * 5 + [vp]
        L.mvb_gemm_status.restype = i
        L.mvb_gemm_status.argtypes = [vp]
        L.mvb_gather_handle_size.restype = i
        L.mvb_gather_create.restype = vp
        L.mvb_gather_create.argtypes = [i, i, i, vp]
        L.mvb_gather_create_batch.restype = vp
        L.mvb_gather_create_batch.argtypes = [i, i, i, i, vp]
        L.mvb_gather_gemm4.restype = i
        L.mvb_gather_gemm4.argtypes = [vp] * 5 + [i] * 4 + [vp]
        L.mvb_gather_connect.restype = i
        L.mvb_gather_connect.argtypes = [vp, vp]
        L.mvb_gather_matvec4.restype = i
        L.mvb_gather_matvec4.argtypes = [vp] * 5 + [i, i, vp]
        L.mvb_gather_output.restype = vp
        L.mvb_gather_output.argtypes = [vp]
        L.mvb_gather_error.restype = i
        L.mvb_gather_error.argtypes = [vp, vp]
        L.mvb_gather_destroy.restype = None
        L.mvb_gather_destroy.argtypes = [vp]
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



def norm_matvec4_static(x, norm_w, eps, w, ws, out, n, d, wbits, stream=None):
    """rmsnorm + quantize + matvec4 on CUDA tensors with no device allocation (scratch in a fixed device array);
    returns the C return code (0, or -1 with last_error())."""
    return lib().mvb_norm_matvec4_static(_ptr(x), _ptr(norm_w), C.c_float(eps), _ptr(w), _ptr(ws), _ptr(out), n, d,
                                         wbits, _stream(stream))


def expf_device(x, y, stream=None):
    """y = the decode's expf of x (float32 CUDA tensors); returns (table entries, probe threshold)."""
    e, t = C.c_int(), C.c_float()
    check(lib().mvb_expf_eval(_ptr(x), _ptr(y), x.numel(), C.byref(e), C.byref(t), _stream(stream)), "mvb_expf_eval")
    return e.value, t.value


def gemm4(w, ws, xq, xs, out, n, d, m, ldx, wbits, stream=None):
    """m tokens through one matrix on the tensor cores (mvb_gemm4): out[t, i] = matvec4 of token t, row i.
    xq: (m, n) int8; xs: (n/32, ldx) fp32 group-major; out: (m, d) fp32 (CUDA tensors, asynchronous)."""
    return check(lib().mvb_gemm4(_ptr(w), _ptr(ws), _ptr(xq), _ptr(xs), _ptr(out), n, d, m, ldx, wbits,
                                 _stream(stream)), "mvb_gemm4")


def gemm_status(stream=None):
    """Synchronizes and returns the GEMM kernels' error word (0 = every internal wait completed)."""
    return lib().mvb_gemm_status(_stream(stream))


# ---- row-sharded matvec with the all-gather in the kernel (include/matvec_b200.h, mvb_gather_*) ----

class _DeviceVector:
    """A CUDA float32 vector at a device address owned by the library, for torch.as_tensor."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None}


class ShardGather:
    """One rank of a row-sharded matvec4 whose output rows are all-gathered inside the kernel.

        g = ShardGather(rank, world, rows)
        handles = exchange(g.handle())           # every rank's handle, in rank order (any host channel)
        g.connect(handles)
        g.matvec4(w_shard, ws_shard, xq, xs, n, 4)
        full = g.output()                        # torch view, rows * world fp32, valid in stream order
    """

    def __init__(self, rank, world, rows, tokens=1):
        L = lib()
        self.rank, self.world, self.rows, self.tokens = rank, world, rows, tokens
        self._m = 1
        buf = (C.c_uint8 * L.mvb_gather_handle_size())()
        self._g = L.mvb_gather_create_batch(rank, world, rows, tokens, buf)
        if not self._g:
            raise MatvecError(f"mvb_gather_create failed: {last_error()}")
        self._handle = bytes(buf)

    def handle(self):
        return self._handle

    def connect(self, handles):
        if len(handles) != self.world:
            raise ValueError(f"need {self.world} handles, got {len(handles)}")
        blob = b"".join(handles)
        check(lib().mvb_gather_connect(self._g, C.c_char_p(blob)), "mvb_gather_connect")

    def matvec4(self, w, ws, xq, xs, n, wbits, stream=None):
        self._m = 1
        return check(lib().mvb_gather_matvec4(self._g, _ptr(w), _ptr(ws), _ptr(xq), _ptr(xs), n, wbits,
                                              _stream(stream)), "mvb_gather_matvec4")

    def gemm4(self, w, ws, xq, xs, n, m, ldx, wbits, stream=None):
        """m tokens (xq (m, n) int8, xs (n/32, ldx) fp32 group-major) through this rank's shard on the tensor cores;
        output() is then (m, rows * world), token-major."""
        self._m = m
        return check(lib().mvb_gather_gemm4(self._g, _ptr(w), _ptr(ws), _ptr(xq), _ptr(xs), n, m, ldx, wbits,
                                            _stream(stream)), "mvb_gather_gemm4")

    def output(self):
        import torch
        ptr = lib().mvb_gather_output(self._g)
        if not ptr:
            raise MatvecError("no gathered output yet (call matvec4 first)")
        t = torch.as_tensor(_DeviceVector(ptr, self._m * self.rows * self.world), device="cuda")
        return t if self._m == 1 else t.view(self._m, self.rows * self.world)

    def error(self, stream=None):
        return lib().mvb_gather_error(self._g, _stream(stream))

    def close(self):
        if getattr(self, "_g", None):
            lib().mvb_gather_destroy(self._g)
            self._g = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- device-resident Qwen2 decode (include/matvec_b200.h, mvb_qwen_*) ----

class QwenDecoder:
    """A .qwb model resident on the current CUDA device, decoding through the captured step graph. A path is
    mapped and uploaded by the library itself (mvb_qwen_load_file); bytes go through mvb_qwen_load."""

    _load, _load_file = "mvb_qwen_load", "mvb_qwen_load_file"

    def __init__(self, path_or_bytes, ctx=1024):
        import numpy as np
        if isinstance(path_or_bytes, (bytes, bytearray, memoryview)):
            img = np.frombuffer(path_or_bytes, np.uint8)
            h = getattr(lib(), self._load)(img.ctypes.data, img.nbytes, ctx)
            who = self._load
        else:
            h = getattr(lib(), self._load_file)(os.fsencode(path_or_bytes), ctx)
            who = self._load_file
        if not h:
            raise MatvecError(who + " failed: " + last_error())
        self.h = h
        self._read_config()

    def _read_config(self):
        cfg = (C.c_int * 9)()
        check(lib().mvb_qwen_config(self.h, cfg), "mvb_qwen_config")
        keys = ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "head_k", "ctx",
                "kernels_per_step")
        self.cfg = dict(zip(keys, list(cfg)))

    @staticmethod
    def _ids(a):
        import numpy as np
        return np.ascontiguousarray(a, dtype=np.int32)

    def forward(self, token, pos, want_logits=True):
        """(greedy head row, logits or None) of one forward at `pos`."""
        import numpy as np
        lg = np.empty(self.cfg["head_k"], np.float32) if want_logits else None
        row = lib().mvb_qwen_forward(self.h, int(token), int(pos), lg.ctypes.data if lg is not None else None)
        if row < 0:
            raise MatvecError("mvb_qwen_forward failed: " + last_error())
        return row, lg

    def prefill(self, prompt):
        p = self._ids(prompt)
        check(lib().mvb_qwen_prefill(self.h, p.ctypes.data_as(C.POINTER(C.c_int)), p.size), "mvb_qwen_prefill")

    def prefill_tokenwise(self, prompt):
        """The same state as prefill(), reached one decode step per fed token."""
        p = self._ids(prompt)
        check(lib().mvb_qwen_prefill_tokenwise(self.h, p.ctypes.data_as(C.POINTER(C.c_int)), p.size),
              "mvb_qwen_prefill_tokenwise")

    def cache(self, positions):
        """(k, v): the KV-cache rows of positions 0 .. positions-1, arrays (n_layers, positions, kv_dim)."""
        import numpy as np
        kvd = self.cfg["n_kv_heads"] * (self.cfg["dim"] // self.cfg["n_heads"])
        k = np.empty((self.cfg["n_layers"], positions, kvd), np.float32)
        v = np.empty_like(k)
        f = C.POINTER(C.c_float)
        check(lib().mvb_qwen_cache(self.h, positions, k.ctypes.data_as(f), v.ctypes.data_as(f)), "mvb_qwen_cache")
        return k, v

    def decode(self, steps):
        import numpy as np
        out = np.empty(steps, np.int32)
        if lib().mvb_qwen_decode(self.h, steps, out.ctypes.data_as(C.POINTER(C.c_int))) != steps:
            raise MatvecError("mvb_qwen_decode failed: " + last_error())
        return out

    def generate(self, prompt, steps):
        import numpy as np
        p = self._ids(prompt)
        out = np.empty(steps, np.int32)
        n = lib().mvb_qwen_generate(self.h, p.ctypes.data_as(C.POINTER(C.c_int)), p.size, steps,
                                    out.ctypes.data_as(C.POINTER(C.c_int)))
        if n < 0:
            raise MatvecError("mvb_qwen_generate failed: " + last_error())
        return out[:n]

    def full_head(self, on=True):
        """Use the whole vocabulary (the tied Q8 embedding) as the head instead of the trimmed head_ids head."""
        check(lib().mvb_qwen_full_head(self.h, int(bool(on))), "mvb_qwen_full_head")
        self._read_config()

    def rewind(self, token, pos, n_prompt):
        check(lib().mvb_qwen_rewind(self.h, token, pos, n_prompt), "mvb_qwen_rewind")

    def launch(self, count):
        check(lib().mvb_qwen_launch(self.h, count), "mvb_qwen_launch")

    def profile(self):
        """Durations (ms) of every kernel of one instrumented step from the current state."""
        import numpy as np
        ms = np.zeros(self.cfg["kernels_per_step"], np.float32)
        n = lib().mvb_qwen_profile(self.h, ms.ctypes.data_as(C.POINTER(C.c_float)), ms.size)
        if n < 0:
            raise MatvecError("mvb_qwen_profile failed: " + last_error())
        return ms[:n]

    def stamps(self):
        """One step as the graph runs it, every kernel stamping the global timer: array (kernels, 2) of
        (first CTA past its wait, last CTA done) in microseconds after the step's start."""
        import numpy as np
        us = np.zeros(2 * self.cfg["kernels_per_step"], np.float64)
        n = lib().mvb_qwen_stamps(self.h, us.ctypes.data_as(C.POINTER(C.c_double)), us.size)
        if n < 0:
            raise MatvecError("mvb_qwen_stamps failed: " + last_error())
        return us[:2 * n].reshape(n, 2)

    def trace(self, token, pos):
        """Residual stream after the embedding and after every attention / FFN block: [2 * n_layers + 1, dim]."""
        import numpy as np
        out = np.empty((2 * self.cfg["n_layers"] + 1, self.cfg["dim"]), np.float32)
        check(lib().mvb_qwen_trace(self.h, int(token), int(pos), out.ctypes.data_as(C.POINTER(C.c_float))),
              "mvb_qwen_trace")
        return out

    def kernel_info(self, pos):
        """[(kind, layer, algorithmic bytes at position pos)] for every kernel of the step."""
        out = []
        for k in range(self.cfg["kernels_per_step"]):
            kind, layer, b = C.create_string_buffer(32), C.c_int(), C.c_double()
            check(lib().mvb_qwen_kernel_info(self.h, k, pos, kind, 32, C.byref(layer), C.byref(b)), "kernel_info")
            out.append((kind.value.decode(), layer.value, b.value))
        return out

    @property
    def stream_handle(self):
        return lib().mvb_qwen_stream(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().mvb_qwen_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RunqDecoder(QwenDecoder):
    """A runq version 2 checkpoint (runq/runq.c's int8 model) resident on the current CUDA device, decoding with
    runq.c's arithmetic through the same captured step graph and the same calls (mvb_runq_load*). ``head_k`` is
    the vocabulary (the classifier's row is the token id), and generate() stops at BOS = 1 like runq.c:1016."""

    _load, _load_file = "mvb_runq_load", "mvb_runq_load_file"
