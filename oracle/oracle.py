"""ctypes access to the test oracles. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only as the
checker or the timed CPU baseline. The product library never calls into it.

Two oracles:
  * ``Restatement``: liboracle.so, the C restatement in matvec_oracle.c (always buildable).
  * ``RefQwen`` / ``RefRunq``: the reference's own qwen.c / runq.c compiled unchanged into oracle/_ref/ by
    oracle/Makefile (present when the reference tree was available at build time; they travel with the
    working tree to machines that do not have it).
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class Restatement:
    """The C restatement (matvec_oracle.c) of qwen.c/runq.c's quantize and matmul_cpu."""

    def __init__(self, path=os.path.join(HERE, "liboracle.so")):
        lib = C.CDLL(path)
        lib.orc_f16.restype = C.c_float
        lib.orc_f16.argtypes = [C.c_uint16]
        lib.orc_quantize_qwen.argtypes = [_i8p, _f32p, _f32p, C.c_int]
        lib.orc_quantize_runq.argtypes = [_i8p, _f32p, _f32p, C.c_int, C.c_int]
        lib.orc_group_sums.argtypes = [_i32p, _u8p, _i8p, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.orc_matvec_f16.argtypes = [_f32p, _u8p, _u16p, _i8p, _f32p, C.c_int, C.c_int, C.c_int]
        lib.orc_matvec_f32.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, C.c_int, C.c_int, C.c_int]
        lib.orc_expf_array.argtypes = [_f32p, _f32p, C.c_long]
        self.lib = lib

    def expf(self, x):
        """The host C library's expf, elementwise."""
        x = _c(x, np.float32)
        y = np.empty_like(x)
        self.lib.orc_expf_array(x, y, x.size)
        return y

    def f16(self, h):
        return self.lib.orc_f16(int(h))

    def quantize_qwen(self, x):
        x = _c(x, np.float32)
        q, s = np.empty(x.size, np.int8), np.empty(x.size // 32, np.float32)
        self.lib.orc_quantize_qwen(q, s, x, x.size)
        return q, s

    def quantize_runq(self, x, gs):
        x = _c(x, np.float32)
        q, s = np.empty(x.size, np.int8), np.empty(x.size // gs, np.float32)
        self.lib.orc_quantize_runq(q, s, x, x.size, gs)
        return q, s

    def group_sums(self, w, xq, n, d, gs, bits):
        out = np.empty(d * (n // gs), np.int32)
        self.lib.orc_group_sums(out, _c(w, np.uint8).reshape(-1), _c(xq, np.int8), n, d, gs, bits)
        return out.reshape(d, n // gs)

    def matvec_f16(self, w, ws, xq, xs, n, d, bits):
        out = np.empty(d, np.float32)
        self.lib.orc_matvec_f16(out, _c(w, np.uint8).reshape(-1), _c(ws, np.uint16).reshape(-1), _c(xq, np.int8),
                                _c(xs, np.float32), n, d, bits)
        return out

    def matvec_f32(self, wq, ws, xq, xs, n, d, gs):
        out = np.empty(d, np.float32)
        self.lib.orc_matvec_f32(out, _c(wq, np.int8).reshape(-1), _c(ws, np.float32).reshape(-1), _c(xq, np.int8),
                                _c(xs, np.float32), n, d, gs)
        return out


def ref_available(name="libref_qwen.so"):
    return os.path.exists(os.path.join(REF_DIR, name))


class RefQwen:
    """qwen/qwen.c itself (harness ref_qwen_harness.c). ``b200=True`` loads the -DFPGA build whose matmuls go
    through libmatvec_b200.so's fpga_matvec4."""

    def __init__(self, b200=False):
        lib = C.CDLL(os.path.join(REF_DIR, "libref_qwen_b200.so" if b200 else "libref_qwen.so"))
        lib.ref_qwen_quantize.argtypes = [_i8p, _f32p, _f32p, C.c_int]
        lib.ref_qwen_f16.restype = C.c_float
        lib.ref_qwen_f16.argtypes = [C.c_uint16]
        lib.ref_qwen_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        lib.ref_qwen_matmul_cpu.argtypes = [_f32p, _u8p, _u16p, _i8p, _f32p, C.c_int, C.c_int, C.c_int]
        lib.ref_qwen_open.argtypes = [C.c_char_p, C.c_int]
        lib.ref_qwen_config.argtypes = [C.POINTER(C.c_int)]
        lib.ref_qwen_forward.restype = C.POINTER(C.c_float)
        lib.ref_qwen_forward.argtypes = [C.c_int, C.c_int]
        lib.ref_qwen_head_ids.restype = C.POINTER(C.c_int32)
        lib.ref_qwen_argmax.argtypes = [C.POINTER(C.c_float), C.c_int]
        self.lib = lib
        self.cfg = None

    def f16(self, h):
        return self.lib.ref_qwen_f16(int(h))

    def quantize(self, x):
        x = _c(x, np.float32)
        q, s = np.empty(x.size, np.int8), np.empty(x.size // 32, np.float32)
        self.lib.ref_qwen_quantize(q, s, x, x.size)
        return q, s

    def rmsnorm(self, x, w, eps):
        x = _c(x, np.float32)
        o = np.empty_like(x)
        self.lib.ref_qwen_rmsnorm(o, x, _c(w, np.float32), x.size, eps)
        return o

    def matmul_cpu(self, w, ws, xq, xs, n, d, bits):
        out = np.empty(d, np.float32)
        self.lib.ref_qwen_matmul_cpu(out, _c(w, np.uint8).reshape(-1), _c(ws, np.uint16).reshape(-1),
                                     _c(xq, np.int8), _c(xs, np.float32), n, d, bits)
        return out

    def open(self, path, ctx):
        if self.lib.ref_qwen_open(path.encode(), ctx) != 0:
            raise RuntimeError("ref_qwen_open failed")
        cfg = (C.c_int * 8)()
        self.lib.ref_qwen_config(cfg)
        self.cfg = dict(zip(("dim", "hidden", "layers", "heads", "kv_heads", "vocab", "head_k", "ctx"), list(cfg)))
        hk = self.cfg["head_k"]
        self.head_ids = np.ctypeslib.as_array(self.lib.ref_qwen_head_ids(), (hk,)).copy()

    def forward(self, token, pos):
        p = self.lib.ref_qwen_forward(int(token), int(pos))
        return np.ctypeslib.as_array(p, (self.cfg["head_k"],)).copy()

    def greedy(self, prompt, n_gen):
        """Feeds the prompt one token at a time and decodes greedily, like qwen.c generate() at -t 0
        (qwen.c:669-701; stops early at <|im_end|> / <|endoftext|>). Returns (generated ids, logits per pos)."""
        out, logits, tok = [], [], prompt[0]
        for pos in range(len(prompt) + n_gen - 1):
            lg = self.forward(tok, pos)
            logits.append(lg)
            if pos < len(prompt) - 1:
                tok = prompt[pos + 1]
                continue
            nxt = int(self.head_ids[int(np.argmax(lg))])
            if nxt in (151645, 151643):
                break
            out.append(nxt)
            if len(out) >= n_gen:
                break
            tok = nxt
        return out, np.stack(logits)


class RefRunq:
    """runq/runq.c itself (harness ref_runq_harness.c, -DTESTING). ``b200=True`` loads the -DFPGA build."""

    def __init__(self, b200=False):
        lib = C.CDLL(os.path.join(REF_DIR, "libref_runq_b200.so" if b200 else "libref_runq.so"))
        lib.ref_runq_quantize.argtypes = [_i8p, _f32p, _f32p, C.c_int, C.c_int]
        lib.ref_runq_matmul_cpu.argtypes = [_f32p, _i8p, _f32p, _i8p, _f32p, C.c_int, C.c_int, C.c_int]
        lib.ref_runq_open.argtypes = [C.c_char_p]
        lib.ref_runq_config.argtypes = [C.POINTER(C.c_int)]
        lib.ref_runq_forward.restype = C.POINTER(C.c_float)
        lib.ref_runq_forward.argtypes = [C.c_int, C.c_int]
        self.lib = lib
        self.cfg = None

    def quantize(self, x, gs):
        x = _c(x, np.float32)
        q, s = np.empty(x.size, np.int8), np.empty(x.size // gs, np.float32)
        self.lib.ref_runq_quantize(q, s, x, x.size, gs)
        return q, s

    def matmul_cpu(self, wq, ws, xq, xs, n, d, gs):
        out = np.empty(d, np.float32)
        self.lib.ref_runq_matmul_cpu(out, _c(wq, np.int8).reshape(-1), _c(ws, np.float32).reshape(-1),
                                     _c(xq, np.int8), _c(xs, np.float32), n, d, gs)
        return out

    def open(self, path):
        if self.lib.ref_runq_open(path.encode()) != 0:
            raise RuntimeError("ref_runq_open failed")
        cfg = (C.c_int * 8)()
        self.lib.ref_runq_config(cfg)
        self.cfg = dict(zip(("dim", "hidden", "layers", "heads", "kv_heads", "vocab", "seq_len", "gs"), list(cfg)))

    def forward(self, token, pos):
        p = self.lib.ref_runq_forward(int(token), int(pos))
        return np.ctypeslib.as_array(p, (self.cfg["vocab"],)).copy()

    def greedy(self, prompt, n_pos):
        """Prompt tokens then greedy argmax for a total of n_pos positions (runq.c generate(), -t 0).
        Returns (ids after the prompt, logits per position)."""
        out, logits, tok = [], [], prompt[0]
        for pos in range(n_pos):
            lg = self.forward(tok, pos)
            logits.append(lg)
            nxt = prompt[pos + 1] if pos + 1 < len(prompt) else int(np.argmax(lg))
            if pos + 1 >= len(prompt):
                out.append(nxt)
            tok = nxt
        return out, np.stack(logits)
