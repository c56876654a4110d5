"""The reference's weight files, written from seeded synthetic values and read back as numpy views.

``.qwb`` (Qwen2 weights for qwen/qwen.c) follows the layout that tools/gguf2qwb.py:5-15 documents and
qwen/qwen.c:211-271 reads:
  header, 256 bytes: "QWB1", uint32 version 1, int32 dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size,
      head_k, max_seq_len, group_size (32), emb_bits (8), float32 rope_theta, rms_eps, zero padding
  float32 attn_norm[L][dim], ffn_norm[L][dim], bq[L][dim], bk[L][kv_dim], bv[L][kv_dim], output_norm[dim]
  int32 head_ids[head_k] (ascending token ids of the output-head rows)
  matrices, each a weight plane then an fp16 scale plane (one per group of 32 along a row):
      wq[L], wk[L], wv[L], wo[L], w1[L] (gate), w2[L] (down), w3[L] (up) as 4-bit; head, embedding as 8-bit
  every array starts on a 64-byte boundary. 4-bit planes hold two's complement nibbles, element 2i of a row
  in the low nibble of byte i.

runq v2 (llama2.c int8 files for runq/runq.c) follows runq.c:318-357 and tools/bin2q80.py:49-58:
  header, 256 bytes: uint32 0x616b3432, int32 version 2, int32 dim, hidden_dim, n_layers, n_heads, n_kv_heads,
      vocab_size, seq_len, uint8 shared_classifier, int32 group_size, zero padding
  float32 rms_att[L][dim], rms_ffn[L][dim], rms_final[dim]
  then int8 values followed by float32 scales (one per group) for: token embedding, wq[L], wk[L], wv[L], wo[L],
  w1[L], w2[L], w3[L] (and the classifier when it is not shared), with no padding.

Synthetic values (no real checkpoints exist here): weights N(0, 0.02) quantized per group of 32 (Q4_0: signed
absmax / -8, values clipped to [-8, 7]; Q8_0: absmax / 127), fp16 scales; norms 1; biases N(0, 0.02);
head_ids the sorted first head_k entries of a seeded permutation of the vocabulary.
"""
import os
import struct

import numpy as np

QWEN05B = dict(dim=896, hidden_dim=4864, n_layers=24, n_heads=14, n_kv_heads=2, vocab_size=151936, head_k=65536,
               max_seq_len=32768, group_size=32, emb_bits=8, rope_theta=1e6, rms_eps=1e-6)
# a small model with the same structure, for tests that must finish in seconds on the CPU oracle. qwen.c's
# matvec output buffer holds max(dim, hidden_dim) floats (qwen.c:295-300) and every head block writes
# min(head_k, 2048) of them, so head_k must not exceed hidden_dim here.
QWEN_TINY = dict(dim=128, hidden_dim=256, n_layers=2, n_heads=2, n_kv_heads=1, vocab_size=1000, head_k=256,
                 max_seq_len=256, group_size=32, emb_bits=8, rope_theta=1e6, rms_eps=1e-6)

STORIES15M = dict(dim=288, hidden_dim=768, n_layers=6, n_heads=6, n_kv_heads=6, vocab_size=32000, seq_len=256)
STORIES110M = dict(dim=768, hidden_dim=2048, n_layers=12, n_heads=12, n_kv_heads=12, vocab_size=32000, seq_len=1024)
RUNQ_TINY = dict(dim=64, hidden_dim=128, n_layers=2, n_heads=2, n_kv_heads=2, vocab_size=300, seq_len=64)

_HDR = "<4sI10i2f"


def _pad64(n):
    return (n + 63) & ~63


def q4_0(x):
    """Q4_0 per group of 32 along the last axis: int8 values in [-8, 7] and fp16 scales."""
    g = x.reshape(*x.shape[:-1], -1, 32)
    idx = np.abs(g).argmax(-1)[..., None]
    m = np.take_along_axis(g, idx, -1)[..., 0]
    d = (m / -8.0).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
    q = np.clip(np.rint(g * inv[..., None]), -8, 7).astype(np.int8)
    return q.reshape(x.shape), d


def q8_0(x, scale_dtype=np.float16):
    """Q8_0 per group of 32 along the last axis: int8 values and scales (fp16 by default)."""
    g = x.reshape(*x.shape[:-1], -1, 32)
    d = (np.abs(g).max(-1) / 127.0).astype(np.float16)
    df = d.astype(np.float32)
    inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
    q = np.clip(np.rint(g * inv[..., None]), -127, 127).astype(np.int8)
    return q.reshape(x.shape), d.astype(scale_dtype)


def pack4(q):
    """int8 values in [-8, 7] (rows of even length) -> packed nibbles, element 2i low (gguf2qwb.py:55-61)."""
    u = (q & 0x0F).astype(np.uint8)
    return u[..., 0::2] | (u[..., 1::2] << 4)


def unpack4(p):
    """packed nibbles -> int8 values, the inverse of pack4."""
    lo = (p & 0x0F).astype(np.int8)
    hi = (p >> 4).astype(np.int8)
    q = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), np.int8)
    q[..., 0::2] = np.where(lo > 7, lo - 16, lo)
    q[..., 1::2] = np.where(hi > 7, hi - 16, hi)
    return q


def qwb_size(cfg):
    L, dim, hid = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"]
    kv = dim // cfg["n_heads"] * cfg["n_kv_heads"]
    off = 256 + L * (3 * _pad64(dim * 4) + 2 * _pad64(kv * 4)) + _pad64(dim * 4) + _pad64(cfg["head_k"] * 4)
    mat = lambda d, n, bits: _pad64(d * n * bits // 8) + _pad64(d * n // 32 * 2)
    off += L * (2 * mat(dim, dim, 4) + 2 * mat(kv, dim, 4) + 3 * mat(hid, dim, 4))
    off += mat(cfg["head_k"], dim, 8) + mat(cfg["vocab_size"], dim, 8)
    return off


def write_synthetic_qwb(path, cfg=QWEN05B, seed=0, rows_per_chunk=8192):
    """Writes a seeded synthetic .qwb; returns its size. The same (cfg, seed) always gives the same bytes."""
    rng = np.random.default_rng(seed)
    L, dim, hid, vocab, hk = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"], cfg["vocab_size"], cfg["head_k"]
    kv = dim // cfg["n_heads"] * cfg["n_kv_heads"]
    head_ids = np.sort(rng.permutation(vocab)[:hk]).astype(np.int32)

    def put(f, a):
        b = np.ascontiguousarray(a).tobytes()
        f.write(b)
        f.write(b"\0" * (-len(b) % 64))

    def put_matrix(f, d, n, bits, src=None):
        # weights then scales, generated and written in row chunks to bound memory
        planes, scales = [], []
        for r0 in range(0, d, rows_per_chunk):
            r = min(rows_per_chunk, d - r0)
            x = src(r0, r) if src is not None else rng.standard_normal((r, n), np.float32) * np.float32(0.02)
            q, s = q4_0(x) if bits == 4 else q8_0(x)
            planes.append(pack4(q) if bits == 4 else q.view(np.uint8))
            scales.append(s)
        put(f, np.concatenate(planes))
        put(f, np.concatenate(scales))

    with open(path, "wb") as f:
        f.write(struct.pack(_HDR, b"QWB1", 1, dim, hid, L, cfg["n_heads"], cfg["n_kv_heads"], vocab, hk,
                            cfg["max_seq_len"], 32, 8, cfg["rope_theta"], cfg["rms_eps"]))
        f.write(b"\0" * (256 - f.tell()))
        for n in (dim, dim):
            for _ in range(L):
                put(f, np.ones(n, np.float32))
        for n in (dim, kv, kv):
            for _ in range(L):
                put(f, rng.standard_normal(n, np.float32) * np.float32(0.02))
        put(f, np.ones(dim, np.float32))
        put(f, head_ids)
        for d, n in ((dim, dim), (kv, dim), (kv, dim), (dim, dim), (hid, dim), (dim, hid), (hid, dim)):
            for _ in range(L):
                put_matrix(f, d, n, 4)
        # the embedding is drawn once (seeded, row-chunked); the head repeats its head_ids rows like gguf2qwb.py:106
        emb_seed = int(rng.integers(1 << 62))
        emb_rows = lambda r0, r: np.random.default_rng([emb_seed, r0]).standard_normal((r, dim), np.float32) * \
            np.float32(0.02)
        chunk = rows_per_chunk

        def head_rows(r0, r):
            ids = head_ids[r0:r0 + r]
            out = np.empty((r, dim), np.float32)
            for c in np.unique(ids // chunk):
                sel = (ids // chunk) == c
                block = emb_rows(int(c) * chunk, min(chunk, vocab - int(c) * chunk))
                out[sel] = block[ids[sel] - int(c) * chunk]
            return out

        put_matrix(f, hk, dim, 8, src=head_rows)
        put_matrix(f, vocab, dim, 8, src=emb_rows)
        size = f.tell()
    assert size == qwb_size(cfg), (size, qwb_size(cfg))
    return size


class Qwb:
    """A .qwb file as numpy views (qwen.c:211-271 walk). ``mats[name]`` is a list of (plane, scales) per layer."""

    def __init__(self, path):
        m = np.memmap(path, dtype=np.uint8, mode="r")
        magic, version, *ints = struct.unpack_from("<4sI10i", m[:48].tobytes())
        theta, eps = struct.unpack_from("<2f", m[48:56].tobytes())
        if magic != b"QWB1" or version != 1:
            raise ValueError(f"{path}: not a .qwb version 1 file")
        keys = ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "head_k", "max_seq_len",
                "group_size", "emb_bits")
        self.cfg = dict(zip(keys, ints), rope_theta=theta, rms_eps=eps)
        c = self.cfg
        if c["group_size"] != 32 or c["emb_bits"] != 8:
            raise ValueError(f"{path}: unsupported group size / embedding width")
        L, dim, hid = c["n_layers"], c["dim"], c["hidden_dim"]
        self.kv_dim = dim // c["n_heads"] * c["n_kv_heads"]
        self.m, self.off, self.offsets = m, 256, {}

        def vecs(name, n):
            self.offsets[name] = self.off
            a = self._take(L * n * 4).view(np.float32).reshape(L, n)
            return a

        self.attn_norm, self.ffn_norm = vecs("attn_norm", dim), vecs("ffn_norm", dim)
        self.bq, self.bk, self.bv = vecs("bq", dim), vecs("bk", self.kv_dim), vecs("bv", self.kv_dim)
        self.offsets["out_norm"] = self.off
        self.out_norm = self._take(dim * 4).view(np.float32)
        self.offsets["head_ids"] = self.off
        self.head_ids = self._take(c["head_k"] * 4).view(np.int32)
        self.mats = {}
        shapes = dict(wq=(dim, dim), wk=(self.kv_dim, dim), wv=(self.kv_dim, dim), wo=(dim, dim), w1=(hid, dim),
                      w2=(dim, hid), w3=(hid, dim))
        for name, (d, n) in shapes.items():
            self.mats[name] = [self._matrix(f"{name}.{l}", d, n, 4) for l in range(L)]
        self.head = self._matrix("head", c["head_k"], dim, 8)
        self.emb = self._matrix("emb", c["vocab_size"], dim, 8)
        if self.off != len(m):
            raise ValueError(f"{path}: size {len(m)}, header describes {self.off}")

    def _take(self, nbytes):
        a = self.m[self.off:self.off + nbytes]
        self.off += _pad64(nbytes)
        return a

    def _matrix(self, name, d, n, bits):
        self.offsets[name] = self.off
        w = self._take(d * n * bits // 8).reshape(d, n * bits // 8)
        self.offsets[name + ".s"] = self.off
        s = self._take(d * n // 32 * 2).view(np.uint16).reshape(d, n // 32)
        return w, s


def write_synthetic_runq(path, cfg=STORIES15M, seed=0, gs=32, shared=True):
    """Writes a seeded synthetic runq v2 Q8_0 file (fp16-rounded scales stored as fp32); returns its size."""
    rng = np.random.default_rng(seed)
    L, dim, hid, vocab = cfg["n_layers"], cfg["dim"], cfg["hidden_dim"], cfg["vocab_size"]
    hs = dim // cfg["n_heads"]
    kv = cfg["n_kv_heads"] * hs

    def q80(f, d, n):
        x = rng.standard_normal((d, n), np.float32) * np.float32(0.02)
        g = x.reshape(-1, gs)
        s = (np.abs(g).max(1) / 127.0).astype(np.float16).astype(np.float32)
        q = np.clip(np.rint(g / np.where(s == 0, 1, s)[:, None]), -127, 127).astype(np.int8)
        f.write(q.tobytes())
        f.write(s.tobytes())

    with open(path, "wb") as f:
        f.write(struct.pack("<Ii7iBi", 0x616B3432, 2, dim, hid, L, cfg["n_heads"], cfg["n_kv_heads"], vocab,
                            cfg["seq_len"], int(shared), gs))
        f.write(b"\0" * (256 - f.tell()))
        f.write(np.ones((2 * L + 1) * dim, np.float32).tobytes())
        q80(f, vocab, dim)
        for d, n in ((dim, dim), (kv, dim), (kv, dim), (dim, dim), (hid, dim), (dim, hid), (hid, dim)):
            for _ in range(L):
                q80(f, d, n)
        if not shared:
            q80(f, vocab, dim)
        return f.tell()


def cached_qwb(directory, cfg=QWEN05B, seed=0):
    """Path of a synthetic .qwb for (cfg, seed) under `directory`, written on first use."""
    tag = "qwen05b" if cfg is QWEN05B else "qwen_%dx%d" % (cfg["dim"], cfg["n_layers"])
    path = os.path.join(directory, f"{tag}_s{seed}.qwb")
    if not (os.path.exists(path) and os.path.getsize(path) == qwb_size(cfg)):
        os.makedirs(directory, exist_ok=True)
        tmp = path + ".tmp%d" % os.getpid()
        write_synthetic_qwb(tmp, cfg, seed)
        os.replace(tmp, path)
    return path
