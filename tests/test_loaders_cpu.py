"""The decode loaders' checks without a GPU (mvb_qwen_load / mvb_runq_load and their _file forms): a malformed or
unsupported model file is refused with a message before any device is touched, the way runq.c:322-337 and
qwen.c:223-262 refuse theirs. No device call runs here."""
import ctypes as C
import struct

import numpy as np
import pytest

from conftest import load_pkg


def load(fn, data, ctx=32):
    mvb = load_pkg()
    buf = np.frombuffer(bytes(data), np.uint8) if len(data) else np.zeros(1, np.uint8)
    h = getattr(mvb.lib(), fn)(buf.ctypes.data if len(data) else None, len(data), ctx)
    return h, mvb.last_error()


@pytest.fixture(scope="module")
def runq_tiny(tmp_path_factory):
    mvb = load_pkg()
    p = tmp_path_factory.mktemp("loaders") / "tiny_runq.bin"
    mvb.qwb.write_synthetic_runq(str(p), mvb.qwb.RUNQ_TINY, seed=1, gs=32)
    return p.read_bytes()


def header(data, **fields):
    """data with runq v2 header fields replaced (runq.c:322-336 layout)."""
    b = bytearray(data)
    keys = ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "vocab_size", "seq_len")
    for k, v in fields.items():
        if k == "magic":
            struct.pack_into("<I", b, 0, v)
        elif k == "version":
            struct.pack_into("<i", b, 4, v)
        elif k == "gs":
            struct.pack_into("<i", b, 37, v)
        else:
            struct.pack_into("<i", b, 8 + 4 * keys.index(k), v)
    return bytes(b)


def test_runq_rejects_bad_headers(runq_tiny):
    for data, msg in ((b"", "not a runq version 2"), (runq_tiny[:255], "not a runq version 2"),
                      (header(runq_tiny, magic=0x12345678), "not a runq version 2"),
                      (header(runq_tiny, version=1), "not a runq version 2"),
                      (header(runq_tiny, gs=16), "group size 32 or 64"),
                      (header(runq_tiny, gs=48), "group size 32 or 64"),
                      (header(runq_tiny, n_heads=3), "head size"),           # 64 / 3 does not divide
                      (header(runq_tiny, n_heads=4), "head size"),           # head size 16
                      (header(runq_tiny, n_kv_heads=3), "unsupported config"),  # 2 % 3
                      (header(runq_tiny, dim=4096, n_heads=64), "dim <="),
                      (header(runq_tiny, n_layers=0), "unsupported config"),
                      (runq_tiny[:-1], "header describes")):
        h, err = load("mvb_runq_load", data)
        assert not h, msg
        assert msg in err, (msg, err)


def test_runq_context_limits(runq_tiny):
    h, err = load("mvb_runq_load", runq_tiny, ctx=1)
    assert not h and "context" in err


def test_qwen_rejects_bad_images(runq_tiny, tmp_path):
    mvb = load_pkg()
    h, err = load("mvb_qwen_load", runq_tiny)
    assert not h and "not a .qwb version 1" in err
    p = tmp_path / "tiny.qwb"
    mvb.qwb.write_synthetic_qwb(str(p), mvb.qwb.QWEN_TINY, seed=2)
    data = p.read_bytes()
    h, err = load("mvb_qwen_load", data[:-64])
    assert not h and "header describes" in err
    bad = bytearray(data)
    struct.pack_into("<i", bad, 8 + 4 * 3, 3)  # n_heads 3: 128 / 3 does not divide
    h, err = load("mvb_qwen_load", bytes(bad))
    assert not h and "unsupported config" in err
    h, err = load("mvb_runq_load", data)
    assert not h and "not a runq version 2" in err


def test_file_loaders_report_missing_files(tmp_path):
    mvb = load_pkg()
    for fn in ("mvb_qwen_load_file", "mvb_runq_load_file"):
        h = getattr(mvb.lib(), fn)(str(tmp_path / "missing.bin").encode(), 32)
        assert not h
        assert "cannot map" in mvb.last_error()
    assert not mvb.lib().mvb_runq_load_file(None, 32)
