"""The CPU restatement (oracle/matvec_oracle.c) against the reference's own outputs (tests/golden/*.npz, made by
tests/golden/make_golden.py from qwen.c and runq.c). Bit-exact everywhere: these are the pins that let the GPU
tests trust the restatement at sizes no fixture covers."""
import os

import numpy as np
import pytest

from conftest import ROOT, golden, golden_cases, load_pkg


def test_f16_table(restatement):
    ref = golden("f16_table.npz")["f32"]
    got = np.array([restatement.f16(h) for h in range(65536)], np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_quantize_qwen(restatement):
    z = golden("quantize.npz")
    for i in range(3):
        q, s = restatement.quantize_qwen(z[f"qwen{i}_x"])
        assert np.array_equal(q, z[f"qwen{i}_q"])
        assert np.array_equal(s.view(np.uint32), z[f"qwen{i}_s"].view(np.uint32))


@pytest.mark.parametrize("gs", [32, 64])
def test_quantize_runq(restatement, gs):
    z = golden("quantize.npz")
    for i in range(3):
        q, s = restatement.quantize_runq(z[f"runq{i}_g{gs}_x"], gs)
        assert np.array_equal(q, z[f"runq{i}_g{gs}_q"])
        assert np.array_equal(s.view(np.uint32), z[f"runq{i}_g{gs}_s"].view(np.uint32))


def test_matvec4_golden(restatement):
    for name, c in golden_cases("matvec4.npz").items():
        n, d, bits = int(c["n"]), int(c["d"]), int(c["bits"])
        isum = restatement.group_sums(c["w"], c["xq"], n, d, 32, bits)
        assert np.array_equal(isum, c["isum"]), name
        out = restatement.matvec_f16(c["w"], c["ws"], c["xq"], c["xs"], n, d, bits)
        assert np.array_equal(out.view(np.uint32), c["out"].view(np.uint32)), name


def test_matvec_runq_golden(restatement):
    for name, c in golden_cases("matvec.npz").items():
        n, d, gs = int(c["n"]), int(c["d"]), int(c["gs"])
        isum = restatement.group_sums(c["wq"].view(np.uint8), c["xq"], n, d, gs, 8)
        assert np.array_equal(isum, c["isum"]), name
        out = restatement.matvec_f32(c["wq"], c["ws"], c["xq"], c["xs"], n, d, gs)
        assert np.array_equal(out.view(np.uint32), c["out"].view(np.uint32)), name


def test_matvec4_tolerance_rule(restatement):
    """The reference testbench's own criterion (hls4/matvec4_tb.cpp:67-79): |out - ref_double| <= 1e-5 * sum|terms|.
    The sequential float sum meets it on every fixture row, special fp16 scales included."""
    f16 = golden("f16_table.npz")["f32"].astype(np.float64)
    for name, c in golden_cases("matvec4.npz").items():
        terms = c["isum"].astype(np.float64) * f16[c["ws"]] * c["xs"].astype(np.float64)[None, :]
        err = np.abs(c["out"].astype(np.float64) - terms.sum(1))
        assert np.all(err <= 1e-5 * np.abs(terms).sum(1) + 0.0), name


def test_synthetic_files_reproduce(tmp_path):
    """The seeded generators reproduce the exact files the end-to-end fixtures were made from."""
    import hashlib
    qwb = load_pkg().qwb
    tmp = str(tmp_path)
    z = golden("qwen_tiny.npz")
    p = os.path.join(tmp, "t_tiny.qwb")
    qwb.write_synthetic_qwb(p, qwb.QWEN_TINY, seed=int(z["seed"]))
    assert hashlib.sha256(open(p, "rb").read()).hexdigest() == str(z["sha256"])
    z = golden("runq_tiny.npz")
    p = os.path.join(tmp, "t_tiny_runq.bin")
    qwb.write_synthetic_runq(p, qwb.RUNQ_TINY, seed=int(z["seed"]), gs=int(z["gs"]))
    assert hashlib.sha256(open(p, "rb").read()).hexdigest() == str(z["sha256"])


def test_qwb_layout_size():
    qwb = load_pkg().qwb
    # qwen.c walks a Qwen2.5-0.5B .qwb with a 65,536-row head to 408,859,392 bytes
    assert qwb.qwb_size(qwb.QWEN05B) == 408_859_392


def test_pack4_roundtrip():
    qwb = load_pkg().qwb
    q = np.random.default_rng(0).integers(-8, 8, (7, 64)).astype(np.int8)
    assert np.array_equal(qwb.unpack4(qwb.pack4(q)), q)
