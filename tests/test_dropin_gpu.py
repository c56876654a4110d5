"""The drop-in gate: the reference's own hosts, compiled unchanged with -DFPGA against include/matvec_fpga.h and
linked with libmatvec_b200.so (oracle/Makefile `ref-b200`), against the same hosts' CPU builds. Both builds
share every host-side instruction; only the matvec backend differs. The bar is bit-identical logits at every
position and identical greedy token ids.

Needs oracle/_ref/ (built where the reference tree is available; it travels with the working tree)."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, golden, load_pkg

pytestmark = pytest.mark.gpu
REF = os.path.join(ROOT, "oracle", "_ref")


def need(*names):
    missing = [n for n in names if not os.path.exists(os.path.join(REF, n))]
    if missing:
        pytest.fail(f"oracle/_ref is missing {missing}: run make -C oracle ref ref-b200 where the reference exists")


def run_qwen(binary, model, ids, n, ctx, dump, threads=None):
    env = dict(os.environ)
    if threads:
        env["OMP_NUM_THREADS"] = str(threads)
    r = subprocess.run([os.path.join(REF, binary), model, "--ids", ",".join(map(str, ids)), "-t", "0", "-n", str(n),
                        "-c", str(ctx), "--logits", dump], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr
    return [int(t) for t in r.stdout.strip().split(",") if t], r.stderr


def test_qwen_tiny_matches_golden_and_cpu(tmp_path):
    need("qwen", "qwen_b200")
    qwb = load_pkg().qwb
    z = golden("qwen_tiny.npz")
    model = str(tmp_path / "tiny.qwb")
    qwb.write_synthetic_qwb(model, qwb.QWEN_TINY, seed=int(z["seed"]))
    prompt, n = [int(t) for t in z["prompt"]], len(z["ids"])
    ids_gpu, err = run_qwen("qwen_b200", model, prompt, n, int(z["ctx"]), str(tmp_path / "gpu.bin"))
    ids_cpu, _ = run_qwen("qwen", model, prompt, n, int(z["ctx"]), str(tmp_path / "cpu.bin"))
    gpu = np.fromfile(tmp_path / "gpu.bin", np.float32)
    cpu = np.fromfile(tmp_path / "cpu.bin", np.float32)
    assert ids_gpu == ids_cpu == [int(t) for t in z["ids"]]
    assert np.array_equal(gpu.view(np.uint32), cpu.view(np.uint32))
    assert np.array_equal(gpu.view(np.uint32), z["logits"].reshape(-1).view(np.uint32))


def test_qwen05b_logits_bit_identical(tmp_path, data_dir):
    """Qwen2.5-0.5B-shaped synthetic .qwb (390 MiB, Q4 layers, 65,536-row Q8 head) through qwen.c: 200
    fpga_matvec4 calls per token, every logit of every position bit-identical to the CPU build."""
    need("qwen", "qwen_b200")
    qwb = load_pkg().qwb
    model = qwb.cached_qwb(data_dir, qwb.QWEN05B, seed=0)
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, 151936, 12)]
    ids_gpu, err = run_qwen("qwen_b200", model, prompt, 12, 64, str(tmp_path / "gpu.bin"))
    ids_cpu, _ = run_qwen("qwen", model, prompt, 12, 64, str(tmp_path / "cpu.bin"))
    gpu = np.fromfile(tmp_path / "gpu.bin", np.float32)
    cpu = np.fromfile(tmp_path / "cpu.bin", np.float32)
    assert gpu.size == cpu.size == 65536 * (len(prompt) + len(ids_cpu) - 1)
    assert ids_gpu == ids_cpu
    assert np.array_equal(gpu.view(np.uint32), cpu.view(np.uint32))


def test_runq_tiny_matches_golden_and_cpu(tmp_path):
    """runq.c's -DFPGA matmul through fpga_matvec (int8, fp32 scales) against its CPU build and the fixture."""
    need("libref_runq.so", "libref_runq_b200.so")
    code = r"""
import sys, numpy as np
sys.path.insert(0, %(oracle)r)
import oracle
r = oracle.RefRunq(b200=%(b200)s)
r.open(%(model)r)
ids, logits = r.greedy(%(prompt)r, %(npos)d)
np.save(%(out)r, logits)
print(",".join(map(str, ids)))
"""
    qwb = load_pkg().qwb
    z = golden("runq_tiny.npz")
    model = str(tmp_path / "tiny_runq.bin")
    qwb.write_synthetic_runq(model, qwb.RUNQ_TINY, seed=int(z["seed"]), gs=int(z["gs"]))
    prompt = [int(t) for t in z["prompt"]]
    res = {}
    for b200 in (False, True):
        out = str(tmp_path / f"runq_{b200}.npy")
        src = code % dict(oracle=os.path.join(ROOT, "oracle"), b200=b200, model=model, prompt=prompt, npos=12, out=out)
        r = subprocess.run(["python", "-c", src], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr
        res[b200] = (r.stdout.strip(), np.load(out))
    assert res[True][0] == res[False][0] == ",".join(map(str, z["ids"]))
    assert np.array_equal(res[True][1].view(np.uint32), res[False][1].view(np.uint32))
    assert np.array_equal(res[True][1].view(np.uint32), z["logits"].view(np.uint32))


def test_runq_stories15m_bit_identical(tmp_path):
    """Config 1's architecture (stories15M, gs 32) through runq.c forward: every logit bit-identical to the CPU
    build for 24 positions."""
    need("libref_runq.so", "libref_runq_b200.so")
    qwb = load_pkg().qwb
    model = str(tmp_path / "s15m.bin")
    qwb.write_synthetic_runq(model, qwb.STORIES15M, seed=3, gs=32)
    prompt = [int(t) for t in np.random.default_rng(4).integers(3, 32000, 4)]
    code = r"""
import sys, numpy as np
sys.path.insert(0, %(oracle)r)
import oracle
r = oracle.RefRunq(b200=%(b200)s)
r.open(%(model)r)
ids, logits = r.greedy(%(prompt)r, 24)
np.save(%(out)r, logits)
print(",".join(map(str, ids)))
"""
    res = {}
    for b200 in (False, True):
        out = str(tmp_path / f"s15_{b200}.npy")
        src = code % dict(oracle=os.path.join(ROOT, "oracle"), b200=b200, model=model, prompt=prompt, out=out)
        r = subprocess.run(["python", "-c", src], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr
        res[b200] = (r.stdout.strip(), np.load(out))
    assert res[True][0] == res[False][0]
    assert np.array_equal(res[True][1].view(np.uint32), res[False][1].view(np.uint32))


def test_fpga_abi_host_buffers(mvb):
    """The reference's calling pattern through the Python mirror: weights and activations carved out of
    fpga_alloc() buffers at 64-byte offsets, written through the host pointer, results read back from it."""
    restatement = __import__("oracle").Restatement()
    assert mvb.fpga_open() == 0
    assert mvb.fpga_open() == 0  # idempotent
    try:
        rng = np.random.default_rng(2)
        n, d = 896, 4864
        w = rng.integers(0, 256, (d, n // 2), dtype=np.uint8)
        ws = ((rng.integers(0, 2, d * 28) << 15) | (rng.integers(5, 11, d * 28) << 10) |
              rng.integers(0, 1024, d * 28)).astype(np.uint16)
        xq = rng.integers(-128, 128, n).astype(np.int8)
        xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
        pad = lambda b: (b + 63) & ~63
        off_ws = pad(w.nbytes)
        wbuf, wphys = mvb.fpga_alloc(off_ws + pad(ws.nbytes))
        wbuf[:w.nbytes] = w.reshape(-1)
        wbuf[off_ws:off_ws + ws.nbytes] = ws.view(np.uint8)
        abuf, aphys = mvb.fpga_alloc(8192 + 256 * 4 + 8192 * 4)
        xs_off, out_off = 8192, 8192 + 1024
        for trial in range(3):  # activations change every call; weights stay resident after the first
            xq = rng.integers(-128, 128, n).astype(np.int8)
            abuf[:n] = xq.view(np.uint8)
            abuf[xs_off:xs_off + xs.nbytes] = xs.view(np.uint8)
            assert mvb.fpga_matvec4(wphys, wphys + off_ws, aphys, aphys + xs_off, aphys + out_off, n, d, 4) == 0
            out = abuf[out_off:out_off + 4 * d].view(np.float32)
            ref = restatement.matvec_f16(w, ws, xq, xs, n, d, 4)
            assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), trial
        # the reference driver's rejections (cpp:212-216) and addresses outside every buffer
        assert mvb.fpga_matvec4(wphys + 8, wphys + off_ws, aphys, aphys + xs_off, aphys + out_off, n, d, 4) == -1
        assert mvb.fpga_matvec4(wphys, wphys + off_ws, aphys, aphys + xs_off, aphys + out_off, 8224, d, 4) == -1
        assert mvb.fpga_matvec4(wphys, wphys + off_ws, aphys, aphys + xs_off, aphys + out_off, n, d, 3) == -1
        assert mvb.fpga_matvec4(wphys, wphys + off_ws, aphys, aphys + xs_off, 1 << 40, n, d, 4) == -1
        assert "not inside a buffer" in mvb.last_error() or "aligned" in mvb.last_error()
        assert mvb.fpga_matvec(wphys, wphys, aphys, aphys, aphys + out_off, 288, 4, 48) == -1
    finally:
        mvb.fpga_close()
        mvb.fpga_close()  # safe twice


def test_fpga_matvec_any_int8_alignment(mvb):
    """fpga_matvec (runq's int8 path) takes its int8 weights and activations at any byte address, as the reference
    driver does (driver/matvec_fpga.cpp:178 checks no alignment): planes at odd offsets inside the fpga_alloc()
    buffers give the restatement's result bit for bit, over repeated calls (the aligned device copy of a misaligned
    weight range is made once). fp32 arrays off their 4-byte alignment are refused."""
    restatement = __import__("oracle").Restatement()
    assert mvb.fpga_open() == 0
    try:
        rng = np.random.default_rng(5)
        for n, d, gs, wo, xo in ((288, 768, 32, 1, 3), (768, 288, 64, 7, 13), (2048, 96, 32, 3, 1)):
            wq = rng.integers(-127, 128, (d, n), dtype=np.int8)
            ws = rng.uniform(1e-3, 2e-2, d * n // gs).astype(np.float32)
            off_ws = (wo + wq.nbytes + 63) & ~63
            wbuf, wphys = mvb.fpga_alloc(off_ws + ws.nbytes)
            wbuf[wo:wo + wq.nbytes] = wq.view(np.uint8).reshape(-1)
            wbuf[off_ws:off_ws + ws.nbytes] = ws.view(np.uint8)
            abuf, aphys = mvb.fpga_alloc(16384 + 4 * d)
            xs_off, out_off = 8192 + 64, 12288
            for trial in range(2):
                x = rng.standard_normal(n).astype(np.float32)
                xq, xs = restatement.quantize_runq(x, gs)
                abuf[xo:xo + n] = xq.view(np.uint8)
                abuf[xs_off:xs_off + xs.nbytes] = xs.view(np.uint8)
                assert mvb.fpga_matvec(wphys + wo, wphys + off_ws, aphys + xo, aphys + xs_off, aphys + out_off,
                                       n, d, gs) == 0, mvb.last_error()
                out = abuf[out_off:out_off + 4 * d].view(np.float32)
                ref = restatement.matvec_f32(wq, ws, xq, xs, n, d, gs)
                assert np.array_equal(out.view(np.uint32), ref.view(np.uint32)), (n, d, gs, trial)
        assert mvb.fpga_matvec(wphys + wo, wphys + off_ws + 2, aphys + xo, aphys + xs_off, aphys + out_off,
                               n, d, gs) == -1
        assert "4-byte aligned" in mvb.last_error()
    finally:
        mvb.fpga_close()


def test_fpga_stats_line():
    """MATVEC_STATS=1: fpga_close() prints the mean per-call split as one JSON line on stderr, over the calls that
    uploaded no weights (here: five calls on resident weights after the first, which uploads them)."""
    code = r"""
import sys, numpy as np
sys.path.insert(0, %(root)r)
from conftest import load_pkg
mvb = load_pkg()
assert mvb.fpga_open() == 0
n, d = 896, 896
wbuf, wphys = mvb.fpga_alloc(d * n // 2 + d * 28 * 2 + 64)
rng = np.random.default_rng(0)
wbuf[: d * n // 2] = rng.integers(0, 256, d * n // 2, dtype=np.uint8)
off = (d * n // 2 + 63) & ~63
wbuf[off: off + d * 56] = np.full(d * 28, 0x2000, np.uint16).view(np.uint8)
abuf, aphys = mvb.fpga_alloc(8192)
abuf[:n] = rng.integers(-128, 128, n, dtype=np.int8).view(np.uint8)
abuf[1024: 1024 + 112] = np.full(28, 0.01, np.float32).view(np.uint8)
for _ in range(6):
    assert mvb.fpga_matvec4(wphys, wphys + off, aphys, aphys + 1024, aphys + 2048, n, d, 4) == 0
mvb.fpga_close()
""" % dict(root=os.path.join(ROOT, "tests"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, MATVEC_STATS="1"))
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stderr.splitlines() if l.startswith("matvec stats: ")]
    assert len(line) == 1, r.stderr[-2000:]
    stats = json.loads(line[0][len("matvec stats: "):])
    assert stats["calls"] == 5 and stats["calls_with_weight_upload"] == 1
    assert stats["us_per_call"] > 0 and stats["kernel_us"] > 0
