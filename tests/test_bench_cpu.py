"""bench.py's CPU side without a GPU: the reference arm of the isolated sweep (--impl reference --mode sweep) times
the reference's own matmul_cpu (qwen.c:436-456) and runq matmul (runq.c:430-458) through timing loops in the
oracle harnesses. Checks that those loops compute what the plain calls compute on the last copy they read, and that
the sweep prints well-formed lines."""
import ctypes as C
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

import oracle

needs_ref = pytest.mark.skipif(not (oracle.ref_available("libref_qwen.so") and oracle.ref_available("libref_runq.so")),
                               reason="oracle/_ref not built (the reference tree was absent at build time)")


def _timer(lib, name):
    fn = getattr(lib, name)
    fn.restype = C.c_double
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_int, C.c_void_p, C.c_void_p,
                   C.c_int, C.c_int, C.c_int, C.c_int]
    return fn


@needs_ref
@pytest.mark.parametrize("bits", [4, 8])
def test_qwen_timing_loop_matches_matmul_cpu(bits):
    ref = oracle.RefQwen()
    rng = np.random.default_rng(5)
    n, d, copies, reps = 896, 40, 3, 5  # the last call reads copy (reps - 1) % copies = 1
    wbytes, ng = d * n * bits // 8, d * n // 32
    w = rng.integers(0, 256, copies * wbytes, dtype=np.uint8)
    s = (rng.random(copies * ng) * 0.019 + 0.001).astype(np.float16).view(np.uint16)
    xq, xs = ref.quantize(rng.standard_normal(n).astype(np.float32))
    out = np.full(d, np.nan, np.float32)
    t = _timer(ref.lib, "ref_qwen_time_matmul_cpu")(out.ctypes.data, w.ctypes.data, s.ctypes.data, wbytes, ng,
                                                    copies, xq.ctypes.data, xs.ctypes.data, n, d, bits, reps)
    assert t > 0
    want = ref.matmul_cpu(w[wbytes:2 * wbytes], s[ng:2 * ng], xq, xs, n, d, bits)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("gs", [32, 64])
def test_runq_timing_loop_matches_matmul(gs):
    ref = oracle.RefRunq()
    rng = np.random.default_rng(6)
    n, d, copies, reps = 768, 24, 2, 4  # the last call reads copy 1
    ng = d * n // gs
    wq = rng.integers(-127, 128, copies * d * n, dtype=np.int8)
    ws = (rng.random(copies * ng) * 0.019 + 0.001).astype(np.float32)
    xq, xs = ref.quantize(rng.standard_normal(n).astype(np.float32), gs)
    out = np.full(d, np.nan, np.float32)
    t = _timer(ref.lib, "ref_runq_time_matmul_cpu")(out.ctypes.data, wq.ctypes.data, ws.ctypes.data, d * n, ng,
                                                    copies, xq.ctypes.data, xs.ctypes.data, n, d, gs, reps)
    assert t > 0
    want = ref.matmul_cpu(wq[d * n:], ws[ng:], xq, xs, n, d, gs)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


@needs_ref
def test_reference_sweep_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--mode", "sweep",
                        "--only", "128x896"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.strip().splitlines()]
    summary = lines[-1]
    assert summary["mode"] == "sweep" and summary["impl"] == "reference"
    assert summary["cores"] == os.cpu_count()
    (res,) = summary["results"]
    assert res["shape"] == "128x896 Q4" and res["us"] > 0 and res["GBps"] > 0
    assert res["bytes"] == 128 * 448 + 128 * 28 * 2 + 896 + 28 * 4 + 4 * 128


@needs_ref
def test_reference_arm_line_keeps_the_contract():
    """`bench.py --impl reference` (the driver's reference arm): one JSON line with BASELINE.json's metric, the
    reference's own qwen.c timed on the host cores, and its cpu_baseline / e2e objects."""
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    base = json.load(open(os.path.join(ROOT, "BASELINE.json")))
    assert line["impl"] == "reference" and line["metric"] == base["metric"]
    assert line["unit"] == "tok/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["n_gpus"] == 1 and line["config"]["workload"]
    # the same config object and step count as the decode line of bench.py's own arm
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert line["config"] == bench.decode_config(1)
    assert line["steps"] == 1 and line["warmup"] == 1
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] == os.cpu_count() and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun only rank 0 runs the reference arm; the other ranks exit 0 without work or output."""
    env = dict(os.environ, RANK="1", LOCAL_RANK="1", WORLD_SIZE="2")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2"],
                       capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_prefill_shapes_by_name():
    """--mode prefill --only: config 4's shapes by rows x columns, any other shape as rows x columns (Q4 unless qN
    follows), nothing for a malformed name."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench.prefill_shapes("") == bench.PREFILL_SHAPES
    assert bench.prefill_shapes("4864x896") == [(896, 4864, 4)]
    assert bench.prefill_shapes("65536x896") == [(896, 65536, 8)]
    assert bench.prefill_shapes("8192x8192") == [(8192, 8192, 4)]
    assert bench.prefill_shapes("1000x896q8") == [(896, 1000, 8)]
    assert bench.prefill_shapes("banana") == []
