"""Generates the golden fixtures in this directory from the reference's own C code.

Run in a checkout that has the reference tree (REF, default the path oracle/Makefile uses): it builds
oracle/_ref/ (qwen/qwen.c and runq/runq.c compiled unchanged) and calls their quantize(), matmul_cpu(), f16()
and forward() through oracle/oracle.py. Inputs follow the reference testbenches' recipes:
  * hls4/matvec4_tb.cpp:52-59, 88-99: random weight bytes, fp16 scales with random sign, exponent 5..10 and
    random mantissa (or exponent field row % 31 for the "special" rows: zero, subnormals up to 65504),
    xq uniform in [-128, 127], xs uniform in [1e-3, 1e-1]; shapes of :141-147 (quick set, plus the two
    special-scale shapes).
  * hls/matvec_tb.cpp:56-62, 90-93: int8 wq and xq uniform in [-128, 127], ws uniform in [1e-4, 2e-2],
    xs uniform in [1e-3, 1e-1]; the testbench shapes that keep the fixture small.
Per-group int32 sums come from the reference too: matmul_cpu() over one group's columns with unit scales
returns (float)isum exactly (|isum| < 2^24).

usage: python tests/golden/make_golden.py
"""
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "local-llama-pynq-z2_b200"))
import oracle  # noqa: E402
import qwb  # noqa: E402

SEED = 20261201


def hls4_mat(rng, n, d, bits, special=False):
    w = rng.integers(0, 256, d * n * bits // 8, dtype=np.uint8).reshape(d, n * bits // 8)
    ng = n // 32
    e = (np.arange(d * ng) // ng % 31) if special else rng.integers(5, 11, d * ng)
    s = (rng.integers(0, 2, d * ng) << 15) | (e << 10) | rng.integers(0, 1024, d * ng)
    return w, s.astype(np.uint16).reshape(d, ng)


def matvec4_case(ref, rng, n, d, bits, special=False):
    w, ws = hls4_mat(rng, n, d, bits, special)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
    out = ref.matmul_cpu(w, ws, xq, xs, n, d, bits)
    gb = 32 * bits // 8  # bytes of one group in a row
    one = np.full((d, 1), 0x3C00, np.uint16)  # fp16 1.0
    isum = np.stack([ref.matmul_cpu(np.ascontiguousarray(w[:, g * gb:(g + 1) * gb]), one,
                                    np.ascontiguousarray(xq[g * 32:(g + 1) * 32]), np.ones(1, np.float32), 32, d, bits)
                     for g in range(n // 32)], axis=1)
    return dict(w=w, ws=ws, xq=xq, xs=xs, out=out, isum=isum.astype(np.int32), n=n, d=d, bits=bits)


def matvec_case(ref, rng, n, d, gs):
    wq = rng.integers(-128, 128, d * n).astype(np.int8).reshape(d, n)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    ws = rng.uniform(1e-4, 2e-2, d * n // gs).astype(np.float32).reshape(d, n // gs)
    xs = rng.uniform(1e-3, 1e-1, n // gs).astype(np.float32)
    out = ref.matmul_cpu(wq, ws, xq, xs, n, d, gs)
    one = np.ones((d, 1), np.float32)
    isum = np.stack([ref.matmul_cpu(np.ascontiguousarray(wq[:, g * gs:(g + 1) * gs]), one,
                                    np.ascontiguousarray(xq[g * gs:(g + 1) * gs]), np.ones(1, np.float32), gs, d, gs)
                     for g in range(n // gs)], axis=1)
    return dict(wq=wq, ws=ws, xq=xq, xs=xs, out=out, isum=isum.astype(np.int32), n=n, d=d, gs=gs)


def quant_inputs(rng):
    """Activation vectors for quantize(): N(0, 1) at the model widths, and one with edge groups."""
    edge = rng.standard_normal(256).astype(np.float32)
    edge[0:32] = 0.0  # all-zero group (qwen.c guards it; runq.c divides 0 by 0)
    edge[32:64] = np.float32(127.0) * (np.arange(32, dtype=np.float32) - 16) / 16  # exact halves after scaling
    edge[64:96] = np.float32(1e-40) * np.arange(1, 33, dtype=np.float32)  # subnormal inputs
    edge[96:128] = rng.standard_normal(32).astype(np.float32) * np.float32(3e4)  # large magnitudes
    edge[128:160] = -np.abs(edge[128:160])  # a negative-only group
    return [rng.standard_normal(896).astype(np.float32), rng.standard_normal(4864).astype(np.float32), edge]


def main():
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all", "ref"], check=True)
    rq, rr = oracle.RefQwen(), oracle.RefRunq()
    rng = np.random.default_rng(SEED)

    # fp16 -> fp32 of every bit pattern (qwen.c:84-94)
    f16 = np.array([rq.f16(h) for h in range(65536)], np.float32)
    np.savez_compressed(os.path.join(HERE, "f16_table.npz"), f32=f16)

    # activation quantization (qwen.c:355-364; runq.c:244-270 at gs 32 and 64)
    qd = {}
    for i, x in enumerate(quant_inputs(rng)):
        q, s = rq.quantize(x)
        qd[f"qwen{i}_x"], qd[f"qwen{i}_q"], qd[f"qwen{i}_s"] = x, q, s
        for gs in (32, 64):
            q, s = rr.quantize(x, gs)
            qd[f"runq{i}_g{gs}_x"], qd[f"runq{i}_g{gs}_q"], qd[f"runq{i}_g{gs}_s"] = x, q, s
    np.savez_compressed(os.path.join(HERE, "quantize.npz"), **qd)

    # matvec4 (qwen.c matmul_cpu): hls4 testbench quick shapes (n, d, wbits) plus the special-scale shapes
    cases = {}
    for (n, d, bits) in ((96, 5, 4), (96, 5, 8), (896, 128, 4), (896, 64, 8), (4864, 32, 4), (8192, 4, 4)):
        cases[f"q_{n}x{d}_w{bits}"] = matvec4_case(rq, rng, n, d, bits)
    for bits in (4, 8):
        cases[f"special_64x31_w{bits}"] = matvec4_case(rq, rng, 64, 31, bits, special=True)
    np.savez_compressed(os.path.join(HERE, "matvec4.npz"),
                        **{f"{k}.{f}": v for k, c in cases.items() for f, v in c.items()})

    # matvec (runq.c matmul): hls testbench shapes (n, d, gs) small enough for a fixture
    cases = {}
    for (n, d, gs) in ((96, 7, 32), (288, 288, 32), (288, 96, 32), (768, 64, 64), (2048, 16, 64), (8192, 3, 32)):
        cases[f"r_{n}x{d}_g{gs}"] = matvec_case(rr, rng, n, d, gs)
    np.savez_compressed(os.path.join(HERE, "matvec.npz"),
                        **{f"{k}.{f}": v for k, c in cases.items() for f, v in c.items()})

    # end to end: a tiny Qwen2-structured .qwb through qwen.c forward (prompt fed token by token, greedy)
    tmp = tempfile.mkdtemp()
    path = os.path.join(tmp, "golden_tiny.qwb")
    qwb.write_synthetic_qwb(path, qwb.QWEN_TINY, seed=11)
    digest = hashlib.sha256(open(path, "rb").read()).hexdigest()
    prompt = [int(t) for t in np.random.default_rng(12).integers(0, qwb.QWEN_TINY["vocab_size"], 6)]
    rq.open(path, 64)
    ids, logits = rq.greedy(prompt, 10)
    np.savez_compressed(os.path.join(HERE, "qwen_tiny.npz"), sha256=np.array(digest), seed=11, prompt=prompt,
                        ids=np.array(ids, np.int32), logits=logits, ctx=64)

    # end to end: a tiny runq v2 file through runq.c forward
    path = os.path.join(tmp, "golden_tiny_runq.bin")
    qwb.write_synthetic_runq(path, qwb.RUNQ_TINY, seed=13, gs=32)
    digest = hashlib.sha256(open(path, "rb").read()).hexdigest()
    prompt = [int(t) for t in np.random.default_rng(14).integers(3, qwb.RUNQ_TINY["vocab_size"], 4)]
    rr.open(path)
    ids, logits = rr.greedy(prompt, 12)
    np.savez_compressed(os.path.join(HERE, "runq_tiny.npz"), sha256=np.array(digest), seed=13, gs=32,
                        prompt=prompt, ids=np.array(ids, np.int32), logits=logits)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
