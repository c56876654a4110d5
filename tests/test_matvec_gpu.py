"""Parity of the sm_100a matvec kernels with the reference, on a B200. Every comparison is bit-exact: int32 group
sums, fp32 outputs (compared as bit patterns) and quantized activations.

  * golden fixtures (tests/golden, made from qwen.c / runq.c themselves) through the device-pointer API and
    through the reference-facing fpga_* ABI with host buffers;
  * the pinned C restatement at the reference's model shapes, the trimmed and full heads, n = 8192 and ragged d;
  * the fused activation-quantization prologue against the reference's quantize() of qwen.c and runq.c;
  * argument validation: the reference driver's rejections return -1, never a fault.
"""
import numpy as np
import pytest

from conftest import golden, golden_cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "a CUDA device is required"
    t.cuda.set_device(0)
    return t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_matvec4(mvb, torch, w, ws, xq, xs, n, d, bits):
    out = torch.full((d,), float("nan"), device="cuda")
    mvb.matvec4(dev(torch, w), dev(torch, ws.view(np.int16)), dev(torch, xq), dev(torch, xs), out, n, d, bits)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def run_matvec(mvb, torch, wq, ws, xq, xs, n, d, gs):
    out = torch.full((d,), float("nan"), device="cuda")
    mvb.matvec(dev(torch, wq), dev(torch, ws), dev(torch, xq), dev(torch, xs), out, n, d, gs)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def test_matvec4_golden(mvb, torch):
    for name, c in golden_cases("matvec4.npz").items():
        n, d, bits = int(c["n"]), int(c["d"]), int(c["bits"])
        out = run_matvec4(mvb, torch, c["w"], c["ws"], c["xq"], c["xs"], n, d, bits)
        assert same_bits(out, c["out"]), name


def test_matvec_runq_golden(mvb, torch):
    for name, c in golden_cases("matvec.npz").items():
        n, d, gs = int(c["n"]), int(c["d"]), int(c["gs"])
        out = run_matvec(mvb, torch, c["wq"], c["ws"], c["xq"], c["xs"], n, d, gs)
        assert same_bits(out, c["out"]), name


def test_group_sums_exact(mvb, torch):
    """Per-group int32 sums: one group's columns with unit scales make the kernel output (float)isum."""
    one16 = np.full(1, 0x3C00, np.uint16)
    for name, c in golden_cases("matvec4.npz").items():
        n, d, bits = int(c["n"]), int(c["d"]), int(c["bits"])
        gb = 32 * bits // 8
        for g in range(min(n // 32, 6)):
            w = np.ascontiguousarray(c["w"][:, g * gb:(g + 1) * gb])
            out = run_matvec4(mvb, torch, w, np.repeat(one16, d), c["xq"][g * 32:(g + 1) * 32], np.ones(1, np.float32),
                              32, d, bits)
            assert np.array_equal(out.astype(np.int64), c["isum"][:, g]), (name, g)
    for name, c in golden_cases("matvec.npz").items():
        n, d, gs = int(c["n"]), int(c["d"]), int(c["gs"])
        for g in range(min(n // gs, 6)):
            wq = np.ascontiguousarray(c["wq"][:, g * gs:(g + 1) * gs])
            out = run_matvec(mvb, torch, wq, np.ones(d, np.float32), c["xq"][g * gs:(g + 1) * gs],
                             np.ones(1, np.float32), gs, d, gs)
            assert np.array_equal(out.astype(np.int64), c["isum"][:, g]), (name, g)


def _random_q(rng, n, d, bits, scale_kind="qwen"):
    w = rng.integers(0, 256, d * n * bits // 8, dtype=np.uint8).reshape(d, -1)
    if scale_kind == "special":
        e = np.arange(d * (n // 32)) // (n // 32) % 31
    else:
        e = rng.integers(5, 11, d * (n // 32))
    ws = ((rng.integers(0, 2, e.size) << 15) | (e << 10) | rng.integers(0, 1024, e.size)).astype(np.uint16)
    return w, ws.reshape(d, n // 32)


@pytest.mark.parametrize("n,d,bits", [(896, 896, 4), (896, 128, 4), (896, 4864, 4), (4864, 896, 4),
                                      (896, 2048, 8), (896, 1, 4), (32, 7, 4), (8192, 5, 4), (8192, 3, 8),
                                      (4864, 33, 8), (96, 5, 4)])
def test_matvec4_vs_restatement(mvb, torch, restatement, n, d, bits):
    rng = np.random.default_rng(n * 7 + d + bits)
    w, ws = _random_q(rng, n, d, bits)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
    out = run_matvec4(mvb, torch, w, ws, xq, xs, n, d, bits)
    assert same_bits(out, restatement.matvec_f16(w, ws, xq, xs, n, d, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_special_scales_all_exponents(mvb, torch, restatement, bits):
    """Row i's scales all have exponent field i % 31 (zero, subnormals ... 65504), as hls4/matvec4_tb.cpp:95."""
    rng = np.random.default_rng(bits)
    n, d = 256, 93
    w, ws = _random_q(rng, n, d, bits, "special")
    xq = rng.integers(-128, 128, n).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
    assert same_bits(run_matvec4(mvb, torch, w, ws, xq, xs, n, d, bits),
                     restatement.matvec_f16(w, ws, xq, xs, n, d, bits))


def test_heads_row_subset(mvb, torch, restatement):
    """The trimmed 65,536-row Q8 head and the full 151,936-row head: kernel over all rows, oracle on a sample."""
    rng = np.random.default_rng(5)
    n = 896
    for d in (65536, 151936):
        w, ws = _random_q(rng, n, d, 8)
        xq = rng.integers(-127, 128, n).astype(np.int8)
        xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
        out = run_matvec4(mvb, torch, w, ws, xq, xs, n, d, 8)
        rows = np.concatenate([np.arange(64), rng.choice(d, 512, replace=False), np.arange(d - 64, d)])
        ref = restatement.matvec_f16(w[rows], ws[rows], xq, xs, n, rows.size, 8)
        assert same_bits(out[rows], ref), d


@pytest.mark.parametrize("n,d,gs", [(288, 288, 32), (288, 768, 32), (768, 288, 32), (768, 768, 64),
                                    (2048, 768, 64), (768, 32000, 64), (288, 32000, 32), (96, 7, 32), (8192, 9, 64)])
def test_matvec_runq_vs_restatement(mvb, torch, restatement, n, d, gs):
    """hls/matvec_tb.cpp:93-95 shapes, its value ranges (:56-58)."""
    rng = np.random.default_rng(n + d + gs)
    wq = rng.integers(-128, 128, d * n).astype(np.int8).reshape(d, n)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    ws = rng.uniform(1e-4, 2e-2, d * n // gs).astype(np.float32)
    xs = rng.uniform(1e-3, 1e-1, n // gs).astype(np.float32)
    out = run_matvec(mvb, torch, wq, ws, xq, xs, n, d, gs)
    assert same_bits(out, restatement.matvec_f32(wq, ws, xq, xs, n, d, gs))


@pytest.mark.parametrize("n,d,bits", [(896, 896, 4), (4864, 896, 4), (896, 4864, 4), (896, 2048, 8), (96, 5, 4)])
def test_fused_quantize_qwen(mvb, torch, restatement, n, d, bits):
    rng = np.random.default_rng(n + d)
    w, ws = _random_q(rng, n, d, bits)
    x = rng.standard_normal(n).astype(np.float32)
    x[32:64] = 0.0  # all-zero group: qwen.c's guard gives scale 0, values 0
    x[64:96] = np.float32(127.0) * (np.arange(32, dtype=np.float32) - 16) / 16 if n >= 96 else x[64:96]
    out = torch.empty(d, device="cuda")
    mvb.qmatvec4(dev(torch, w), dev(torch, ws.view(np.int16)), dev(torch, x), out, n, d, bits)
    torch.cuda.synchronize()
    xq, xs = restatement.quantize_qwen(x)
    assert same_bits(out.cpu().numpy(), restatement.matvec_f16(w, ws, xq, xs, n, d, bits))


@pytest.mark.parametrize("n,d,gs", [(288, 768, 32), (768, 2048, 64), (2048, 768, 64)])
def test_fused_quantize_runq(mvb, torch, restatement, n, d, gs):
    rng = np.random.default_rng(n + d + gs)
    wq = rng.integers(-127, 128, d * n).astype(np.int8).reshape(d, n)
    ws = rng.uniform(1e-4, 2e-2, d * n // gs).astype(np.float32)
    x = rng.standard_normal(n).astype(np.float32)
    x[:gs] = 0.0  # runq.c divides 0 by 0 here; the NaN converts to 0
    out = torch.empty(d, device="cuda")
    mvb.qmatvec(dev(torch, wq), dev(torch, ws), dev(torch, x), out, n, d, gs)
    torch.cuda.synchronize()
    xq, xs = restatement.quantize_runq(x, gs)
    assert same_bits(out.cpu().numpy(), restatement.matvec_f32(wq, ws, xq, xs, n, d, gs))


def test_fused_quantize_golden(mvb, torch):
    """The prologue's quantization equals qwen.c's own on the golden vectors: a unit identity-like matrix whose
    row g picks group g's scale makes out[g] = (sum of one group's xq) * xs[g]."""
    z = golden("quantize.npz")
    for i in range(3):
        x = z[f"qwen{i}_x"]
        n = x.size
        ng = n // 32
        # row g: int8 ones on group g's columns, scale 1.0 -> (float)sum(xq_g) * xs[g]
        w = np.zeros((ng, n), np.int8)
        for g in range(ng):
            w[g, g * 32:(g + 1) * 32] = 1
        ws = np.full((ng, ng), 0x3C00, np.uint16)
        out = torch.empty(ng, device="cuda")
        mvb.qmatvec4(dev(torch, w.view(np.uint8)), dev(torch, ws.view(np.int16)), dev(torch, x), out, n, ng, 8)
        torch.cuda.synchronize()
        q, s = z[f"qwen{i}_q"], z[f"qwen{i}_s"]
        expect = (q.reshape(ng, 32).astype(np.int32).sum(1).astype(np.float32) * np.float32(1.0)) * s
        assert same_bits(out.cpu().numpy(), expect.astype(np.float32)), i


def test_rejections_do_not_fault(mvb, torch):
    w = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    s = torch.zeros(1 << 16, dtype=torch.int16, device="cuda")
    x = torch.zeros(8192, dtype=torch.int8, device="cuda")
    xs = torch.zeros(256, device="cuda")
    out = torch.zeros(1024, device="cuda")
    L = mvb.lib()
    ptr = lambda t, off=0: t.data_ptr() + off
    for args in [(8224, 4, 4), (8192 + 32, 4, 8), (100, 4, 4), (896, 0, 4), (896, 4, 5), (0, 4, 4)]:
        n, d, bits = args
        assert L.mvb_matvec4(ptr(w), ptr(s), ptr(x), ptr(xs), ptr(out), n, d, bits, None) == -1, args
    # misaligned weight / activation pointers are rejected, not loaded
    assert L.mvb_matvec4(ptr(w, 8), ptr(s), ptr(x), ptr(xs), ptr(out), 896, 4, 4, None) == -1
    assert L.mvb_matvec4(ptr(w), ptr(s), ptr(x, 4), ptr(xs), ptr(out), 896, 4, 4, None) == -1
    assert L.mvb_matvec(ptr(w), ptr(xs), ptr(x), ptr(xs), ptr(out), 288, 4, 48, None) == -1
    torch.cuda.synchronize()
    assert mvb.rows_per_tile(896, 65536) >= 1


def test_deterministic(mvb, torch):
    rng = np.random.default_rng(9)
    n, d = 4864, 896
    w, ws = _random_q(rng, n, d, 4)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
    a = run_matvec4(mvb, torch, w, ws, xq, xs, n, d, 4)
    b = run_matvec4(mvb, torch, w, ws, xq, xs, n, d, 4)
    assert same_bits(a, b)


def test_every_fp16_scale_pattern(mvb, torch, restatement):
    """All 65,536 fp16 bit patterns as weight scales (2048 rows x 32 groups), exponent 31 included: qwen.c's f16()
    maps it to a finite value (qwen.c:89-91) where IEEE would give inf/nan; the kernel follows qwen.c."""
    rng = np.random.default_rng(31)
    n, d = 1024, 2048
    w = rng.integers(0, 256, (d, n // 2), dtype=np.uint8)
    ws = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(d, n // 32)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
    out = run_matvec4(mvb, torch, w, ws, xq, xs, n, d, 4)
    ref = restatement.matvec_f16(w, ws, xq, xs, n, d, 4)
    assert same_bits(out, ref)


@pytest.mark.parametrize("n,d,bits", [(4096, 8195, 4), (896, 65539, 8), (8192, 4100, 4)])
def test_large_matrices_ragged(mvb, torch, restatement, n, d, bits):
    """Large matrices with a ragged last tile: bit-exact on sampled rows, every row written."""
    rng = np.random.default_rng(n + d)
    w, ws = _random_q(rng, n, d, bits)
    xq = rng.integers(-128, 128, n).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
    out = run_matvec4(mvb, torch, w, ws, xq, xs, n, d, bits)
    rows = np.concatenate([np.arange(40), rng.choice(d, 300, replace=False), np.arange(d - 40, d)])
    assert same_bits(out[rows], restatement.matvec_f16(w[rows], ws[rows], xq, xs, n, rows.size, bits))
    assert not np.isnan(out).any()
