"""The tensor-core prefill matmul (mvb_gemm4) against the pinned restatement: every token's output row must be
bit-identical to fpga_matvec4's computation for that token (qwen.c:436-456), for int4 and int8 weights, token
counts that fill or leave ragged the 16/32/64/128-token tiles, row counts that are not multiples of 128, column
counts that are not multiples of 128, every fp16 scale pattern and the extreme group sums."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available(), "a CUDA device is required"
    t.cuda.set_device(0)
    return t


def _random_case(rng, n, d, m, bits, scales="qwen"):
    w = rng.integers(0, 256, d * n * bits // 8, dtype=np.uint8).reshape(d, -1)
    ng = n // 32
    if scales == "all":  # every fp16 bit pattern, cycled over the rows and groups
        ws = (np.arange(d * ng) * 7919 % 65536).astype(np.uint16).reshape(d, ng)
    else:
        e = rng.integers(5, 11, d * ng)
        ws = ((rng.integers(0, 2, e.size) << 15) | (e << 10) | rng.integers(0, 1024, e.size)).astype(np.uint16)
        ws = ws.reshape(d, ng)
    xq = rng.integers(-128, 128, (m, n)).astype(np.int8)
    xs = rng.uniform(1e-3, 1e-1, (m, ng)).astype(np.float32)
    return w, ws, xq, xs


def _run(mvb, torch, w, ws, xq, xs, n, d, m, bits):
    ng = n // 32
    ldx = (m + 3) // 4 * 4
    xs_gm = np.zeros((ng, ldx), np.float32)
    xs_gm[:, :m] = xs.T
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out = torch.full((m, d), float("nan"), device="cuda")
    mvb.gemm4(dev(w), dev(ws.view(np.int16)), dev(xq), dev(xs_gm), out, n, d, m, ldx, bits)
    assert mvb.gemm_status() == 0
    return out.cpu().numpy()


def _expect(restatement, w, ws, xq, xs, n, d, m, bits):
    return np.stack([restatement.matvec_f16(w, ws, xq[t], xs[t], n, d, bits) for t in range(m)])


def _same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("n,d,m,bits", [
    (896, 896, 16, 4), (896, 4864, 128, 4), (4864, 896, 64, 4), (896, 128, 33, 4), (896, 1000, 130, 4),
    (8192, 256, 17, 4), (96, 200, 5, 4), (160, 130, 1, 4),
    (896, 4096, 128, 8), (896, 300, 7, 8), (4864, 384, 48, 8), (224, 129, 100, 8),
])
def test_gemm_matches_matvec_per_token(mvb, torch, restatement, n, d, m, bits):
    rng = np.random.default_rng(n * 7 + d * 3 + m + bits)
    w, ws, xq, xs = _random_case(rng, n, d, m, bits)
    out = _run(mvb, torch, w, ws, xq, xs, n, d, m, bits)
    assert _same_bits(out, _expect(restatement, w, ws, xq, xs, n, d, m, bits))


@pytest.mark.parametrize("n,d,m,bits", [(896, 20000, 128, 8), (896, 19456, 100, 4), (1024, 40000, 16, 8)])
def test_gemm_persistent_tiles(mvb, torch, restatement, n, d, m, bits):
    """More tiles than one wave (one CTA per SM walking several tiles, the pipeline running on from one tile into
    the next; the last shape runs one CTA per tile with two CTAs per SM): every token's row bit-identical too."""
    rng = np.random.default_rng(d + m + bits)
    w, ws, xq, xs = _random_case(rng, n, d, m, bits)
    out = _run(mvb, torch, w, ws, xq, xs, n, d, m, bits)
    assert _same_bits(out, _expect(restatement, w, ws, xq, xs, n, d, m, bits))


def test_gemm_scales_two_byte_aligned(mvb, torch, restatement):
    """Weight scales that start 2 bytes past an 8-byte boundary (the launcher accepts any even address): the
    epilogue reads them one by one instead of four at a time, with the same results."""
    rng = np.random.default_rng(77)
    n, d, m, bits = 896, 1000, 40, 4
    w, ws, xq, xs = _random_case(rng, n, d, m, bits)
    ng = n // 32
    ldx = (m + 3) // 4 * 4
    xs_gm = np.zeros((ng, ldx), np.float32)
    xs_gm[:, :m] = xs.T
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    buf = torch.zeros(d * ng + 4, dtype=torch.int16, device="cuda")
    wsd = buf[1:1 + d * ng]
    wsd.copy_(dev(ws.view(np.int16).reshape(-1)))
    assert wsd.data_ptr() % 8 == 2
    out = torch.full((m, d), float("nan"), device="cuda")
    mvb.gemm4(dev(w), wsd, dev(xq), dev(xs_gm), out, n, d, m, ldx, bits)
    assert mvb.gemm_status() == 0
    assert _same_bits(out.cpu().numpy(), _expect(restatement, w, ws, xq, xs, n, d, m, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_gemm_every_scale_pattern_and_extreme_sums(mvb, torch, restatement, bits):
    rng = np.random.default_rng(5 + bits)
    n, d, m = 512, 4096, 24  # 16 groups x 4096 rows = 65,536 scales: every fp16 pattern once
    w, ws, xq, xs = _random_case(rng, n, d, m, bits, scales="all")
    # extreme group sums in some rows and tokens: weights all -8 (int4: nibble 8) or -128, activations -128
    w[:64] = 0x88 if bits == 4 else 0x80
    xq[:4] = -128
    out = _run(mvb, torch, w, ws, xq, xs, n, d, m, bits)
    assert _same_bits(out, _expect(restatement, w, ws, xq, xs, n, d, m, bits))


def test_gemm_rejections(mvb, torch):
    import ctypes
    L = mvb.lib()
    w = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    s = torch.zeros(1 << 12, dtype=torch.int16, device="cuda")
    x = torch.zeros(1 << 14, dtype=torch.int8, device="cuda")
    xs = torch.zeros(1 << 10, device="cuda")
    out = torch.zeros(1 << 12, device="cuda")
    vp = lambda t, off=0: ctypes.c_void_p(t.data_ptr() + off)
    for n, d, m, ldx, bits in [(100, 4, 4, 4, 4), (96, 4, 4, 4, 5), (96, 0, 4, 4, 4), (96, 4, 0, 4, 4),
                               (96, 4, 5, 5, 4), (96, 4, 8, 4, 4), (8224, 4, 4, 4, 4)]:
        assert L.mvb_gemm4(vp(w), vp(s), vp(x), vp(xs), vp(out), n, d, m, ldx, bits, None) == -1
    assert L.mvb_gemm4(vp(w, 8), vp(s), vp(x), vp(xs), vp(out), 96, 4, 4, 4, 4, None) == -1
    assert L.mvb_gemm4(vp(w), vp(s), vp(x), vp(xs, 4), vp(out), 96, 4, 4, 4, 4, None) == -1
    assert mvb.gemm_status() == 0
