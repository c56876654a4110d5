"""The decode's expf (csrc/expf_ref.h) against the host C library's expf, which the reference's softmax and SiLU
call (qwen.c:350, :560): bit-identical on whole binades and on random inputs over the whole table domain."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def device_expf(mvb, torch, x):
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    entries, thresh = mvb.expf_device(xd, yd)
    torch.cuda.synchronize()
    return yd.cpu().numpy(), entries, thresh


@pytest.mark.parametrize("lo_bits,hi_bits", [(0xBC000000, 0xBC800000),   # [-2^-7, -2^-8): softmax near the max
                                              (0x3F800000, 0x40000000)])  # [1, 2): SiLU arguments
def test_expf_whole_binades(mvb, restatement, lo_bits, hi_bits):
    import torch
    x = np.arange(lo_bits, hi_bits, dtype=np.uint32).view(np.float32)
    y, entries, thresh = device_expf(mvb, torch, x)
    ref = restatement.expf(x)
    bad = np.flatnonzero(y.view(np.uint32) != ref.view(np.uint32))
    print(f"table entries {entries}, probe threshold {thresh:.4f} ulp, mismatches {bad.size} of {x.size}")
    assert bad.size == 0, x[bad[:5]]


def test_expf_random_domain(mvb, restatement):
    import torch
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-104, 89, 10_000_000), rng.standard_normal(10_000_000) * 4,
                        [0.0, -0.0, -104.0, 89.0, 88.72, -87.34, -103.97, 1e-30, -1e-30, np.inf, -np.inf]])
    x = x.astype(np.float32)
    y, _, _ = device_expf(mvb, torch, x)
    ref = restatement.expf(x)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
