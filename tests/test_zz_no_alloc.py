"""mvb_norm_matvec4_static: the decode's head path (final rmsnorm, quantize, head matvec) for callers that cannot
allocate device memory while running, e.g. hosts that fix every device buffer at start-up as the reference's own
qwen.c does, or code where cudaMalloc's device-wide synchronization is not acceptable. Its scratch is a fixed
device array inside the library, so the call takes its inputs and output and allocates nothing.

Checked through the C ABI against the existing entry point that computes the same thing with scratch the model
allocates: mvb_qwen_forward's head logits, on two calls in a row, bit for bit (the tolerance of every parity test
here). Kept in a file of its own that pytest collects last; it needs nothing from the other tests."""
import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu


def test_no_alloc_head_path_matches_decode(tmp_path):
    import torch
    mvb = load_pkg()
    torch.cuda.set_device(0)
    path = str(tmp_path / "tiny.qwb")
    mvb.qwb.write_synthetic_qwb(path, mvb.qwb.QWEN_TINY, seed=11)
    M = mvb.qwb.Qwb(path)
    c = M.cfg
    dim, hk, L = c["dim"], c["head_k"], c["n_layers"]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    w, ws = dev(M.head[0]), dev(M.head[1].view(np.int16))
    norm = dev(M.out_norm)
    dec = mvb.QwenDecoder(path, ctx=64)
    try:
        for tok, pos in ((5, 0), (777, 0)):  # two calls in a row; the second reuses the first call's scratch
            _, logits = dec.forward(tok, pos)
            x = dev(dec.trace(tok, pos)[2 * L])  # residual stream before the final rmsnorm
            out = torch.full((hk,), float("nan"), device="cuda")
            rc = mvb.norm_matvec4_static(x, norm, np.float32(c["rms_eps"]), w, ws, out, dim, hk, 8)
            assert rc == 0, mvb.last_error()
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), logits.view(np.uint32)), (tok, pos)
    finally:
        dec.close()
    # beyond the fixed scratch: a clear error, nothing launched
    big = torch.zeros(4096, device="cuda")
    assert mvb.norm_matvec4_static(big, big, 1e-6, w, ws, out, 4096, 4, 8) == -1
    assert "at most n = 2048" in mvb.last_error()
    # refused pointers (checked before any launch): no output, or misaligned weights; the previous output stays
    before = out.clone()
    assert mvb.norm_matvec4_static(x, norm, np.float32(c["rms_eps"]), w, ws, None, dim, hk, 8) == -1
    assert "null pointer" in mvb.last_error()
    w_odd = torch.empty(w.numel() + 16, dtype=torch.uint8, device="cuda")[1:1 + w.numel()]
    assert mvb.norm_matvec4_static(x, norm, np.float32(c["rms_eps"]), w_odd, ws, out, dim, hk, 8) == -1
    assert "misaligned" in mvb.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int32), before.view(torch.int32))
