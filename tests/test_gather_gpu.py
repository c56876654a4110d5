"""The row-sharded matvec whose all-gather runs inside the kernel (mvb_gather_*), against the pinned restatement.

One GPU (world 1): the gathered output of the scatter kernel and its bounded arrival wait equals the restatement
bit for bit, over repeated calls (the double-buffered output and the running arrival counter).

Two GPUs (one process per GPU, skipped with fewer): every rank computes its contiguous row block and the output
every rank reads is the whole unsharded result, bit for bit, including a row count that does not divide evenly;
then one rank skips a call, so the other's wait runs out and reports it through mvb_gather_error instead of
hanging. No rank leaves while any kernel of the gather is in flight.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _random_q(rng, n, d, bits):
    w = rng.integers(0, 256, d * n * bits // 8, dtype=np.uint8).reshape(d, -1)
    e = rng.integers(5, 11, d * (n // 32))
    ws = ((rng.integers(0, 2, e.size) << 15) | (e << 10) | rng.integers(0, 1024, e.size)).astype(np.uint16)
    return w, ws.reshape(d, n // 32)


def _inputs(rng, n):
    return rng.integers(-128, 128, n).astype(np.int8), rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)


def _same_bits(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _shard(w, ws, rank, rows, d):
    """Rank's row block, padded with zero rows to `rows`."""
    r0 = rank * rows
    mine = max(0, min(rows, d - r0))
    ws_blk = np.zeros((rows, ws.shape[1]), np.uint16)
    w_blk = np.zeros((rows, w.shape[1]), np.uint8)
    w_blk[:mine], ws_blk[:mine] = w[r0:r0 + mine], ws[r0:r0 + mine]
    return w_blk, ws_blk


@pytest.mark.parametrize("n,d,bits", [(896, 4864, 4), (8192, 1027, 4), (896, 151936 // 8, 8), (4864, 896, 8)])
def test_gather_one_rank(mvb, restatement, n, d, bits):
    import torch
    torch.cuda.set_device(0)
    rng = np.random.default_rng(n + d + bits)
    w, ws = _random_q(rng, n, d, bits)
    g = mvb.ShardGather(0, 1, d)
    try:
        g.connect([g.handle()])
        wd = torch.from_numpy(w).cuda()
        wsd = torch.from_numpy(ws.view(np.int16)).cuda()
        for call in range(3):  # both output buffers, then the first again
            xq, xs = _inputs(rng, n)
            g.matvec4(wd, wsd, torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), n, bits)
            out = g.output().cpu().numpy()
            assert g.error() == 0
            assert _same_bits(out, restatement.matvec_f16(w, ws, xq, xs, n, d, bits)), call
    finally:
        g.close()


def _xs_group_major(xs, m):
    ldx = (m + 3) // 4 * 4
    out = np.zeros((xs.shape[1], ldx), np.float32)
    out[:, :m] = xs.T
    return out, ldx


@pytest.mark.parametrize("n,d,m,bits", [(896, 4864, 32, 4), (8192, 1027, 20, 4), (896, 2048, 32, 8)])
def test_gather_gemm_one_rank(mvb, restatement, n, d, m, bits):
    """The batched gather (tensor-core matmul whose epilogue stores into the gathered output): token-major output,
    every token's row bit-identical to its matvec, over repeated calls."""
    import torch
    torch.cuda.set_device(0)
    rng = np.random.default_rng(n + d + m + bits)
    w, ws = _random_q(rng, n, d, bits)
    g = mvb.ShardGather(0, 1, d, tokens=m)
    try:
        g.connect([g.handle()])
        wd = torch.from_numpy(w).cuda()
        wsd = torch.from_numpy(ws.view(np.int16)).cuda()
        for call in range(3):
            xq = rng.integers(-128, 128, (m, n)).astype(np.int8)
            xs = rng.uniform(1e-3, 1e-1, (m, n // 32)).astype(np.float32)
            xs_gm, ldx = _xs_group_major(xs, m)
            g.gemm4(wd, wsd, torch.from_numpy(xq).cuda(), torch.from_numpy(xs_gm).cuda(), n, m, ldx, bits)
            out = g.output().cpu().numpy()
            assert g.error() == 0
            ref = np.stack([restatement.matvec_f16(w, ws, xq[t], xs[t], n, d, bits) for t in range(m)])
            assert _same_bits(out, ref), call
    finally:
        g.close()


def test_gather_rejections(mvb):
    import torch
    torch.cuda.set_device(0)
    with pytest.raises(mvb.MatvecError):
        mvb.ShardGather(2, 2, 16)
    with pytest.raises(mvb.MatvecError):
        mvb.ShardGather(0, 9, 16)
    g = mvb.ShardGather(0, 2, 64)
    try:
        w = torch.zeros(64 * 448, dtype=torch.uint8, device="cuda")
        ws = torch.zeros(64 * 28, dtype=torch.int16, device="cuda")
        xq = torch.zeros(896, dtype=torch.int8, device="cuda")
        xs = torch.zeros(28, device="cuda")
        with pytest.raises(mvb.MatvecError, match="not mapped"):  # rank 1's buffer was never connected
            g.matvec4(w, ws, xq, xs, 896, 4)
    finally:
        g.close()
    g = mvb.ShardGather(0, 1, 64)
    try:
        g.connect([g.handle()])
        for n, bits in [(900, 4), (896, 5), (8224, 4)]:
            with pytest.raises(mvb.MatvecError):
                g.matvec4(w, ws, xq, xs, n, bits)
        vp = ctypes.c_void_p  # misaligned weights are rejected, not loaded
        assert mvb.lib().mvb_gather_matvec4(g._g, vp(w.data_ptr() + 8), vp(ws.data_ptr()), vp(xq.data_ptr()),
                                            vp(xs.data_ptr()), 896, 4, None) == -1
        torch.cuda.synchronize()
    finally:
        g.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    import datetime
    import sys

    import torch
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from conftest import ROOT, load_pkg
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    results = {}
    try:
        mvb = load_pkg()
        orc = oracle.Restatement()
        for n, d, bits in [(896, 4864, 4), (896, 1027, 8), (8192, 2048, 4)]:
            rng = np.random.default_rng(d)  # every rank draws the same full matrix and inputs
            w, ws = _random_q(rng, n, d, bits)
            rows = -(-d // world)
            w_blk, ws_blk = _shard(w, ws, rank, rows, d)
            g = mvb.ShardGather(rank, world, rows)
            handles = [None] * world
            dist.all_gather_object(handles, g.handle())
            g.connect(handles)
            wd, wsd = torch.from_numpy(w_blk).cuda(), torch.from_numpy(ws_blk.view(np.int16)).cuda()
            ok = True
            for call in range(3):
                xq, xs = _inputs(rng, n)
                g.matvec4(wd, wsd, torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), n, bits)
                out = g.output()[:d].cpu().numpy()
                ok &= g.error() == 0 and _same_bits(out, orc.matvec_f16(w, ws, xq, xs, n, d, bits))
            results[(n, d, bits)] = bool(ok)
            torch.cuda.synchronize()
            dist.barrier()  # no rank's kernel still writes into a buffer about to be freed
            g.close()
            dist.barrier()
        # batch of 32 tokens through the tensor-core matmul, rows gathered by its epilogue
        n, d, bits, m = 896, 1027, 4, 32
        rng = np.random.default_rng(77)
        w, ws = _random_q(rng, n, d, bits)
        rows = -(-d // world)
        w_blk, ws_blk = _shard(w, ws, rank, rows, d)
        g = mvb.ShardGather(rank, world, rows, tokens=m)
        handles = [None] * world
        dist.all_gather_object(handles, g.handle())
        g.connect(handles)
        xq = rng.integers(-128, 128, (m, n)).astype(np.int8)
        xs = rng.uniform(1e-3, 1e-1, (m, n // 32)).astype(np.float32)
        xs_gm, ldx = _xs_group_major(xs, m)
        g.gemm4(torch.from_numpy(w_blk).cuda(), torch.from_numpy(ws_blk.view(np.int16)).cuda(),
                torch.from_numpy(xq).cuda(), torch.from_numpy(xs_gm).cuda(), n, m, ldx, bits)
        out = g.output()[:, :d].cpu().numpy()
        ref = np.stack([orc.matvec_f16(w, ws, xq[t], xs[t], n, d, bits) for t in range(m)])
        results["batch32"] = bool(g.error() == 0 and _same_bits(out, ref))
        torch.cuda.synchronize()
        dist.barrier()
        g.close()
        dist.barrier()
        # A rank that skips a call: the other rank's bounded wait gives up and reports it.
        g = mvb.ShardGather(rank, world, 256)
        handles = [None] * world
        dist.all_gather_object(handles, g.handle())
        g.connect(handles)
        w = torch.zeros(256 * 448, dtype=torch.uint8, device="cuda")
        ws = torch.zeros(256 * 28, dtype=torch.int16, device="cuda")
        xq = torch.zeros(896, dtype=torch.int8, device="cuda")
        xs = torch.zeros(28, device="cuda")
        if rank == 0:
            g.matvec4(w, ws, xq, xs, 896, 4)
            results["timeout_reported"] = g.error() == 1
        torch.cuda.synchronize()
        dist.barrier()
        g.close()
        dist.barrier()
        q.put((rank, results))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


def test_gather_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (one process per GPU)")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert "error" not in results[r], results[r]
        assert all(v for k, v in results[r].items()), results[r]
    assert results[0]["timeout_reported"]


def test_gather_graph_replay_one_rank(mvb, restatement):
    """The fused gather keeps its call number on the device, so calls captured in a CUDA graph replay correctly:
    after the graph of three calls is replayed twice (six calls, alternating output buffers), the output the
    library reports is the last call's and equals the restatement bit for bit."""
    import torch
    torch.cuda.set_device(0)
    n, d, bits = 896, 2048, 4
    rng = np.random.default_rng(99)
    w, ws = _random_q(rng, n, d, bits)
    g = mvb.ShardGather(0, 1, d)
    try:
        g.connect([g.handle()])
        wd, wsd = torch.from_numpy(w).cuda(), torch.from_numpy(ws.view(np.int16)).cuda()
        xq, xs = _inputs(rng, n)
        xqd, xsd = torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda()
        g.matvec4(wd, wsd, xqd, xsd, n, bits)  # one eager call first
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(3):
                g.matvec4(wd, wsd, xqd, xsd, n, bits)
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        assert g.error() == 0
        assert _same_bits(g.output().cpu().numpy(), restatement.matvec_f16(w, ws, xq, xs, n, d, bits))
        del graph
    finally:
        g.close()
