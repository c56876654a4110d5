"""Row sharding of a matvec across ranks (the config-5 path of bench.py --mode sharded), on the CPU with two gloo
ranks: each rank computes its contiguous row block (the oracle restatement stands in for the device kernel),
all_gather_into_tensor assembles the blocks, and the gathered output must equal the unsharded result bit for bit
on every rank, including a row count that does not divide evenly."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, n, d, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = oracle.Restatement()
        rng = np.random.default_rng(0)  # every rank draws the same full matrix and input
        w = rng.integers(0, 256, (d, n // 2), dtype=np.uint8)
        ws = ((rng.integers(0, 2, d * (n // 32)) << 15) | (rng.integers(5, 11, d * (n // 32)) << 10)
              | rng.integers(0, 1024, d * (n // 32))).astype(np.uint16).reshape(d, n // 32)
        xq = rng.integers(-128, 128, n).astype(np.int8)
        xs = rng.uniform(1e-3, 1e-1, n // 32).astype(np.float32)
        rows = -(-d // world)  # rows per rank; the last block is padded with unused rows
        r0 = rank * rows
        mine = max(0, min(rows, d - r0))
        part = np.zeros(rows, np.float32)
        if mine:
            part[:mine] = orc.matvec_f16(w[r0:r0 + mine], ws[r0:r0 + mine], xq, xs, n, mine, 4)
        full = torch.empty(rows * world)
        dist.all_gather_into_tensor(full, torch.from_numpy(part))
        ref = orc.matvec_f16(w, ws, xq, xs, n, d, 4)
        q.put((rank, bool(np.array_equal(full.numpy()[:d].view(np.uint32), ref.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("d", [1024, 1027])
def test_row_sharded_allgather_two_ranks(d):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, 256, d, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}
