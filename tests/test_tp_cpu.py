"""CPU (gloo, world_size 2): the host-side logic of the column-parallel GEMM.
Each rank owns the reference's shard widths (dream_tp_matmul_column,
training.inc:1604-1630), computes its columns with the oracle, and the
gathered columns must equal the un-split product and the reference's own
output (tests/golden/tp.npz)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT, normwise


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, G_list, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from oracle import orc
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = np.load(os.path.join(ROOT, "tests", "golden", "tp.npz"))
    res = {}
    for (M, K, N) in [(12, 16, 24), (9, 10, 23)]:
        X, W = g[f"X_{M}_{K}_{N}"], g[f"W_{M}_{K}_{N}"]
        c0, nc = orc.tp_shard(N, world, rank)
        part = orc.gemm_f64(X, W[:, c0:c0 + nc].copy()) if nc else np.zeros((M, 0))
        # all-gather of variable-width column shards: pad to the widest
        width = orc.tp_shard(N, world, 0)[1]
        buf = torch.zeros(M, width, dtype=torch.float64)
        buf[:, :nc] = torch.from_numpy(part)
        bufs = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(bufs, buf)
        Y = np.zeros((M, N))
        for r in range(world):
            rc0, rnc = orc.tp_shard(N, world, r)
            Y[:, rc0:rc0 + rnc] = bufs[r][:, :rnc].numpy()
        res[(M, K, N)] = Y
    dist.destroy_process_group()
    if rank == 0:
        out.put({k: v.tolist() for k, v in res.items()})


def test_two_rank_column_split_matches_reference(golden):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, None, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = golden("tp")
    for key, Y in res.items():
        M, K, N = key
        Y = np.array(Y)
        assert normwise(Y, g[f"X_{M}_{K}_{N}"] @ g[f"W_{M}_{K}_{N}"]) < 1e-13
        assert normwise(Y, g[f"Y_{M}_{K}_{N}_2"]) < 1e-13
