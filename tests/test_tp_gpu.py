"""GPU: the fused column-parallel GEMM (dgx_tp_gemm_colsplit) — every rank
ends with the full product, which must match the oracle; a rank that never
joins a call makes the others' bounded completion wait report
DGX_ETIMEOUT (no hang, no fault). Runs on every visible GPU (1 GPU: the
single-rank path)."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, normwise

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, out):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch
    import torch.distributed as dist
    import dreamcompiler_b200 as dgx
    from dreamcompiler_b200 import tp
    from oracle import orc
    torch.cuda.set_device(rank)
    dgx.init(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    result = {"rank": rank}
    try:
        if mode == "wide":
            # bf16 C with shards wide enough for the 2-SM kernel at 2 ranks
            # (1-SM tiles beyond): every staged output box goes to all ranks
            # by TMA stores; 64 sampled rows against the oracle, and every
            # rank's C byte-identical
            M, N, K = 4096, 4096, 1024
            orc.set_seed(4)
            out_dtype = torch.bfloat16
        else:
            M, N, K = 512, 1000, 384
            orc.set_seed(3)
            out_dtype = torch.float32
        A = orc.randn(M, K)
        B = orc.randn(K, N)
        g = tp.ColumnParallelGemm(M, N, K, rank, world, out_dtype=out_dtype)
        Ad = torch.from_numpy(A).cuda().bfloat16()
        Bs = torch.from_numpy(B[:, g.col0:g.col0 + g.ncol].copy()).cuda().bfloat16()
        if mode == "wide":
            import hashlib
            for _ in range(2):
                Cb = g(Ad, Bs)
            dgx.sync_check()
            rows = np.random.default_rng(5).choice(M, 64, replace=False)
            ref = orc.gemm_f64(orc.round_bf16(A[rows]).astype(np.float64), orc.round_bf16(B).astype(np.float64))
            result["err"] = normwise(Cb.float().cpu().numpy()[rows], ref)
            result["digest"] = hashlib.sha1(Cb.view(torch.int16).cpu().numpy().tobytes()).hexdigest()
        elif mode == "ok":
            ref = orc.gemm_f64(orc.round_bf16(A).astype(np.float64), orc.round_bf16(B).astype(np.float64))
            for _ in range(3):
                Cf = g(Ad, Bs)
            dgx.sync_check()
            result["err"] = normwise(Cf.cpu().numpy(), ref)
        else:
            # rank world-1 never joins the second call: the others must time out
            g(Ad, Bs)
            dgx.sync_check()
            dist.barrier()
            if rank != world - 1:
                g(Ad, Bs, timeout_ms=300)
                try:
                    dgx.sync_check()
                    result["status"] = "ok"
                except dgx.DgxError as e:
                    result["status"] = e.status
            dist.barrier()
        g.close()
    finally:
        dist.destroy_process_group()
    out.put(result)


def _run(mode):
    world = torch.cuda.device_count()
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return world, res


def test_fused_allgather_matches_oracle():
    world, res = _run("ok")
    for r in res:
        assert r["err"] < 1e-2, r


def test_fused_allgather_tma_store_path():
    world, res = _run("wide")
    for r in res:
        assert r["err"] < 1e-2, r
    assert len({r["digest"] for r in res}) == 1, "ranks disagree on C"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_missing_rank_times_out_cleanly():
    from dreamcompiler_b200 import _lib
    world, res = _run("timeout")
    for r in res:
        if r["rank"] != world - 1:
            assert r["status"] == _lib.DGX_ETIMEOUT, r
