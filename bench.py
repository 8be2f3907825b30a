"""Benchmark: GEMM & FlashAttention fwd+bwd TFLOPS on B200 vs the host CPU.

Default workload = BASELINE configs[1]: causal FlashAttention forward +
backward, batch 8 x 16 heads, seq 2048, head dim 64, bf16 Q/K/V/dO ~ N(0,1),
scale 1/8, fp32 softmax statistics. One step = dgx_flash_fwd + dgx_flash_bwd
over one batch resident in HBM. Multi-GPU: one process per GPU, each rank
runs its own batch (attention shards by batch x head with no communication,
so scaling is weak); time = max over ranks of CUDA-event time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Prints ONE JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GEMM & FlashAttn fwd+bwd TFLOPS (% tensor peak) at 1/2/4/8 B200 vs host CPU"
B, H, S, D = 8, 16, 2048, 64
BH = B * H
FWD_FLOP = 4.0 * BH * S * S * D / 2   # causal: half the S^2 pairs
BWD_FLOP = 10.0 * BH * S * S * D / 2
HEAD_FLOP = (FWD_FLOP + BWD_FLOP) / BH
NOMINAL_DENSE_BF16 = 2250.0
CONFIG = {"workload": "FlashAttention fwd+bwd, causal (BASELINE configs[1])", "batch": B, "heads": H,
          "seq_len": S, "head_dim": D, "causal": True, "scale": 1.0 / 8,
          "parallelism": "batch x head across ranks, no communication (weak: each rank a full batch)",
          "l2": "two rotating input sets (256 MiB of inputs > 126 MB L2)"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the other configs' numbers (N=1 only)")
    return ap.parse_args()


def peaks():
    """(burst, sustained, source) dense bf16 TFLOP/s. The headline kernels are
    timed in a region of a few milliseconds, so the burst figure is their
    denominator."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:
        return 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------- CPU side
def _cpu_worker(args):
    kind, seed = args
    from oracle import cpu_bench
    return cpu_bench.flash_head(kind, seed, S, D)


def cpu_flash_sample(workers: int, kind: str, seed0: int = 0):
    """`workers` heads in parallel, one per process (the reference's
    FlashAttention is single-threaded). Returns (TFLOPS, wall seconds)."""
    ctx = mp.get_context("spawn")
    with ctx.Pool(workers) as pool:
        pool.map(_cpu_worker, [(kind, 1)] * workers)  # load the library in every worker
        times = pool.map(_cpu_worker, [(kind, seed0 + i) for i in range(workers)])
    t = max(times)
    return workers * HEAD_FLOP / t / 1e12, t


def cpu_workers() -> int:
    n = os.cpu_count() or 1
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:
        pass
    return max(1, min(n, 32))


# ---------------------------------------------------------------- clocks
def nvml_handle(pynvml, device_index: int):
    """NVML handle of CUDA device `device_index`, matched by UUID (NVML
    numbers every GPU of the machine, CUDA only the visible ones), else by
    PCI bus id, else by index."""
    try:
        import torch
        props = torch.cuda.get_device_properties(device_index)
        uuid = getattr(props, "uuid", None)
        if uuid is not None:
            u = str(uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-") else "GPU-" + u)
    except Exception:
        pass
    try:
        import torch
        props = torch.cuda.get_device_properties(device_index)
        bus = "%08X:%02X:%02X.0" % (getattr(props, "pci_domain_id"), getattr(props, "pci_bus_id"),
                                    getattr(props, "pci_device_id"))
        return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
    except Exception:
        pass
    return pynvml.nvmlDeviceGetHandleByIndex(device_index)


def pin_to_gpu_cpus(device_index: int) -> None:
    """Restrict this process to the CPU cores NVML reports as local to the
    GPU, so that pinned host buffers allocated afterwards sit on the GPU's
    own socket (the end-to-end copies cross PCIe from there)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        words = pynvml.nvmlDeviceGetCpuAffinity(nvml_handle(pynvml, device_index), 64)
        cpus = {w * 64 + b for w, m in enumerate(words) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
    except Exception:
        pass


class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) in a thread during a region."""

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.stop_flag = [], set(), False
        self.max_mhz, self.ok = None, False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = nvml_handle(pynvml, device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass
        self.names = {}
        if self.ok:
            nv = self.nv
            for attr, name in (("nvmlClocksEventReasonHwSlowdown", "hw_slowdown"),
                               ("nvmlClocksEventReasonHwThermalSlowdown", "hw_thermal_slowdown"),
                               ("nvmlClocksEventReasonSwThermalSlowdown", "sw_thermal_slowdown"),
                               ("nvmlClocksEventReasonSwPowerCap", "sw_power_cap"),
                               ("nvmlClocksEventReasonHwPowerBrakeSlowdown", "hw_power_brake"),
                               ("nvmlClocksEventReasonApplicationsClocksSetting", "applications_clocks_setting"),
                               ("nvmlClocksEventReasonSyncBoost", "sync_boost")):
                if hasattr(nv, attr):
                    self.names[getattr(nv, attr)] = name

    def _run(self):
        while not self.stop_flag:
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.names.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.0005)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 0.5:  # first sample before the region starts
                time.sleep(0.0002)
        return self

    def __exit__(self, *exc):
        self.stop_flag = True
        if self.ok:
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0,
                    "source": "nvml" if self.ok else "unavailable"}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml, 0.5 ms poll"}


# ---------------------------------------------------------------- GPU side
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import dreamcompiler_b200 as dgx
    from dreamcompiler_b200 import _lib

    torch.cuda.set_device(local_rank)
    dgx.init(local_rank)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = [[torch.randn(BH, S, D, device=dev, generator=gen).bfloat16() for _ in range(4)] for _ in range(2)]
    O = torch.empty(BH, S, D, device=dev, dtype=torch.bfloat16)
    L = torch.empty(BH, S, device=dev, dtype=torch.float32)
    dQ, dK, dV = (torch.empty_like(O) for _ in range(3))
    ws = torch.empty(dgx.flash_bwd_workspace_size(BH, S, D) // 4 + 1, device=dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)

    def step(i, timer=None):
        q, k, v, do = sets[i & 1]
        dgx.flash_fwd(q, k, v, out=O, lse=L)
        if timer is not None:
            lib.dgx_set_timer_events(timer[0].cuda_event, timer[1].cuda_event)
        dgx.flash_bwd(q, k, v, O, do, L, dQ=dQ, dK=dK, dV=dV, workspace=ws)

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        step(i)
    dgx.sync_check()
    K = args.steps
    timers = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for a, b in timers:  # materialise the CUDA events
        a.record(stream)
        b.record(stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clocks:
        e0.record(stream)
        for i in range(K):
            step(i, timers[i])
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    dgx.sync_check()
    elapsed = e0.elapsed_time(e1) / 1e3
    bwd_kernel_s = sum(a.elapsed_time(b) for a, b in timers) / 1e3 / K

    # ---- end to end: host bf16 buffers in pinned memory, H2D -> fwd -> bwd -> D2H,
    # pipelined over head chunks on three streams.
    pin_to_gpu_cpus(local_rank)
    host_in = [torch.empty(BH, S, D, dtype=torch.bfloat16, pin_memory=True) for _ in range(4)]
    for h, d in zip(host_in, sets[0]):
        h.copy_(d)
    host_out = [torch.empty(BH, S, D, dtype=torch.bfloat16, pin_memory=True) for _ in range(4)]
    # 32-head chunks (8 MiB per tensor copy) in a ring of 4 device slots:
    # the fastest of the chunk / ring sizes tried (8-32 heads, 2-4 slots).
    CH = 32
    nch = BH // CH
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    ring = 4
    dbuf = [[torch.empty(CH, S, D, device=dev, dtype=torch.bfloat16) for _ in range(8)] for _ in range(ring)]
    dl = [torch.empty(CH, S, device=dev) for _ in range(ring)]
    wsc = torch.empty(dgx.flash_bwd_workspace_size(CH, S, D) // 4 + 1, device=dev)
    ev_in = [torch.cuda.Event() for _ in range(ring)]
    ev_cmp = [torch.cuda.Event() for _ in range(ring)]
    ev_out = [torch.cuda.Event() for _ in range(ring)]

    def e2e_step():
        for c in range(nch):
            r = c % ring
            q, k, v, do, o, gq, gk, gv = dbuf[r]
            sl = slice(c * CH, (c + 1) * CH)
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_out[r])
                for dst, src in zip((q, k, v, do), host_in):
                    dst.copy_(src[sl], non_blocking=True)
                ev_in[r].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[r])
                dgx.flash_fwd(q, k, v, out=o, lse=dl[r])
                dgx.flash_bwd(q, k, v, o, do, dl[r], dQ=gq, dK=gk, dV=gv, workspace=wsc)
                ev_cmp[r].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[r])
                for dst, src in zip(host_out, (o, gq, gk, gv)):
                    dst[sl].copy_(src, non_blocking=True)
                ev_out[r].record(s_out)

    e2e_steps = max(3, min(K, 20))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    # Steps follow one another without a host or stream barrier: step i+1's
    # uploads overlap step i's downloads (PCIe is full duplex); the ring events
    # keep each device buffer's reuse in order.
    t0.record(s_in)
    for _ in range(e2e_steps):
        e2e_step()
    s_out.wait_stream(s_cmp)
    t1.record(s_out)
    torch.cuda.synchronize(dev)
    barrier()
    dgx.sync_check()
    e2e_s = t0.elapsed_time(t1) / 1e3 / e2e_steps

    t = torch.tensor([elapsed, e2e_s], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t[0].item(), t[1].item(), bwd_kernel_s, clocks.summary()


def run_reference_api_e2e(steps: int):
    """The same config-2 step through the reference's own operator boundary:
    the Dream runtime with the B200 backend (refside), f64 `Tensor*` in and
    out. One step = dream_flash_attention(Q, K, V, 128, 2048, 64) then
    backward(sum(O * G)) (how a Dream program injects dO = G), every operand
    a host f64 tensor; the backend uploads Q, K, V, G, converts, runs the
    kernels and writes O and the three gradients back into the host tensors.
    Each step changes one element of Q, K, V and G first, so every step
    uploads its inputs (the device copies fail their fingerprints). Host wall
    time per step (host work included: the runtime's allocations, the
    elementwise mul and sum on the host)."""
    import ctypes as C
    import numpy as np
    from dreamcompiler_b200 import refside
    if not refside.available():
        return {"unavailable": "libdream_ref_b200.so not built"}
    R = refside
    R.load()
    rng = np.random.default_rng(17)
    shape = (BH, S * D)
    ts = [R.tensor(rng.standard_normal(shape)) for _ in range(4)]
    Q, K, V, G = ts
    args = [R.scalar(v) for v in (BH, S, D, 64)]
    views = [R.view(t) for t in ts]

    def step(i):
        for v in views:
            v[i % v.size] += 1e-3
        O = R.call("dream_flash_attention", Q, K, V, *args)
        prod = R.call("tensor_mul", O, G)
        loss = R.call("sum", prod)
        R.call("backward", loss)
        for t in (loss, prod, O):
            R.call("tensor_decref", t)

    before = R.counts()
    step(0)
    walls = []
    tb = R.times_us()
    for i in range(steps):
        t0 = time.perf_counter()
        step(i + 1)
        walls.append(time.perf_counter() - t0)
    after = R.counts()
    ta = R.times_us()
    t = statistics.median(walls)
    nbytes = BH * S * D * 8
    return {"value": (FWD_FLOP + BWD_FLOP) / t / 1e12, "unit": "TFLOPS", "ms_per_step": t * 1e3,
            "steps": steps, "h2d_bytes_per_step": 4 * nbytes, "d2h_bytes_per_step": 4 * nbytes,
            "device_ops": {k: after[k] - before[k] for k in after},
            "backend_host_ms_per_step": {k: (ta[k] - tb[k]) / steps / 1e3 for k in ta},
            "path": "reference Dream runtime (its own struct Tensor, ops and autograd) with the B200 backend: "
                    "f64 host tensors Q, K, V, G -> dream_flash_attention + backward(sum(O*G)) -> O, dQ, dK, dV "
                    "as f64 host tensors; host wall time, median over steps"}


TP_N = 16384


def run_tp_gemm(args, rank, world, local_rank):
    """BASELINE config 4 at its largest size: bf16 C = A.B, M=N=K=16384, B
    column-sharded over the ranks (reference widths), the all-gather of C
    fused into the GEMM epilogue (NVLink peer stores). Strong scaling: the
    problem is fixed, each rank computes N/world columns. Returns the max over
    ranks of the per-step time, and (N > 1) the max over ranks of a 1-GPU
    pass of the whole product timed just before it on the same GPUs, the
    denominator of the strong-scaling efficiency."""
    import torch
    import torch.distributed as dist
    import dreamcompiler_b200 as dgx
    from dreamcompiler_b200 import tp
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    n = TP_N
    steps = max(3, min(args.steps, 20))
    t1 = None
    if world > 1:
        # every rank runs the unsharded GEMM alone (no peer traffic): T(1)
        A1 = (torch.randn(n, n, device=dev, generator=g) / n ** 0.5).bfloat16()
        B1 = (torch.randn(n, n, device=dev, generator=g) / n ** 0.5).bfloat16()
        C1 = torch.empty(n, n, device=dev, dtype=torch.bfloat16)
        s1 = max(3, steps // 2)
        for _ in range(2):
            dgx.gemm(A1, B1, out=C1)
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(s1):
            dgx.gemm(A1, B1, out=C1)
        e1.record()
        torch.cuda.synchronize(dev)
        dgx.sync_check()
        tt = torch.tensor([e0.elapsed_time(e1) / 1e3 / s1], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t1 = tt.item()
        del A1, B1, C1
        torch.cuda.empty_cache()
    gemm = tp.ColumnParallelGemm(n, n, n, rank, world, out_dtype=torch.bfloat16, device=dev)
    A = (torch.randn(n, n, device=dev, generator=g) / n ** 0.5).bfloat16()
    B = (torch.randn(n, gemm.ncol, device=dev, generator=g) / n ** 0.5).bfloat16()
    for _ in range(3):
        gemm(A, B)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        gemm(A, B)
    e1.record()
    torch.cuda.synchronize(dev)
    dgx.sync_check()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3 / steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    gemm.close()
    del A, B, gemm
    torch.cuda.empty_cache()
    return t.item(), steps, (t1 if t1 is not None else t.item())


def run_secondary(local_rank):
    """The other BASELINE configs on this GPU, each timed with CUDA events
    after warm-up (rank 0 at N=1 only):
      configs[4]  int8 weight-only dense 4096x4096, B in {1, 16, 256}, both modes
      configs[0]  f32 GEMM 1024^3 + dA/dB backward (3xTF32 tcgen05)
      configs[2]  char-level GPT training step (fwd + bwd + AdamW), tokens/s
      configs[3]  bf16 GEMM 4096/8192/16384^3, single GPU (last: the 16384^3
                  GEMMs leave the part power-capped for a while)
    Operands that fit in L2 are cycled through enough copies to exceed it.
    Each entry carries the median SM clock sampled over its timed replays
    (the latency-bound int8 layer runs first, before the GEMM sweeps)."""
    import torch
    import dreamcompiler_b200 as dgx
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(5)
    res = {}

    def timed(fn, iters, reps=5):
        """Device time per call: `iters` calls captured in one CUDA graph
        (so microsecond kernels are not measured as Python launch overhead),
        replayed `reps` times between CUDA events after warm-up."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                fn(0)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for i in range(iters):
                fn(i)
        graph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clk:
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize(dev)
        summ = clk.summary()
        last_clk.clear()
        last_clk.update({"sm_mhz": summ["sm_mhz"], "sm_max_mhz": summ["sm_max_mhz"], "reasons": summ["reasons"]})
        dgx.sync_check()
        del graph
        return e0.elapsed_time(e1) / 1e3 / (iters * reps)

    last_clk = {}

    # int8 weight-only 4096x4096; 16 weight copies (256 MB) cycle past L2
    N = K = 4096
    Ws = [torch.randint(-127, 128, (N, K), device=dev, dtype=torch.int8, generator=g) for _ in range(16)]
    sc = torch.rand(N, device=dev, generator=g) * 9e-3 + 1e-3
    bias = torch.randn(N, device=dev, generator=g)
    w8 = {}
    for Bn in (1, 16, 256):
        X = torch.randn(Bn, K, device=dev, generator=g)
        Y = torch.empty(Bn, N, device=dev)
        for mode in (0, 1):
            t = timed(lambda i: dgx.gemm_w8(X, Ws[i % 16], sc, bias, mode=mode, out=Y), 64)
            byts = N * K + Bn * K * 4 + Bn * N * 4 + N * 8
            w8[f"B{Bn}_{'w8a32' if mode == 0 else 'w8a8'}"] = {"us": t * 1e6, "gb_s": byts / t / 1e9,
                                                               "tops": 2 * Bn * N * K / t / 1e12,
                                                               "clocks": dict(last_clk)}
    res["config5_int8_w8"] = w8
    del Ws
    torch.cuda.empty_cache()

    # FlashAttention fwd+bwd at head dim 128 (the reference's GPU kernel serves
    # dk <= 128): config 2's shape otherwise, the two-half tiles forward and
    # the two-kernel backward; two input sets (512 MiB) alternate past L2
    Sd, Dd = 2048, 128
    fa_sets = [[torch.randn(BH, Sd, Dd, device=dev, generator=g).bfloat16() for _ in range(4)] for _ in range(2)]
    Od = torch.empty(BH, Sd, Dd, device=dev, dtype=torch.bfloat16)
    Ld = torch.empty(BH, Sd, device=dev)
    gq, gk, gv = (torch.empty_like(Od) for _ in range(3))
    wsd = torch.empty(dgx.flash_bwd_workspace_size(BH, Sd, Dd) // 4 + 1, device=dev)

    def fa128_step(i):
        q, k, v, do = fa_sets[i & 1]
        dgx.flash_fwd(q, k, v, out=Od, lse=Ld)
        dgx.flash_bwd(q, k, v, Od, do, Ld, dQ=gq, dK=gk, dV=gv, workspace=wsd)
    t = timed(fa128_step, 10)
    fl = 14.0 * BH * Sd * Sd * Dd / 2
    res["fa_d128_fwd_bwd"] = {"ms_per_step": t * 1e3, "tflops": fl / t / 1e12, "clocks": dict(last_clk),
                              "shape": f"BH={BH} (8 x 16) S={Sd} D={Dd} causal",
                              "flop": "(4 + 10) * BH * S^2 * D / 2 (algorithmic; the backward issues 14)"}
    del fa_sets, Od, Ld, gq, gk, gv, wsd
    torch.cuda.empty_cache()

    # f32 1024^3 forward + backward; 24 operand sets (288 MB) cycle past L2
    n = 1024
    sets = [[torch.randn(n, n, device=dev, generator=g) for _ in range(3)] for _ in range(24)]
    C = torch.empty(n, n, device=dev)
    dA = torch.empty(n, n, device=dev)
    dB = torch.empty(n, n, device=dev)
    ws = torch.empty(dgx.gemm_workspace_size(n, n, n) // 4 + 1, device=dev)

    def f32_step(i):
        A, B, dC = sets[i % len(sets)]
        dgx.gemm(A, B, out=C, workspace=ws)
        dgx.gemm(dC, B, transB=True, out=dA, workspace=ws)
        dgx.gemm(A, dC, transA=True, out=dB, workspace=ws)
    t = timed(f32_step, 50)
    res["config1_f32_gemm_1024_fwd_bwd"] = {"ms_per_step": t * 1e3, "tflops": 6 * n ** 3 / t / 1e12,
                                            "clocks": dict(last_clk),
                                            "path": "3xTF32 on tcgen05 kind::tf32 (3 MMAs per K step)"}
    del sets, C, dA, dB, ws

    # char-level GPT training step (6 layers, d 384, 6 heads, seq 256,
    # batch 64, vocab 65): forward, backward and AdamW, synthetic uniform token ids
    from dreamcompiler_b200.gpt import GPT, GPTConfig
    cfg = GPTConfig()
    model = GPT(cfg, device=dev, seed=0)
    gtok = torch.Generator().manual_seed(3)
    tok = torch.randint(0, cfg.vocab, (cfg.batch * cfg.seq_len,), generator=gtok, dtype=torch.int32)
    model.set_batch(tok, torch.randint(0, cfg.vocab, tok.shape, generator=gtok, dtype=torch.int32))
    t = timed(lambda i: model.step(), 4)
    res["config3_gpt_train_step"] = {"ms_per_step": t * 1e3, "tokens_per_s": cfg.batch * cfg.seq_len / t,
                                     "tflops": cfg.flops_per_step() / t / 1e12, "loss": float(model.loss.item()),
                                     "clocks": dict(last_clk),
                                     "params": cfg.n_params(), "algorithmic_flop_per_step": cfg.flops_per_step(),
                                     "precision": "bf16 GEMM/attention operands, fp32 master weights, grads, AdamW"}
    del model
    torch.cuda.empty_cache()

    # bf16 GEMM sweep, C bf16
    sweep = {}
    for n in (4096, 8192, 16384):
        copies = 4 if n == 4096 else 1   # 4 x 64 MiB of operands > L2 at 4096
        A = [(torch.randn(n, n, device=dev, generator=g) / n ** 0.5).bfloat16() for _ in range(copies)]
        B = [(torch.randn(n, n, device=dev, generator=g) / n ** 0.5).bfloat16() for _ in range(copies)]
        Cb = torch.empty(n, n, device=dev, dtype=torch.bfloat16)
        t = timed(lambda i: dgx.gemm(A[i % copies], B[i % copies], out=Cb), 20 if n < 16384 else 6)
        sweep[str(n)] = {"ms": t * 1e3, "tflops": 2 * n ** 3 / t / 1e12, "clocks": dict(last_clk)}
        del A, B, Cb
        torch.cuda.empty_cache()
    res["config4_bf16_gemm"] = sweep

    return res


def traffic_per_launch():
    """DRAM bytes per flash_bwd_kernel launch from the committed ncu summary
    (profiles/flash_bwd_traffic.json), scaled to this workload's heads."""
    try:
        with open(os.path.join(ROOT, "profiles", "flash_bwd_traffic.json")) as f:
            p = json.load(f)
        return p["dram_bytes_per_launch"] * BH / p["bh"]
    except Exception:
        return None


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(world, 1)

    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import cpu_bench
        kind = cpu_bench.available_kind()
        w = cpu_workers()
        vals = []
        per_step = None
        steps_run = 0
        for i in range(args.warmup + args.steps):
            tf, wall = cpu_flash_sample(w, kind, seed0=i * w)
            per_step = wall if per_step is None else per_step
            if i >= args.warmup:
                vals.append(tf)
                steps_run += 1
            # keep the whole reference run to a few minutes
            if steps_run >= 1 and (i + 1) * max(per_step, 1.0) > 150:
                break
        v = statistics.median(vals) if vals else 0.0
        ms = HEAD_FLOP * w / (v * 1e12) * 1e3 if v else None
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOPS", "n_gpus": n,
            "steps": steps_run, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic N(0,1), reference RNG",
            "config": CONFIG,
            "cpu_baseline": {"value": v, "unit": "TFLOPS", "cores": w, "kind": kind,
                             "sample": f"{w} heads of config 2 (S=2048, dk=64) per step, one per process, "
                                       "dream_flash_attention + backward (single-threaded per head)"},
            "e2e": {"value": v, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    cpu = None
    if n == 1 and not args.no_cpu_baseline:
        # Before any CUDA work: worker processes are spawned, never forked.
        from oracle import cpu_bench
        kind = cpu_bench.available_kind()
        w = cpu_workers()
        samples = [cpu_flash_sample(w, kind, seed0=i * w) for i in range(3)]
        tfs = sorted(tf for tf, _ in samples)
        cpu = {"value": statistics.median(tfs), "unit": "TFLOPS", "cores": w, "kind": kind,
               "samples": tfs,
               "sample": f"median of 3 samples, each {w} heads of config 2 (S=2048, dk=64) fwd+bwd, one per "
                         f"process ({', '.join('%.2f' % wl for _, wl in samples)} s wall)"}

    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    elapsed, e2e_s, bwd_kernel_s, clocks = run_ours(args, rank, world, local_rank)
    # the secondary configs (1 GPU) before the TP GEMM: its 16384^3 steps
    # leave the part power-capped for a while
    ref_api = run_reference_api_e2e(3) if world == 1 and not args.no_secondary else None
    secondary = run_secondary(local_rank) if world == 1 and not args.no_secondary else None
    tp_s, tp_steps, tp_s1 = run_tp_gemm(args, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    step_flop = FWD_FLOP + BWD_FLOP
    value = n * step_flop * args.steps / elapsed / 1e12
    burst, sustained, src = peaks()
    achieved = BWD_FLOP / bwd_kernel_s / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": n, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: bf16 Q/K/V/dO ~ N(0,1), seeded, config 2 shapes", "config": CONFIG,
        "pct_of_peak": {"per_gpu_tflops": value / n, "of_nominal_dense_bf16_2250": value / n / NOMINAL_DENSE_BF16,
                        f"of_{src}_bf16_burst": value / n / burst},
        "roofline": {"kernel": "flash_bwd_kernel", "bound": "tensor", "achieved": achieved, "peak": burst,
                     "peak_source": f"{src} bf16 burst (the kernel is timed in a region of a few ms)",
                     "unit": "TFLOP/s", "frac": achieved / burst, "traffic": traffic_per_launch(),
                     "algorithmic": f"{BWD_FLOP:.4g} FLOP per launch = 10*BH*S^2*D/2 (causal)"},
        "e2e": {"value": n * step_flop / e2e_s / 1e12, "unit": "TFLOPS", "h2d_bytes_per_step": 4 * BH * S * D * 2,
                "d2h_bytes_per_step": 4 * BH * S * D * 2,
                "host_cpus": len(os.sched_getaffinity(0)),
                "path": "pinned host bf16 Q,K,V,dO -> dgx_flash_fwd/bwd -> O,dQ,dK,dV to host, 32-head chunks "
                        "pipelined on 3 streams, consecutive steps overlapped (PCIe Gen5 x16: about 49 GB/s "
                        "each way when both directions run)"},
        "tp_gemm": {"config": f"bf16 C=A.B, M=N=K={TP_N} (BASELINE configs[3]), B column-sharded over {n} "
                              "GPU(s), all-gather fused into the epilogue (NVLink peer stores)",
                    "scaling": "strong", "value": 2.0 * TP_N ** 3 / tp_s / 1e12, "unit": "TFLOPS",
                    "ms_per_step": tp_s * 1e3, "steps": tp_steps,
                    "ms_per_step_1gpu_same_run": tp_s1 * 1e3,
                    "efficiency_vs_n1": tp_s1 / (n * tp_s),
                    "per_gpu_frac_of_measured_bf16": 2.0 * TP_N ** 3 / tp_s / 1e12 / n / burst},
        "gpu_launches": 4 * args.steps,
        "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if ref_api is not None:
        line["e2e_reference_api"] = ref_api
    if secondary is not None:
        line["other_configs"] = secondary
    print(json.dumps(line))


if __name__ == "__main__":
    main()
