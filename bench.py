#!/usr/bin/env python
"""Benchmark of the quantized decode GEMV on B200.

Headline workload: Q4_K weight, 4096 output rows x 14336 inputs, M = 1 token,
the shape the decode-GEMV target is quoted on.  One step = one pass over a
ring of R distinct weight copies (R * 33 MB > 4 x the 126 MB L2, so every
GEMV streams its weights from HBM), each copy with its own activation row:
per copy one GEMV kernel (the Q8_0 activation quantisation is fused into its
shared-memory stage), replayed from a CUDA graph with programmatic dependent
launch.

Reported (one JSON line on rank 0):
  value       whole-job algorithmic GB/s (weights + x + y bytes / time)
  e2e         same metric through odi_cuda_matmul_host (host x -> device,
              product, device -> host y, per call), the reference-facing call
  roofline    the GEMV kernel alone: algorithmic bytes / average launch time
              (CUDA events around a graph of GEMV-only launches) vs the
              measured HBM copy bandwidth in MEASURED_PEAKS.json
  cpu_baseline the oracle's restatement of the reference loop on the host
              cores (the reference itself throws on Q4_K), bounded sample
  configs     (1 GPU) the reference's other configurations: the 7B decode
              GEMV sweep (Q8_0 / Q4_K / Q6_K, M = 1 and 8), the tensor-core
              prefill GEMM (Q4_K, M = 512 and 2048, TFLOP/s) and the 70B
              Q4_K GEMV shapes (M = 1 and 32)
  decode_7b   (1 GPU) the second half of the metric: tokens/s of greedy
              decode of a Llama-2-7B-shaped Q4_K/Q6_K model with 2048 prompt
              tokens in the fp16 KV cache, 256 timed steps (CUDA events
              around graph replays), its HBM roofline (weights + mean KV
              bytes per token), an end-to-end figure through
              DecodeModel.generate and a host-core sample of the same
              token's matrix products

Multi-GPU (torchrun, N > 1): weak scaling by output-row sharding -- every
rank holds a 4096-row shard of each weight (the full matrix has 4096*N
rows), computes its slice and the slices are all-gathered with NCCL after
every GEMV.

--impl reference: the reference's CPU loop (oracle restatement for Q4_K,
since CPUBackend::matmul throws for K-quants) on the host cores, same
metric, each step one GEMV of the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DT_NAME = "Q4_K"
N_ROWS, K_COLS, M_TOK = 4096, 14336, 1
L2_BYTES = 126 * 1024 * 1024
SWEEPS = 64  # passes over the weight ring per step


def q4k_bytes(N, K):
    return N * (K // 256) * 144


def algo_bytes(N, K, M):
    """Algorithmic bytes of one GEMV: packed weights + fp32 x + fp32 y."""
    return q4k_bytes(N, K) + M * K * 4 + M * N * 4


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first_sample(self, timeout=5.0):
        """Block until nvidia-smi is producing samples, then drop the idle ones."""
        t0 = time.time()
        while self.proc and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.01)
        self.lines.clear()

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline
# ---------------------------------------------------------------------------
CPU_REPS = 8  # GEMVs of the workload per CPU sample (one reference-arm step)


def host_threads():
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_port_gemv_time(nthreads: int, reps: int = CPU_REPS, N=N_ROWS, K=K_COLS):
    """The oracle's restatement of the reference loop (matmul_q4_0's
    per-block dequantise-and-accumulate structure over Q4_K blocks) on
    nthreads host threads: mean seconds per GEMV over `reps` GEMVs of the
    workload, after one untimed GEMV.  Both arms use this one sample, so
    their CPU figures agree.  The reference runs an M=1 product on ONE thread
    (parallel_for is serial below 4 x threads rows, cpu_backend.cpp:149), so
    the port on every host thread is a generous baseline."""
    import oracle as O

    if "b" not in _PORT:
        w = O.seeded_weights(N, K, seed=0)
        _PORT["b"] = O.quantize(O.Q4_K, w)
        _PORT["x"] = O.seeded_acts(M_TOK, K, seed=1)
    b, x = _PORT["b"], _PORT["x"]
    O.matmul_ref(O.Q4_K, x, b, N, nthreads)  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        O.matmul_ref(O.Q4_K, x, b, N, nthreads)
    return (time.perf_counter() - t0) / reps


def cpu_sample_text(nthreads, reps=CPU_REPS):
    return (f"{reps} Q4_K {N_ROWS}x{K_COLS} M=1 GEMVs on {nthreads} host threads: the oracle's restatement of the "
            "reference block loop (CPUBackend::matmul throws for K-quants); the reference itself runs M=1 on one "
            "thread (cpu_backend.cpp:149), so this is a generous baseline")


def reference_q4_0_config1(budget_s: float):
    """The UNMODIFIED reference CPUBackend::matmul (oracle/_ref) on config 1:
    Q4_0 4096x4096, M=1.  Returns (GB/s, seconds per call, threads used) or None."""
    import oracle as O

    L = O.ref_lib()
    if L is None:
        return None
    w = O.seeded_weights(4096, 4096, seed=0)
    b = O.quantize(O.Q4_0, w)
    x = O.seeded_acts(1, 4096, seed=1)
    out = np.zeros((1, 4096), np.float32)
    nproc = os.cpu_count() or 1
    t1 = L.ref_matmul_time(O.Q4_0, out.ctypes.data, x.ctypes.data, b.ctypes.data, 1, 4096, 4096, nproc, 1)
    reps = max(1, int(budget_s / max(t1, 1e-4)))
    t = L.ref_matmul_time(O.Q4_0, out.ctypes.data, x.ctypes.data, b.ctypes.data, 1, 4096, 4096, nproc, reps)
    per = t / reps
    gb = (b.nbytes + 4096 * 4 + 4096 * 4) / per / 1e9
    # parallel_for runs serially when M < 4 * threads (cpu_backend.cpp:149)
    return gb, per, 1 if 1 < 4 * nproc else nproc


def run_reference(args, rank):
    """The reference arm: the reference's CPU loop for this path on the host
    cores (the oracle restatement: CPUBackend::matmul throws on Q4_K), same
    metric and config as our arm; each step = one CPU sample of CPU_REPS
    GEMVs of the workload."""
    if rank != 0:
        return 0
    nthreads = host_threads()
    step_bytes = algo_bytes(N_ROWS, K_COLS, M_TOK)
    times = []
    for i in range(args.warmup + args.steps):
        t = cpu_port_gemv_time(nthreads)
        if i >= args.warmup:
            times.append(t)
    tmean = sum(times) / len(times)
    value = step_bytes / tmean / 1e9
    R = max(4, -(-4 * L2_BYTES // q4k_bytes(N_ROWS, K_COLS)))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tmean * CPU_REPS * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(R, args.gpus),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": nthreads, "kind": "port",
                         "sample": cpu_sample_text(nthreads)},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_decode:
        t_cpu, sample = cpu_decode_sample(nthreads)
        print(json.dumps({"aux": "decode_7b", "impl": "reference",
                          "metric": "7B-shape Q4_K decode tokens/s (1 sequence, greedy)",
                          "value": round(1.0 / t_cpu, 4), "unit": "tokens/s",
                          "cpu_baseline": {"value": round(1.0 / t_cpu, 4), "unit": "tokens/s", "cores": nthreads,
                                           "kind": "port", "sample": sample}}), flush=True)
    print(json.dumps(line), flush=True)
    return 0


_PORT = {}


METRIC = "Q4_K decode GEMV HBM GB/s (4096x14336, M=1)"


def workload_config(R, world, gather="fused"):
    return {
        "workload": f"Q4_K GEMV {N_ROWS}x{K_COLS} (out x in), M={M_TOK}; a step = {SWEEPS} passes over a "
                    f"ring of {R} weight copies",
        "dtype": DT_NAME, "N_per_gpu": N_ROWS, "N_total": N_ROWS * world, "K": K_COLS, "M": M_TOK,
        "ring_copies": R, "l2": "inputs larger than L2: each step streams the whole ring "
                                 f"({R} x {q4k_bytes(N_ROWS, K_COLS) / 1e6:.1f} MB > 126 MB L2)",
        "act_mode": "q8 (activations quantised to Q8_0, int8 dp4a dots, fp32 scales)",
        "parallelism": (f"row-shard x{world}, gathered by the GEMV epilogue (NVLink peer stores + arrival "
                        f"counters)" if gather == "fused" else f"row-shard x{world} + NCCL all-gather")
        if world > 1 else "single GPU",
    }


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import ctypes

    import torch

    import odiengine_b200 as ob

    torch.cuda.set_device(local_rank)
    ob.init(local_rank)
    L = ob.lib()
    dev = torch.device("cuda", local_rank)
    dt = ob.ODI_DTYPE_Q4_K
    N, K, M = N_ROWS, K_COLS, M_TOK
    wbytes = q4k_bytes(N, K)
    R = max(4, -(-4 * L2_BYTES // wbytes))  # ring >= 4 x L2
    if args.profile:
        R = 4
    stream = torch.cuda.Stream(device=dev)
    s_ptr = stream.cuda_stream

    # --- weights: seeded N(0, 0.02) fp32 on the device, quantised on the device
    gen = torch.Generator(device=dev)
    weights = []
    with torch.cuda.stream(stream):
        for r in range(R):
            gen.manual_seed(1000 * rank + r)
            wf = torch.empty((N, K), dtype=torch.float32, device=dev).normal_(0.0, 0.02, generator=gen)
            blocks = ob.quantize_weight(dt, wf, stream=stream)
            del wf
            weights.append(ob.repack(dt, blocks, N, K, stream=stream))
            del blocks
        gen.manual_seed(7 + rank)
        xs = [torch.empty((M, K), dtype=torch.float32, device=dev).normal_(0.0, 1.0, generator=gen) for _ in range(R)]
        ys = [torch.zeros((M, N), dtype=torch.float32, device=dev) for _ in range(R)]
        gathered = [torch.zeros((world * M, N), dtype=torch.float32, device=dev) for _ in range(R)] \
            if world > 1 else None
    stream.synchronize()
    ws_bytes = ob.workspace_bytes(dt, M, N, K, ob.ACT_Q8)
    ws = ob.new_workspace(ws_bytes, dev)

    if args.profile:
        # Small case for ncu: three eager products on distinct ring copies
        # (each weight 33 MB, the ring > L2), nothing else.
        for r in range(3):
            ob.check(L.odi_cuda_matmul(dt, weights[r].data_ptr(), xs[r].data_ptr(), ys[r].data_ptr(), M, N, K,
                                       ob.ACT_Q8, ws.data_ptr(), ws.numel(), 0, s_ptr))
        stream.synchronize()
        assert ob.workspace_status(ws) == 0
        print(json.dumps({"profile": "ok", "launches": 6}))
        return 0

    pg = None
    fused = world > 1 and args.gather == "fused"
    if world > 1:
        import torch.distributed as dist

        pg = dist.group.WORLD
    if fused:
        # Row shards gathered by the GEMV itself: each rank's GEMV stores its
        # slice into every rank's buffer for that ring copy (NVLink peer
        # stores) and bumps per-rank arrival counters; a one-block kernel
        # waits for all ranks (bounded) before the next product.
        from odiengine_b200.sharded import SymmetricBuffer

        obytes = M * N * world * 4
        sym = SymmetricBuffer(256 + R * obytes, pg)
        own = sym.ptrs[rank]
        inc = (ctypes.c_uint64 * world)(*([L.odi_cuda_scatter_signals(dt, M, N, K, ob.ACT_Q8)] * world))
        scatters = []
        for r in range(R):
            sc = ob.Scatter()
            for p in range(world):
                sc.out[p] = sym.ptrs[p] + 256 + r * obytes
                sc.counters[p] = sym.ptrs[p]
            sc.nranks, sc.rank, sc.row0, sc.ld = world, rank, rank * N, N * world
            scatters.append(sc)

    def step_body(flags=ob.FLAG_PDL, gemv_only=False):
        # one product = one kernel (activation quantisation is fused in);
        # gemv_only leaves out the multi-GPU gathers
        for r in range(R):
            if fused and not gemv_only:
                ob.check(L.odi_cuda_matmul_scatter(dt, weights[r].data_ptr(), xs[r].data_ptr(), M, N, K, ob.ACT_Q8,
                                                   ws.data_ptr(), ws.numel(), flags, ctypes.byref(scatters[r]),
                                                   s_ptr))
                ob.check(L.odi_cuda_wait_peers(own, own + 64, inc, world, ws.data_ptr(), s_ptr))
                continue
            ob.check(L.odi_cuda_matmul(dt, weights[r].data_ptr(), xs[r].data_ptr(), ys[r].data_ptr(), M, N, K,
                                       ob.ACT_Q8, ws.data_ptr(), ws.numel(), flags, s_ptr))
            if world > 1 and not gemv_only:
                import torch.distributed as dist

                dist.all_gather_into_tensor(gathered[r], ys[r], group=pg)

    # warm up eagerly (sets kernel attributes, NCCL comms) then capture graphs
    with torch.cuda.stream(stream):
        step_body()
        step_body(gemv_only=True)
    stream.synchronize()
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step, stream=stream):
        step_body()
    g_gemv = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_gemv, stream=stream):
        step_body(gemv_only=True)
    stream.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # --- headline: whole steps.  A step = SWEEPS passes over the ring (graph
    # replays on `stream`, where the events are recorded).
    def run_steps(graph, n):
        with torch.cuda.stream(stream):
            for _ in range(n * SWEEPS):
                graph.replay()

    run_steps(g_step, args.warmup)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        clk.wait_first_sample()
        ev0.record(stream)
        run_steps(g_step, args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms_step = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    bytes_step = SWEEPS * R * (world * wbytes + M * K * 4 * world + M * N * 4 * world)
    value = bytes_step / (ms_step * 1e-3) / 1e9

    # --- roofline: the GEMV kernel alone (no collectives), average launch time
    run_steps(g_gemv, 1)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(5, args.steps)
    e0.record(stream)
    run_steps(g_gemv, reps)
    e1.record(stream)
    torch.cuda.synchronize()
    us_gemv = e0.elapsed_time(e1) * 1e3 / (reps * SWEEPS * R)
    achieved = algo_bytes(N, K, M) / (us_gemv * 1e-6) / 1e9
    peak, peak_kind = measured_peak()

    # --- e2e through the host-buffer C ABI (per-call H2D x, product, D2H y)
    import numpy as _np

    e2e = None
    if world == 1:
        hw = []
        for r in range(R):
            h = ctypes.c_void_p()
            # upload once: the device copy made by odi_cuda_weight_upload from host GGUF bytes
            hb = ob.unpack(dt, weights[r], N, K).cpu().numpy()
            ob.check(L.odi_cuda_weight_upload(hb.ctypes.data_as(ctypes.c_void_p), dt, N, K, ctypes.byref(h)))
            hw.append(h)
        hx = torch.empty((R, M, K), dtype=torch.float32).pin_memory()
        hy = torch.empty((R, M, N), dtype=torch.float32).pin_memory()
        hx.copy_(torch.stack([x.cpu() for x in xs]))
        px = [hx[r].data_ptr() for r in range(R)]
        py = [hy[r].data_ptr() for r in range(R)]
        mm_async, mm_sync, host_sync = L.odi_cuda_matmul_host_async, L.odi_cuda_matmul_host, L.odi_cuda_host_sync

        def e2e_step_async():
            # the step's products queued back to back, one sync (and error
            # word check) at the end: x pulled from page-locked memory while
            # the product before it runs, y stored into page-locked memory
            for _ in range(SWEEPS):
                for r in range(R):
                    rc = mm_async(hw[r], px[r], py[r], M, ob.ACT_Q8, s_ptr)
                    if rc:
                        ob.check(rc)
            ob.check(host_sync(s_ptr))

        def e2e_step_sync():
            for _ in range(SWEEPS):
                for r in range(R):
                    rc = mm_sync(hw[r], px[r], py[r], M, ob.ACT_Q8, s_ptr)
                    if rc:
                        ob.check(rc)

        e2e_steps = max(3, min(args.steps, 20))
        for _ in range(args.warmup):
            e2e_step_async()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step_async()
        el = (time.perf_counter() - t0) / e2e_steps
        for _ in range(min(args.warmup, 2)):
            e2e_step_sync()
        sync_steps = max(2, e2e_steps // 4)
        t0 = time.perf_counter()
        for _ in range(sync_steps):
            e2e_step_sync()
        el_sync = (time.perf_counter() - t0) / sync_steps
        e2e = {"value": round(bytes_step / el / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": SWEEPS * R * M * K * 4, "d2h_bytes_per_step": SWEEPS * R * M * N * 4,
               "steps": e2e_steps,
               "ms_per_step": round(el * 1e3, 4),
               "call": "odi_cuda_matmul_host_async per weight, odi_cuda_host_sync once per step (the error word "
                       "checked); pinned host x/y: x pulled by a kernel ahead of each product, y stored by the "
                       "GEMV into host memory",
               "sync_per_call": {"value": round(bytes_step / el_sync / 1e9, 3), "unit": "GB/s",
                                 "ms_per_step": round(el_sync * 1e3, 4), "steps": sync_steps,
                                 "call": "odi_cuda_matmul_host per weight, each call waits for its product"}}
        ref_y = ys[-1].cpu().numpy()
        _np.testing.assert_allclose(hy[-1].numpy(), ref_y, rtol=0, atol=0)
        for h in hw:
            L.odi_cuda_weight_free(h)

    # --- CPU baseline (rank 0, N = 1 only): the reference arm's own sample
    cpu = None
    ref_cfg1 = None
    if rank == 0 and world == 1 and not args.no_cpu:
        nth = host_threads()
        per = cpu_port_gemv_time(nth)
        cpu = {"value": round(algo_bytes(N, K, M) / per / 1e9, 4), "unit": "GB/s", "cores": nth, "kind": "port",
               "sample": cpu_sample_text(nth)}
        r1 = reference_q4_0_config1(min(5.0, args.cpu_budget))
        if r1:
            ref_cfg1 = {"aux": "reference_cpu_config1", "value": round(r1[0], 4), "unit": "GB/s",
                        "ms_per_call": round(r1[1] * 1e3, 3), "threads_used": r1[2], "kind": "reference",
                        "sample": "unmodified CPUBackend::matmul, Q4_0 4096x4096 M=1 (config 1)"}

    decode = None
    configs = None
    if world == 1 and (not args.no_decode or not args.no_configs):
        g_step = g_gemv = None  # release the graphs before the other legs allocate
        if not args.no_decode:
            decode = run_decode(args, local_rank)
        if not args.no_configs:
            configs = run_config_legs(args)

    sharded = None
    if world > 1 and not args.no_configs:
        g_step = g_gemv = None  # graphs with collectives go before the next ones are made
        sharded = run_sharded_70b(args, rank, world, local_rank)

    if rank == 0:
        # Full detail first, one JSON object per line; the headline comes last
        # and ends with compact summaries of the same numbers, so the end of
        # stdout carries them.
        for aux in (ref_cfg1, decode and dict(aux="decode_7b", **decode), configs and dict(aux="configs", **configs),
                    sharded and dict(aux="sharded_70b", **sharded)):
            if aux:
                print(json.dumps(aux), flush=True)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_k weights x q8_0 activations (int8 dp4a, fp32 accumulate)", "data": "synthetic",
            "config": workload_config(R, world, args.gather),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic_per_launch(),
                         "traffic_source": TRAFFIC_SOURCE,
                         "kernel": "qgemv_kernel<Q4_K,1,false>", "us_per_launch": round(us_gemv, 3),
                         "algorithmic_bytes_per_launch": algo_bytes(N, K, M), "peak_kind": peak_kind},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "gpu_launches": args.steps * SWEEPS * R * (2 if fused else 1),
        }
        if decode:
            line["decode_7b"] = {"value": decode["value"], "unit": "tokens/s",
                                 "frac": decode["roofline"]["frac"],
                                 "e2e": decode["e2e"]["value"],
                                 "cpu": decode["cpu_baseline"]["value"] if decode.get("cpu_baseline") else None}
        if configs:
            line["configs_frac"] = config_summary(configs)
        if sharded:
            line["sharded_70b_frac"] = {f"{r['N']}x{r['K']} M{r['M']}": [r["frac_gemv"], r["frac_nccl"], r.get("frac_fused")]
                                        for r in sharded["rows"]}
        print(json.dumps(line), flush=True)
    g_step = g_gemv = None
    if fused:
        torch.cuda.synchronize()
        st = ob.workspace_status(ws)
        if st:
            raise RuntimeError(f"peer wait gave up (error word {st:#x})")
        if world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[local_rank])
        sym.close()
    return 0


SHARD_SHAPES = ((28672, 8192), (8192, 28672), (128256, 8192))  # the 70B shapes of the row-sharding config


def run_sharded_70b(args, rank, world, local_rank, reps=10):
    """The row-sharding configuration (strong scaling): each 70B-shaped Q4_K
    weight split by output rows over the `world` ranks (S = N / world rows
    each), at M = 1 and 32 tokens (ODI_CUDA_ACT_AUTO).  Per shape and token
    count, device time per product (CUDA events around graph replays over a
    ring of shard copies > 4 x L2, max over ranks) of
      gemv   the rank's shard product alone;
      nccl   the product through odi_cuda_matmul_sharded: shard product,
             in-place ncclAllGather of the slices, layout of [M, N] (C ABI);
      fused  (M = 1) the shard product storing its slice into every rank's
             output over NVLink, then the bounded wait for all ranks.
    GB/s counts the whole weight (all shards) + x + y per product; frac is
    against world x the measured HBM copy bandwidth."""
    import ctypes

    import torch
    import torch.distributed as dist

    import odiengine_b200 as ob
    from odiengine_b200.sharded import SymmetricBuffer

    L = ob.lib()
    dev = torch.device("cuda", local_rank)
    peak, _ = measured_peak()
    dt = ob.ODI_DTYPE_Q4_K
    uid = ctypes.create_string_buffer(ob.NCCL_ID_BYTES)
    if rank == 0:
        ob.check(L.odi_cuda_nccl_unique_id(uid))
    box = [uid.raw if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    uid = ctypes.create_string_buffer(box[0], ob.NCCL_ID_BYTES)
    comm = ctypes.c_void_p()
    ob.check(L.odi_cuda_nccl_init(uid, world, rank, ctypes.byref(comm)))
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    rows = []

    def timed(body):
        with torch.cuda.stream(stream):
            body()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            body()
        with torch.cuda.stream(stream):
            g.replay()
        stream.synchronize()
        dist.barrier(device_ids=[local_rank])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        stream.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        return float(t.item())

    try:
        for N, K in SHARD_SHAPES:
            S = N // world
            R = max(2, -(-4 * L2_BYTES // ob.tiled_bytes(dt, S, K)))
            gen = torch.Generator(device=dev)
            gen.manual_seed(100 + rank)
            wf = torch.empty((S, K), dtype=torch.float32, device=dev).normal_(0.0, 0.02, generator=gen)
            base = ob.repack(dt, ob.quantize_weight(dt, wf), S, K)
            del wf
            ring = [base] + [base.clone() for _ in range(R - 1)]
            for M in (1, 32):
                mode = ob.ACT_AUTO
                gen.manual_seed(7)
                xs = [torch.empty((M, K), dtype=torch.float32, device=dev).normal_(0.0, 1.0, generator=gen)
                      for _ in range(R)]
                ysh = torch.empty((M, S), dtype=torch.float32, device=dev)
                yfull = torch.empty((M, N), dtype=torch.float32, device=dev)
                wsg = ob.new_workspace(ob.workspace_bytes(dt, M, S, K, mode), dev)
                wss = ob.new_workspace(L.odi_cuda_sharded_workspace_bytes(comm, dt, M, S, K, mode), dev)

                def gemv():
                    for r in range(R):
                        ob.check(L.odi_cuda_matmul(dt, ring[r].data_ptr(), xs[r].data_ptr(), ysh.data_ptr(), M, S, K,
                                                   mode, wsg.data_ptr(), wsg.numel(), ob.FLAG_PDL, sp))

                def nccl():
                    for r in range(R):
                        ob.check(L.odi_cuda_matmul_sharded(comm, dt, ring[r].data_ptr(), xs[r].data_ptr(),
                                                           yfull.data_ptr(), M, N, S, K, mode, wss.data_ptr(),
                                                           wss.numel(), ob.FLAG_PDL, sp))

                row = {"N": N, "K": K, "M": M, "S": S, "ring": R}
                algo = ob.gguf_bytes(dt, N, K) + M * K * 4 + M * N * 4
                for name, body in (("gemv", gemv), ("nccl", nccl)):
                    us = timed(body) * 1e3 / (reps * R)
                    row["us_" + name] = round(us, 2)
                    row["frac_" + name] = round(algo / us / 1e3 / (world * peak), 4)
                if M == 1:
                    obytes = M * N * 4
                    sym = SymmetricBuffer(256 + R * obytes)
                    own = sym.ptrs[rank]
                    inc = (ctypes.c_uint64 * world)(*([L.odi_cuda_scatter_signals(dt, M, S, K, ob.ACT_Q8)] * world))
                    scs = []
                    for r in range(R):
                        sc = ob.Scatter()
                        for p in range(world):
                            sc.out[p] = sym.ptrs[p] + 256 + r * obytes
                            sc.counters[p] = sym.ptrs[p]
                        sc.nranks, sc.rank, sc.row0, sc.ld = world, rank, rank * S, N
                        scs.append(sc)
                    wsf = ob.new_workspace(ob.workspace_bytes(dt, M, S, K, ob.ACT_Q8), dev)

                    def fused():
                        for r in range(R):
                            ob.check(L.odi_cuda_matmul_scatter(dt, ring[r].data_ptr(), xs[r].data_ptr(), M, S, K,
                                                               ob.ACT_Q8, wsf.data_ptr(), wsf.numel(), ob.FLAG_PDL,
                                                               ctypes.byref(scs[r]), sp))
                            ob.check(L.odi_cuda_wait_peers(own, own + 64, inc, world, wsf.data_ptr(), sp))

                    us = timed(fused) * 1e3 / (reps * R)
                    row["us_fused"] = round(us, 2)
                    row["frac_fused"] = round(algo / us / 1e3 / (world * peak), 4)
                    torch.cuda.synchronize()
                    st = ob.workspace_status(wsf)
                    dist.barrier(device_ids=[local_rank])
                    sym.close()
                    if st:
                        raise RuntimeError(f"peer wait gave up (error word {st:#x})")
                for k in ("gemv", "nccl", "fused"):
                    if "us_" + k in row:
                        row["GBs_" + k] = round(algo / row["us_" + k] / 1e3, 1)
                rows.append(row)
            del ring, base
            torch.cuda.empty_cache()
    finally:
        torch.cuda.synchronize()
        ob.check(L.odi_cuda_nccl_free(comm))
    return {"metric": "Q4_K GEMV HBM GB/s, 70B shapes split by rows over the GPUs (strong scaling)",
            "n_gpus": world, "rows": rows, "peak_per_gpu": peak,
            "method": "CUDA events around CUDA-graph replays (PDL) over a ring of shard copies > 4 x L2, max over "
                      "ranks; gemv = the shard product alone, nccl = odi_cuda_matmul_sharded (product + in-place "
                      "ncclAllGather + [M, N] layout), fused = the product's epilogue storing to every rank over "
                      "NVLink + the bounded wait"}


def time_products(dt, N, K, M, act_mode, reps=20, seed=0, dev=None):
    """Device time per product y = x . W^T (us) of odi_cuda_matmul chained
    with programmatic dependent launch in a CUDA graph, over a ring of
    distinct weight copies larger than 4 x L2 (every product streams its
    weight from HBM), each copy with its own activations.  Returns
    (us per product, algorithmic bytes per product, ring copies)."""
    import torch

    import odiengine_b200 as ob

    L = ob.lib()
    dev = dev or torch.device("cuda", torch.cuda.current_device())
    wb = ob.tiled_bytes(dt, N, K)
    R = max(2, -(-4 * L2_BYTES // wb))
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    with torch.cuda.stream(stream):
        wf = torch.empty((N, K), dtype=torch.float32, device=dev).normal_(0.0, 0.02, generator=gen)
        base = ob.repack(dt, ob.quantize_weight(dt, wf, stream=stream), N, K, stream=stream)
        del wf
        ring = [base] + [base.clone() for _ in range(R - 1)]
        xs = [torch.empty((M, K), dtype=torch.float32, device=dev).normal_(0.0, 1.0, generator=gen) for _ in range(R)]
        ys = [torch.zeros((M, N), dtype=torch.float32, device=dev) for _ in range(R)]
    stream.synchronize()
    ws = ob.new_workspace(ob.workspace_bytes(dt, M, N, K, act_mode), dev)

    def body():
        for r in range(R):
            ob.check(L.odi_cuda_matmul(dt, ring[r].data_ptr(), xs[r].data_ptr(), ys[r].data_ptr(), M, N, K,
                                       act_mode, ws.data_ptr(), ws.numel(), ob.FLAG_PDL, sp))

    with torch.cuda.stream(stream):
        body()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        body()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    stream.synchronize()
    if ob.workspace_status(ws):
        raise RuntimeError("a bounded device wait gave up")
    us = e0.elapsed_time(e1) * 1e3 / (reps * R)
    del g, ring, base, xs, ys
    torch.cuda.empty_cache()
    return us, ob.gguf_bytes(dt, N, K) + M * K * 4 + M * N * 4, R


def run_config_legs(args):
    """The reference configurations beside the headline, on one GPU:
    config 2 (7B decode GEMV shapes, Q8_0 / Q4_K / Q6_K, M = 1 and 8),
    config 3 (prefill GEMM on the tensor cores, Q4_K, M = 512 and 2048),
    config 5 (70B Q4_K GEMV shapes, M = 1 and 32)."""
    import odiengine_b200 as ob

    peak_hbm, kind = measured_peak()
    peak_tc = measured_tc_peak()
    out = {"gemv_sweep": [], "prefill_gemm": [], "gemv_70b": [],
           "method": "CUDA events over CUDA-graph replays of PDL-chained odi_cuda_matmul (ODI_CUDA_ACT_AUTO) over a "
                     "ring of weight copies > 4 x L2; GB/s = (packed weight + fp32 x + fp32 y bytes) / time"}
    names = {ob.ODI_DTYPE_Q8_0: "Q8_0", ob.ODI_DTYPE_Q4_K: "Q4_K", ob.ODI_DTYPE_Q6_K: "Q6_K"}
    for dt in (ob.ODI_DTYPE_Q8_0, ob.ODI_DTYPE_Q4_K, ob.ODI_DTYPE_Q6_K):
        for N, K in ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)):
            for M in (1, 8):
                us, b, R = time_products(dt, N, K, M, ob.ACT_AUTO, reps=10)
                gbs = b / us / 1e3
                path = ("Q8 records, one 8-token pass, int8 mma.sync dots" if M == 8
                        else "Q8_0 activations quantised on chip, int8 dp4a dots")
                out["gemv_sweep"].append({"dtype": names[dt], "N": N, "K": K, "M": M, "us": round(us, 3),
                                          "GBs": round(gbs, 1), "hbm_frac": round(gbs / peak_hbm, 4),
                                          "path": path})
    for N, K in ((14336, 4096), (4096, 14336)):
        for M in (512, 2048):
            us, _, R = time_products(ob.ODI_DTYPE_Q4_K, N, K, M, ob.ACT_AUTO, reps=5)
            tf = 2.0 * M * N * K / us / 1e6
            out["prefill_gemm"].append({"dtype": "Q4_K", "N": N, "K": K, "M": M, "us": round(us, 2),
                                        "TFLOPs": round(tf, 1), "tensor_frac": round(tf / peak_tc, 4),
                                        "path": "tcgen05 (fp16-decoded weights, fp32 accumulate in TMEM)"})
    for N, K in ((28672, 8192), (8192, 28672), (128256, 8192)):
        for M in (1, 32):
            us, b, R = time_products(ob.ODI_DTYPE_Q4_K, N, K, M, ob.ACT_AUTO, reps=5)
            gbs = b / us / 1e3
            out["gemv_70b"].append({"dtype": "Q4_K", "N": N, "K": K, "M": M, "us": round(us, 2),
                                    "GBs": round(gbs, 1), "hbm_frac": round(gbs / peak_hbm, 4)})
    out["peaks"] = {"hbm_gbs": peak_hbm, "bf16_tflops": peak_tc, "kind": kind}
    return out


def measured_tc_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


DEC_PROMPT, DEC_GEN = 2048, 256


def run_decode(args, local_rank):
    """7B-shape decode (Llama-2-7B shape: 32 layers, hidden 4096, 32 heads of
    128, ffn 11008, vocab 32000; Q4_K attention and gate/up, Q6_K down and
    output, seeded N(0, 0.02) weights quantised on the device; fp16 KV
    cache), driven by the library's own decoder (odi_cuda_decoder_*, the
    C-ABI path a C++ engine calls): the KV cache is filled from 2048 seeded
    random prompt tokens, then DEC_GEN greedy steps are timed on the device
    (CUDA events around the graph replays, inside the library).  The Python
    DecodeModel runs the same steps on the same weights as a cross-check of
    the tokens."""
    import torch

    from odiengine_b200.decode import CDecoder, DecodeModel, LlamaConfig, seeded_model

    dev = torch.device("cuda", local_rank)
    P, G = args.decode_prompt, args.decode_gen
    cfg = LlamaConfig(ctx=P + G + 8)
    t0 = time.perf_counter()
    mw = seeded_model(cfg, seed=0, device=dev)
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t0
    cd = CDecoder(cfg, mw, max_record=G + 16)
    gen = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (P,), generator=gen).tolist()
    t0 = time.perf_counter()
    cd.reset(prompt[0], 0, clear_cache=True)
    cd.prefill(prompt[:-1])
    t_prefill = time.perf_counter() - t0

    def from_prompt_end():
        # the last prompt token at its own position: its argmax is the first
        # generated token
        cd.reset(prompt[-1], P - 1)

    from_prompt_end()
    cd.generate(max(3, args.warmup))  # warm-up steps
    from_prompt_end()
    with ClockSampler(local_rank) as clk:
        clk.wait_first_sample()
        ms = cd.time(G)
    ms_tok = ms / G
    toks = cd.tokens(0, G)
    # end to end: the same G steps through odi_cuda_decoder_generate (one
    # host call: the replays, the G tokens read back, the error words
    # checked), wall clock
    from_prompt_end()
    t0 = time.perf_counter()
    toks2 = cd.generate(G)
    el = time.perf_counter() - t0
    assert toks2 == toks, "decode is not deterministic"
    launches = cd.launches_per_step()
    cd.free()
    # cross-check: the Python-driven DecodeModel on the same weights
    dm = DecodeModel(cfg, mw, device=dev)
    dm.reset(1, 0)
    dm.generate(1)
    dm.clear_cache()
    dm.reset(1, 0)
    dm.capture()
    dm.clear_cache()
    dm.prefill(prompt[:-1])
    dm.reset(prompt[-1], P - 1)
    toks_py = dm.generate(G)
    same = toks_py == toks
    del dm
    wb = cfg.weight_bytes()
    kvb = cfg.kv_bytes(P + G // 2)  # mean cache length read per step
    bytes_tok = wb + kvb
    peak, peak_kind = measured_peak()
    achieved = bytes_tok / (ms_tok * 1e-3) / 1e9
    res = {
        "metric": "7B-shape Q4_K decode tokens/s (1 sequence, greedy)", "value": round(1e3 / ms_tok, 2),
        "unit": "tokens/s", "ms_per_token": round(ms_tok, 4), "higher_is_better": True,
        "path": "odi_cuda_decoder (the library's decode step, captured once and replayed per token from C++)",
        "config": {"workload": f"Llama-2-7B-shape decode, {P} prompt tokens in the fp16 KV cache, then {G} greedy "
                               "steps", "layers": cfg.layers, "hidden": cfg.hidden, "heads": cfg.heads,
                   "head_dim": cfg.head_dim, "ffn": cfg.ffn, "vocab": cfg.vocab,
                   "weights": "Q4_K attention + gate/up, Q6_K down + output, seeded N(0, 0.02)",
                   "l2": "inputs larger than L2: each step streams 4.1 GB of weights"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "bytes_per_token": bytes_tok,
                     "weight_bytes": wb, "kv_bytes_mean": kvb, "peak_kind": peak_kind},
        "e2e": {"value": round(G / el, 2), "unit": "tokens/s", "h2d_bytes_per_step": round(16 / G, 4),
                "d2h_bytes_per_step": 4,
                "call": "odi_cuda_decoder_generate from the prompt's end (16-byte state written once, graph replays, "
                        "the tokens read back and the error words checked at the end)"},
        "python_path_same_tokens": same,
        "gpu_launches_per_token": launches,
        "prefill_s": round(t_prefill, 2), "build_s": round(t_build, 2),
        "first_tokens": toks[:8], "clocks": clk.summary(),
        "cpu_baseline": None,
    }
    if not args.no_cpu:
        nth = host_threads()
        t_cpu, sample = cpu_decode_sample(nth)
        res["cpu_baseline"] = {"value": round(1.0 / t_cpu, 4), "unit": "tokens/s", "cores": nth, "kind": "port",
                               "sample": sample}
    del mw
    torch.cuda.synchronize()
    return res


def cpu_decode_sample(nthreads: int, reps: int = 3):
    """Host-core time of one 7B-shape decode token's matrix products: the
    oracle restatement of the reference loop (the reference's CPUBackend
    throws on K-quants) on one layer's four products (Q4_K QKV 12288x4096,
    O 4096x4096, gate|up 22016x4096; Q6_K down 4096x11008) times 32 layers,
    plus the Q6_K 32000x4096 output product.  Attention, norms and the
    elementwise ops are left out, so this overstates the CPU's speed.
    Returns (seconds per token, sample description)."""
    import oracle as O

    shapes = [(O.Q4_K, 12288, 4096), (O.Q4_K, 4096, 4096), (O.Q4_K, 22016, 4096), (O.Q6_K, 4096, 11008)]
    out = (O.Q6_K, 32000, 4096)

    def best_time(dt, N, K):
        b = O.quantize(dt, O.seeded_weights(N, K, seed=0))
        x = O.seeded_acts(1, K, seed=1)
        O.matmul_ref(dt, x, b, N, nthreads)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            O.matmul_ref(dt, x, b, N, nthreads)
            ts.append(time.perf_counter() - t0)
        return min(ts)

    layer = sum(best_time(*sh) for sh in shapes)
    t = 32 * layer + best_time(*out)
    return t, (f"one layer's 4 products + the output product, best of {reps}, scaled to 32 layers; "
               f"{nthreads} threads; oracle restatement of the reference loop; matrix products only")


TRAFFIC_SOURCE = ("profiles/qgemv_q4k_4096x14336_m1.md: ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                  "launch of this kernel at this shape (bench.py --profile); ncu cannot run inside the timed bench")


def config_summary(configs):
    """The configuration legs in one short dict: HBM fraction per GEMV shape
    and token count, tensor fraction per prefill shape."""
    out = {}
    for r in configs.get("gemv_sweep", []):
        out[f"{r['dtype']} {r['N']}x{r['K']} M{r['M']}"] = r["hbm_frac"]
    for r in configs.get("prefill_gemm", []):
        out[f"prefill {r['N']}x{r['K']} M{r['M']} TF"] = r["tensor_frac"]
    for r in configs.get("gemv_70b", []):
        out[f"70b {r['N']}x{r['K']} M{r['M']}"] = r["hbm_frac"]
    return out


def traffic_per_launch():
    """DRAM bytes per GEMV launch from the committed ncu summary, if any."""
    import re

    path = os.path.join(ROOT, "profiles", "qgemv_q4k_4096x14336_m1.md")
    try:
        with open(path) as f:
            m = re.search(r"^dram_bytes_per_launch = (\d+)", f.read(), re.M)
        return int(m.group(1)) if m else None
    except OSError:
        return None


# Small cases for ncu captures of the other configurations' kernels (one GPU):
# name -> (dtype, N, K, M, act_mode name, what it captures)
PROFILE_CASES = {
    "tc_prefill_m2048": ("Q4_K", 4096, 14336, 2048, "ACT_AUTO", "qgemm_tc_kernel, the tcgen05 prefill GEMM"),
    "gemv8_q6k_4096": ("Q6_K", 4096, 4096, 8, "ACT_AUTO", "qgemv_kernel<Q6_K,8,...>, the 8-token mma.sync GEMV"),
    "gemv8_q4k_14336": ("Q4_K", 4096, 14336, 8, "ACT_AUTO", "qgemv_kernel<Q4_K,8,...>, the 8-token mma.sync GEMV"),
}


def run_profile_case(name, local_rank):
    """Three eager products of one configuration on the device (seeded
    weights quantised on the device, fp32 activations), nothing timed."""
    import torch

    import odiengine_b200 as ob

    dtn, N, K, M, mode, _ = PROFILE_CASES[name]
    torch.cuda.set_device(local_rank)
    ob.init(local_rank)
    dev = torch.device("cuda", local_rank)
    dt = ob.DTYPES[dtn]
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    wf = torch.empty((N, K), dtype=torch.float32, device=dev).normal_(0.0, 0.02, generator=gen)
    w = ob.repack(dt, ob.quantize_weight(dt, wf), N, K)
    del wf
    x = torch.empty((M, K), dtype=torch.float32, device=dev).normal_(0.0, 1.0, generator=gen)
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    am = getattr(ob, mode)
    ws = ob.new_workspace(ob.workspace_bytes(dt, M, N, K, am), dev)
    for _ in range(3):
        ob.matmul_dev(dt, w, x, y, N, K, am, ws)
    torch.cuda.synchronize()
    assert ob.workspace_status(ws) == 0
    print(json.dumps({"profile_case": name, "ok": True}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="leave out the 7B-shape decode tokens/s")
    ap.add_argument("--decode-only", action="store_true", help="run only the 7B-shape decode leg (1 GPU)")
    ap.add_argument("--decode-prompt", type=int, default=DEC_PROMPT, help="prompt tokens in the KV cache")
    ap.add_argument("--decode-gen", type=int, default=DEC_GEN, help="timed greedy steps")
    ap.add_argument("--no-configs", action="store_true",
                    help="leave out the other reference configurations (GEMV sweep, prefill GEMM, 70B shapes)")
    ap.add_argument("--profile", action="store_true", help="small case for ncu: 3 products, no timing")
    ap.add_argument("--profile-case", default=None, choices=list(PROFILE_CASES),
                    help="small case for ncu of another configuration's kernel: 3 products, no timing")
    ap.add_argument("--gather", default="fused", choices=["fused", "nccl"],
                    help="N > 1: gather the row shards from the GEMV epilogue (fused) or with ncclAllGather")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.profile_case:
        return run_profile_case(args.profile_case, local_rank)
    if args.decode_only:
        if world > 1:
            raise SystemExit("--decode-only runs on one GPU")
        import torch

        import odiengine_b200 as ob

        torch.cuda.set_device(local_rank)
        ob.init(local_rank)
        print(json.dumps({"decode_7b": run_decode(args, local_rank)}), flush=True)
        return 0
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
