"""Row-sharded product over several ranks (odiengine_b200.sharded).

CPU: world-size-2 and -3 gloo ranks (spawned processes) run the sharding and
the all-gather with the oracle's restated product as each rank's local
compute; the gathered [M, N] must equal the oracle's full product bit for
bit (rows are independent, so sharding changes no arithmetic), for even and
ragged N and for M = 1 and M > 1 (the rank-major permute).
GPU: with two or more devices, two NCCL ranks run the CUDA product on their
shards and must reproduce the single-GPU result up to fp32 summation order
(the work split depends on the shard's row count); the fused scatter (peer
stores from the GEMV epilogue, arrival counters, bounded wait) must equal
the NCCL all-gather bit for bit over repeated calls.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O
from odiengine_b200.sharded import shard_rows

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shard_rows_cover_exactly():
    for N in (1, 7, 64, 4096, 28672, 128256, 1001):
        for g in (1, 2, 3, 4, 8):
            spans = [shard_rows(N, g, r) for r in range(g)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            for (lo, hi, S), (lo2, _, _) in zip(spans, spans[1:]):
                assert hi == lo2 and hi - lo <= S
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def _oracle_local(dtype, blocks, x, rows, K):
    import torch

    y = O.matmul_ref(dtype, x.numpy(), blocks, rows)
    return torch.from_numpy(y)


def _cpu_worker(rank, world, port, cases, out_q):
    import torch.distributed as dist
    import torch

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from odiengine_b200.sharded import RowShardedWeight

        for dt, N, K, M in cases:
            b = O.quantize(dt, O.seeded_weights(N, K, seed=N + K))
            x = torch.from_numpy(O.seeded_acts(M, K, seed=M))
            w = RowShardedWeight(dt, N, K, local_fn=_oracle_local).load(b)
            y = w.matmul(x)
            if rank == 0:
                out_q.put((dt, N, K, M, y.numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_gather_on_cpu_ranks(world):
    import torch.multiprocessing as mp

    cases = [(O.Q4_K, 256, 512, 1), (O.Q4_K, 200, 512, 3), (O.Q8_0, 97, 64, 2), (O.Q6_K, 130, 256, 5)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cpu_worker, args=(r, world, port, cases, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in cases]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for dt, N, K, M, y in results:
        b = O.quantize(dt, O.seeded_weights(N, K, seed=N + K))
        ref = O.matmul_ref(dt, O.seeded_acts(M, K, seed=M), b, N)
        assert y.shape == (M, N)
        assert np.array_equal(y, ref), (dt, N, K, M)


def _gpu_worker(rank, world, port, out_q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    import odiengine_b200 as ob

    ob.init(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from odiengine_b200.sharded import RowShardedWeight

        res = []
        for dt, N, K, M, mode in [(O.Q4_K, 1024, 2048, 1, ob.ACT_Q8), (O.Q4_K, 1000, 2048, 32, ob.ACT_AUTO),
                                  (O.Q6_K, 512, 1024, 3, ob.ACT_Q8)]:
            b = O.quantize(dt, O.seeded_weights(N, K, seed=1))
            x = torch.from_numpy(O.seeded_acts(M, K, seed=2)).cuda()
            w = RowShardedWeight(dt, N, K).load(b)
            y = w.matmul(x, act_mode=mode)
            torch.cuda.synchronize()
            res.append(y.cpu().numpy())
        # fused scatter (GEMV epilogue stores to every rank + counters) must
        # give exactly the NCCL all-gather result, call after call
        fused_ok = []
        for dt, N, K, M in [(O.Q4_K, 1024, 2048, 1), (O.Q6_K, 1000, 1024, 4), (O.Q4_K, 130, 512, 8)]:
            b = O.quantize(dt, O.seeded_weights(N, K, seed=3))
            wn = RowShardedWeight(dt, N, K).load(b)
            wf = RowShardedWeight(dt, N, K, fused=True).load(b)
            for call in range(4):
                x = torch.from_numpy(O.seeded_acts(M, K, seed=10 + call)).cuda()
                yn = wn.matmul(x, act_mode=ob.ACT_Q8).cpu()
                yf = wf.matmul(x, act_mode=ob.ACT_Q8).cpu()
                fused_ok.append(bool(torch.equal(yn, yf)))
            wf.sym.close()
        res.append(fused_ok)
        if rank == 0:
            out_q.put(res)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_sharded_two_gpus_match_one():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import odiengine_b200 as ob

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_worker, args=(r, 2, port, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=300)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    assert all(got[-1]), got[-1]
    got = got[:-1]
    ob.init(0)
    torch.cuda.set_device(0)
    for (dt, N, K, M, mode), y in zip([(O.Q4_K, 1024, 2048, 1, ob.ACT_Q8), (O.Q4_K, 1000, 2048, 32, ob.ACT_AUTO),
                                       (O.Q6_K, 512, 1024, 3, ob.ACT_Q8)], got):
        b = O.quantize(dt, O.seeded_weights(N, K, seed=1))
        dw = ob.DeviceWeight(ob.QuantWeight(dt, (K, N), b))
        ref = dw.matmul(torch.from_numpy(O.seeded_acts(M, K, seed=2)).cuda(), act_mode=mode).cpu().numpy()
        # the work split (K chunks per cluster) depends on the row count, so
        # shard and whole differ only by fp32 summation order: both lie within
        # the reordering bound of the restated arithmetic
        xs = O.seeded_acts(M, K, seed=2)
        if mode == ob.ACT_AUTO and M >= ob.TC_MIN_TOKENS:
            _, bound = O.matmul_f16(dt, xs, b, N)
        else:
            _, _, mag = O.matmul_q8act(dt, xs, b, N, with_mag=True)
            bound = 2.0 * (K / 8 + 64) * 2.0 ** -24 * mag.astype(np.float64)
        assert (np.abs(y.astype(np.float64) - ref) <= 2 * bound + 1e-30).all()


# --------------------------------------------------------------------------
# The C-ABI sharded product (odi_cuda_nccl_* / odi_cuda_matmul_sharded): what a
# C++ Backend calls to shard without Python
# --------------------------------------------------------------------------
def _capi_shard_weight(ob, dt, blocks, N, K, world, rank):
    """This rank's S-row tiled weight on the device: its GGUF block-rows, the
    last rank's padded with zero rows."""
    import torch

    from odiengine_b200.sharded import shard_blocks, shard_rows

    _, _, S = shard_rows(N, world, rank)
    mine = shard_blocks(blocks, dt, N, K, world, rank)
    pad = np.zeros(S * ob.gguf_bytes(dt, 1, K), np.uint8)
    pad[: mine.size] = mine
    return ob.repack(dt, torch.from_numpy(pad).cuda(), S, K), S


def _capi_product(ob, comm, dt, w, x, N, S, K, mode):
    import torch

    L = ob.lib()
    M = x.shape[0]
    y = torch.full((M, N), float("nan"), device="cuda")
    ws = ob.new_workspace(L.odi_cuda_sharded_workspace_bytes(comm, dt, M, S, K, mode))
    ob.check(L.odi_cuda_matmul_sharded(comm, dt, w.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, S, K, mode,
                                       ws.data_ptr(), ws.numel(), 0, None))
    torch.cuda.synchronize()
    assert ob.workspace_status(ws) == 0
    return y.cpu().numpy()


CAPI_CASES = [(O.Q4_K, 1024, 2048, 1, 0), (O.Q6_K, 512, 1024, 3, 0), (O.Q4_K, 1000, 2048, 32, 3)]


@pytest.mark.gpu
def test_capi_sharded_one_rank_equals_plain_product(cuda_lib):
    """A one-rank communicator: the sharded product is the plain product bit
    for bit (the all-gather is in place; M > 1 goes through the unshard
    kernel)."""
    import ctypes

    import torch

    ob = cuda_lib
    L = ob.lib()
    uid = ctypes.create_string_buffer(128)
    ob.check(L.odi_cuda_nccl_unique_id(uid))
    comm = ctypes.c_void_p()
    ob.check(L.odi_cuda_nccl_init(uid, 1, 0, ctypes.byref(comm)))
    try:
        n, r = ctypes.c_int(), ctypes.c_int()
        ob.check(L.odi_cuda_comm_ranks(comm, ctypes.byref(n), ctypes.byref(r)))
        assert (n.value, r.value) == (1, 0)
        for dt, N, K, M, mode in CAPI_CASES:
            b = O.quantize(dt, O.seeded_weights(N, K, seed=1))
            w, S = _capi_shard_weight(ob, dt, b, N, K, 1, 0)
            x = torch.from_numpy(O.seeded_acts(M, K, seed=2)).cuda()
            y = _capi_product(ob, comm, dt, w, x, N, S, K, mode)
            ref = torch.empty((M, N), device="cuda")
            ob.matmul_dev(dt, w, x, ref, N, K, mode)
            torch.cuda.synchronize()
            assert np.array_equal(y.view(np.uint32), ref.cpu().numpy().view(np.uint32)), (dt, N, K, M)
        # a split that does not cover N is refused
        with pytest.raises(ob.OdiCudaError, match="does not split"):
            ob.check(L.odi_cuda_matmul_sharded(comm, O.Q4_K, 16, 16, 16, 1, 1024, 512, 2048, 0, 16, 1 << 20, 0,
                                               None))
    finally:
        ob.check(L.odi_cuda_nccl_free(comm))


def _capi_worker(rank, world, uid_bytes, out_q):
    import ctypes

    import torch

    torch.cuda.set_device(rank)
    import odiengine_b200 as ob

    ob.init(rank)
    L = ob.lib()
    uid = ctypes.create_string_buffer(bytes(uid_bytes), 128)
    comm = ctypes.c_void_p()
    ob.check(L.odi_cuda_nccl_init(uid, world, rank, ctypes.byref(comm)))
    try:
        res = []
        for dt, N, K, M, mode in CAPI_CASES:
            b = O.quantize(dt, O.seeded_weights(N, K, seed=1))
            w, S = _capi_shard_weight(ob, dt, b, N, K, world, rank)
            x = torch.from_numpy(O.seeded_acts(M, K, seed=2)).cuda()
            res.append(_capi_product(ob, comm, dt, w, x, N, S, K, mode))
        if rank == 0:
            out_q.put(res)
    finally:
        ob.check(L.odi_cuda_nccl_free(comm))


@pytest.mark.gpu
def test_capi_sharded_two_gpus():
    """Two processes, one GPU each, a communicator made from one rank's id:
    every rank's gathered product lies within the oracle's bound (the shard's
    work split differs from the whole weight's, so only the fp32 summation
    order differs)."""
    import ctypes

    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import odiengine_b200 as ob

    uid = ctypes.create_string_buffer(128)
    ob.check(ob.lib().odi_cuda_nccl_unique_id(uid))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    # daemon children: a rank that never joins cannot keep pytest alive
    procs = [ctx.Process(target=_capi_worker, args=(r, 2, uid.raw, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=300)
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    for (dt, N, K, M, mode), y in zip(CAPI_CASES, got):
        b = O.quantize(dt, O.seeded_weights(N, K, seed=1))
        xs = O.seeded_acts(M, K, seed=2)
        if mode == 3 and M >= 9:
            y16, bound = O.matmul_f16(dt, xs, b, N)
            assert (np.abs(y.astype(np.float64) - y16) <= bound + 1e-30).all()
        else:
            yq, _, mag = O.matmul_q8act(dt, xs, b, N, with_mag=True)
            bound = 2.0 * (K / 8 + 64) * 2.0 ** -24 * mag.astype(np.float64)
            assert (np.abs(y.astype(np.float64) - yq) <= bound + 1e-30).all()


@pytest.mark.gpu
def test_capi_nccl_init_failure_injected():
    """A communicator that cannot form (host-side injection,
    ODI_CUDA_INJECT=nccl, in a child process) is reported as
    ODI_CUDA_ERR_BACKEND_INIT_FAILED (odi_error_t 301), with nothing left
    half-made."""
    import subprocess
    import sys

    code = (
        "import ctypes, sys; sys.path.insert(0, %r)\n"
        "import odiengine_b200 as ob\n"
        "L = ob.lib(); ob.init(0)\n"
        "uid = ctypes.create_string_buffer(128); ob.check(L.odi_cuda_nccl_unique_id(uid))\n"
        "c = ctypes.c_void_p(); rc = L.odi_cuda_nccl_init(uid, 1, 0, ctypes.byref(c))\n"
        "print(rc, c.value, L.odi_cuda_last_error().decode())\n" % ROOT)
    env = dict(os.environ, ODI_CUDA_INJECT="nccl")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rc, ptr, msg = r.stdout.strip().split(" ", 2)
    assert rc == "301" and ptr == "None" and "ODI_CUDA_INJECT=nccl" in msg
