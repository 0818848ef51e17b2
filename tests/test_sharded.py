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
    procs = [ctx.Process(target=_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
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
