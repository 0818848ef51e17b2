"""Tensor-core (tcgen05) GEMM path, ODI_CUDA_ACT_F16, against the oracle.

Two checks per output element:
  * vs the restatement of the same arithmetic (oracle.matmul_f16: fp16
    activations, the exact fp16 weight decode, exact products):
        |y - y16| <= 2 (K + 16) 2^-24 sum |x16 w16|     (fp32 summation order)
  * vs the exact real product of the GGUF weights (the reference's matmul up
    to fp32 rounding), oracle.f16_bound (fp16 rounding of both operands).
At the full prefill and batched-decode shapes the reference is computed for
a sample of weight rows (rows are independent outputs).  The shapes cover
every token block (32, 64, 128, 256) and K splits of 1, 2, 4 and 8 CTAs
(cluster reduce-scatter through distributed shared memory).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

TC = [O.Q4_K, O.Q6_K]


def _run(ob, dt, blocks, x, N, K, mode):
    import torch

    t = ob.repack(dt, torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda(), N, K)
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    y = torch.full((x.shape[0], N), float("nan"), dtype=torch.float32, device="cuda")
    ws = ob.new_workspace(ob.workspace_bytes(dt, x.shape[0], N, K, mode))
    ob.matmul_dev(dt, t, xd, y, N, K, mode, ws)
    torch.cuda.synchronize()
    assert ob.workspace_status(ws) == 0
    return y.cpu().numpy()


def _check(dt, x, blocks, N, y, rows=None):
    K = x.shape[1]
    if rows is not None:
        Kb = K // O.BLOCK_ELEMS[dt]
        bb = O.BLOCK_BYTES[dt]
        blocks = np.ascontiguousarray(blocks.reshape(N, Kb * bb)[rows])
        y = y[:, rows]
        N = len(rows)
    assert np.isfinite(y).all()
    y16, b16 = O.matmul_f16(dt, x, blocks, N)
    err16 = np.abs(y.astype(np.float64) - y16)
    assert (err16 <= b16 + 1e-30).all(), f"vs fp16 restatement: max {err16.max()}"
    W = O.dequantize(dt, blocks, N, K).astype(np.float64)
    exact = x.astype(np.float64) @ W.T
    err = np.abs(y.astype(np.float64) - exact)
    assert (err <= O.f16_bound(dt, x, blocks, N)).all(), f"vs exact: max {err.max()}"
    return err.max(), (err / np.maximum(np.abs(x.astype(np.float64)) @ np.abs(W).T, 1e-30)).max()


@pytest.mark.parametrize("dt", TC)
@pytest.mark.parametrize("N,K,M", [(128, 256, 64), (256, 1024, 128), (200, 512, 130), (64, 768, 1),
                                   (1000, 2048, 300), (512, 4096, 16), (4096, 4096, 8), (330, 7936, 40),
                                   (384, 1024, 64)])
def test_tc_small(cuda_lib, dt, N, K, M):
    b = O.quantize(dt, O.seeded_weights(N, K, seed=N))
    x = O.seeded_acts(M, K, seed=K)
    y = _run(cuda_lib, dt, b, x, N, K, cuda_lib.ACT_F16)
    _check(dt, x, b, N, y)


@pytest.mark.parametrize("dt", TC)
@pytest.mark.parametrize("N,K,M", [(14336, 4096, 512), (4096, 14336, 512), (14336, 4096, 2048),
                                   (4096, 14336, 2048), (28672, 8192, 32), (8192, 28672, 32)])
def test_tc_prefill_shapes(cuda_lib, dt, N, K, M):
    b = O.quantize(dt, O.seeded_weights(N, K, seed=0))
    x = O.seeded_acts(M, K, seed=1)
    y = _run(cuda_lib, dt, b, x, N, K, cuda_lib.ACT_F16)
    rows = np.random.default_rng(5).choice(N, size=96, replace=False)
    rows = np.unique(np.concatenate([rows, [0, 127, 128, N - 1]]))
    assert np.isfinite(y).all()
    _check(dt, x, b, N, y, rows=rows)


@pytest.mark.parametrize("dt", TC)
def test_tc_deterministic_and_auto_mode(cuda_lib, dt):
    N, K = 384, 1024
    b = O.quantize(dt, O.seeded_weights(N, K, seed=3))
    x = O.seeded_acts(cuda_lib.TC_MIN_TOKENS, K, seed=4)
    y1 = _run(cuda_lib, dt, b, x, N, K, cuda_lib.ACT_F16)
    y2 = _run(cuda_lib, dt, b, x, N, K, cuda_lib.ACT_F16)
    ya = _run(cuda_lib, dt, b, x, N, K, cuda_lib.ACT_AUTO)
    assert np.array_equal(y1, y2) and np.array_equal(y1, ya)
    xs = x[: cuda_lib.TC_MIN_TOKENS - 1]
    assert np.array_equal(_run(cuda_lib, dt, b, xs, N, K, cuda_lib.ACT_AUTO),
                          _run(cuda_lib, dt, b, xs, N, K, cuda_lib.ACT_Q8))


def test_tc_unsupported_dtype_refused(cuda_lib):
    import torch

    ob = cuda_lib
    N, K, M = 64, 256, 64
    b = O.quantize(O.Q8_0, O.seeded_weights(N, K))
    t = ob.repack(O.Q8_0, torch.from_numpy(b.reshape(-1)).cuda(), N, K)
    x = torch.zeros((M, K), device="cuda")
    y = torch.zeros((M, N), device="cuda")
    ws = ob.new_workspace(1 << 20)
    with pytest.raises(ob.OdiCudaError, match="no tensor-core path"):
        ob.matmul_dev(O.Q8_0, t, x, y, N, K, ob.ACT_F16, ws)
    assert ob.lib().odi_cuda_tc_supported(O.Q4_K) == 1 and ob.lib().odi_cuda_tc_supported(O.Q8_0) == 0
