"""Every configuration the benchmark times, at its full size, every output
element checked against the oracle through the C ABI.

* The 7B decode GEMV sweep: Q8_0 / Q4_K / Q6_K at 4096x4096, 11008x4096,
  4096x11008 and 32000x4096, M = 1 (on-chip Q8_0 staging, dp4a units) and
  M = 8 (Q8 records, one 8-token pass on the mma.sync units), both through
  ODI_CUDA_ACT_AUTO as the benchmark calls them.  Tolerance: the Q8 bounds
  of tests/test_gpu_parity.py (vs the oracle's integer-block restatement
  2 (K/8 + 64) 2^-24 sum|block terms|, and vs the reference's fp32 loop
  Bact + B32 + that term).
* The tensor-core prefill GEMM: Q4_K 14336x4096 and 4096x14336 at M = 512
  and 2048, every row.
* The 70B decode shapes at M = 32 through ODI_CUDA_ACT_AUTO (the tcgen05
  path): Q4_K 28672x8192, 8192x28672 and 128256x8192, every row.
  Tolerance for both tensor-core groups: vs the oracle's fp16 restatement
  2 (K + 16) 2^-24 sum|x16 w16|, and vs the exact product oracle.f16_bound
  (the fp16 rounding of both operands), as in tests/test_gpu_tc.py.

The reference loop these restate is matmul_q4_0 / matmul_q8_0
(src/compute/cpu/cpu_backend.cpp:786-854): per output row, blocks in order,
fp32 accumulation.  Rows are independent outputs, so the oracle runs over row
chunks on all host threads; weights are made on the device (seeded normal
draws, the device quantiser, bit-exact with the oracle's by
test_quantize_weight_bit_exact) and copied back for the oracle.
"""
import concurrent.futures as cf

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _weights(ob, dt, N, K, seed):
    """Seeded N(0, 0.02) weights quantised on the device: (tiled device
    weight, host GGUF blocks [N, row bytes])."""
    import torch

    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    wf = torch.empty((N, K), dtype=torch.float32, device="cuda").normal_(0.0, 0.02, generator=gen)
    blocks = ob.quantize_weight(dt, wf)
    del wf
    tiled = ob.repack(dt, blocks, N, K)
    host = blocks.cpu().numpy().reshape(N, -1)
    del blocks
    return tiled, host


def _product(ob, dt, tiled, x, N, K, mode):
    import torch

    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    y = torch.full((x.shape[0], N), float("nan"), dtype=torch.float32, device="cuda")
    ws = ob.new_workspace(ob.workspace_bytes(dt, x.shape[0], N, K, mode))
    ob.matmul_dev(dt, tiled, xd, y, N, K, mode, ws)
    torch.cuda.synchronize()
    assert ob.workspace_status(ws) == 0
    return y.cpu().numpy()


def _check_q8(dt, x, b, y):
    N = b.shape[0]
    K = x.shape[1]
    assert np.isfinite(y).all()
    yq, bact, mag = O.matmul_q8act(dt, x, b, N, with_mag=True)
    reorder = 2.0 * (K / 8 + 64) * 2.0 ** -24 * mag.astype(np.float64)
    err = np.abs(y.astype(np.float64) - yq)
    bad = err > reorder
    assert not bad.any(), f"vs q8 restatement: {bad.sum()} outputs, max err {err.max()}"
    ref = O.matmul_ref(dt, x, b, N)
    b32 = O.fp32_bound(dt, x, b, N)
    err_ref = np.abs(y.astype(np.float64) - ref)
    bad = err_ref > bact + b32 + reorder
    assert not bad.any(), f"vs reference loop: {bad.sum()} outputs, max err {err_ref.max()}"


def _check_f16_rows(dt, x, b, y, chunk=2048):
    """Every row of a tensor-core product, in row chunks on a thread pool
    (the oracle's C loops and numpy's matmul release the GIL)."""
    N, K = b.shape[0], x.shape[1]
    x64 = x.astype(np.float64)
    assert np.isfinite(y).all()

    def one(n0):
        bc = np.ascontiguousarray(b[n0:n0 + chunk])
        n = bc.shape[0]
        yc = y[:, n0:n0 + n].astype(np.float64)
        y16, b16 = O.matmul_f16(dt, x, bc, n)
        e16 = np.abs(yc - y16)
        W = O.dequantize(dt, bc, n, K).astype(np.float64)
        e = np.abs(yc - x64 @ W.T)
        fb = O.f16_bound(dt, x, bc, n)
        return int((e16 > b16 + 1e-30).sum()), int((e > fb).sum()), float(e16.max()), float(e.max())

    with cf.ThreadPoolExecutor(4) as ex:
        res = list(ex.map(one, range(0, N, chunk)))
    assert sum(r[0] for r in res) == 0, f"vs fp16 restatement: max err {max(r[2] for r in res)}"
    assert sum(r[1] for r in res) == 0, f"vs exact product: max err {max(r[3] for r in res)}"


SWEEP = [(N, K) for N, K in ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096))]


@pytest.mark.parametrize("dt", [O.Q8_0, O.Q4_K, O.Q6_K], ids=["Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("N,K", SWEEP)
@pytest.mark.parametrize("M", [1, 8])
def test_decode_sweep_full(cuda_lib, dt, N, K, M):
    ob = cuda_lib
    tiled, b = _weights(ob, dt, N, K, seed=N + K + M)
    x = O.seeded_acts(M, K, seed=M + 1)
    y = _product(ob, dt, tiled, x, N, K, ob.ACT_AUTO)
    _check_q8(dt, x, b, y)


@pytest.mark.parametrize("N,K", [(14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("M", [512, 2048])
def test_prefill_all_rows(cuda_lib, N, K, M):
    ob = cuda_lib
    dt = O.Q4_K
    tiled, b = _weights(ob, dt, N, K, seed=0)
    x = O.seeded_acts(M, K, seed=1)
    y = _product(ob, dt, tiled, x, N, K, ob.ACT_AUTO)
    _check_f16_rows(dt, x, b, y)


@pytest.mark.parametrize("N,K", [(28672, 8192), (8192, 28672), (128256, 8192)])
def test_70b_m32_all_rows(cuda_lib, N, K):
    ob = cuda_lib
    dt = O.Q4_K
    tiled, b = _weights(ob, dt, N, K, seed=7)
    x = O.seeded_acts(32, K, seed=2)
    y = _product(ob, dt, tiled, x, N, K, ob.ACT_AUTO)
    _check_f16_rows(dt, x, b, y)


@pytest.mark.parametrize("N,K", [(28672, 8192), (8192, 28672)])
def test_70b_m32_q8_passes(cuda_lib, N, K):
    """The same 70B shapes at 32 tokens on the streaming GEMV (ACT_Q8: four
    passes of 8 tokens over the Q8 records), every output."""
    ob = cuda_lib
    dt = O.Q4_K
    tiled, b = _weights(ob, dt, N, K, seed=11)
    x = O.seeded_acts(32, K, seed=3)
    y = _product(ob, dt, tiled, x, N, K, ob.ACT_Q8)
    _check_q8(dt, x, b, y)
