"""Parity of the sm_100a kernels with the oracle, through the C ABI.

* packing / unpacking / activation quantisation: bit-exact;
* ACT_F32 product vs the reference arithmetic (oracle restatement, itself
  bit-exact with the reference for Q4_0/Q8_0):
      |y - y_ref| <= 2 * B32,  B32 = 2*(K+16)*2^-24 * sum_k |x_k|*|w_k|
  (both are fp32 evaluations of the same sum; B32 bounds each against the
  exact value);
* ACT_Q8 product vs the oracle's Q8 restatement (same integer block dots):
      |y - y_q8| <= 2*(K/8+64)*2^-24 * sum|block terms|
  and vs the reference fp32 product:
      |y - y_ref| <= Bact + B32 + (the reordering term above)
  where Bact = sum_b 0.5625*d_x,b * sum_{k in b} |w_k| bounds the activation
  quantisation error (d_x the block's fp16 scale).
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

LEGACY = [O.Q4_1, O.Q5_0, O.Q5_1]
ALL = [O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K] + LEGACY
U24 = 2.0 ** -24


def to_dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def upload(ob, dt, blocks, N, K):
    return ob.repack(dt, to_dev(blocks.reshape(-1)), N, K)


def run_matmul(ob, dt, w_tiled, x, N, K, mode, flags=0, ws=None):
    import torch

    xd = to_dev(x.astype(np.float32))
    y = torch.full((x.shape[0], N), float("nan"), dtype=torch.float32, device="cuda")
    if ws is None:
        ws = ob.new_workspace(ob.workspace_bytes(dt, x.shape[0], N, K, mode))
    ob.matmul_dev(dt, w_tiled, xd, y, N, K, mode, ws, flags)
    torch.cuda.synchronize()
    assert ob.workspace_status(ws) == 0
    return y.cpu().numpy(), ws


def make(dt, N, K, seed=0, M=1):
    Kw = (K + O.BLOCK_ELEMS[dt] - 1) // O.BLOCK_ELEMS[dt] * O.BLOCK_ELEMS[dt]
    w = O.seeded_weights(N, Kw, seed=seed)
    b = O.quantize(dt, w)
    x = O.seeded_acts(M, K, seed=seed + 1)
    return b, x


# --------------------------------------------------------------------------
# layout
# --------------------------------------------------------------------------
@pytest.mark.parametrize("dt", ALL)
@pytest.mark.parametrize("N,K", [(1, 256), (65, 512), (130, 768), (256, 4096)])
def test_repack_bit_exact(cuda_lib, dt, N, K):
    b, _ = make(dt, N, K)
    t = upload(cuda_lib, dt, b, N, K).cpu().numpy()
    assert np.array_equal(t, O.repack(dt, b, N, K))
    back = cuda_lib.unpack(dt, to_dev(t), N, K).cpu().numpy()
    assert np.array_equal(back, b.reshape(-1))


@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0] + LEGACY)
@pytest.mark.parametrize("K", [32, 80, 300])
def test_repack_ragged_bit_exact(cuda_lib, dt, K):
    b, _ = make(dt, 70, K)
    t = upload(cuda_lib, dt, b, 70, K).cpu().numpy()
    assert np.array_equal(t, O.repack(dt, b, 70, K))


@pytest.mark.parametrize("dt", ALL)
def test_dequantize_bit_exact(cuda_lib, dt):
    N, K = 96, 768
    b, _ = make(dt, N, K, seed=3)
    t = upload(cuda_lib, dt, b, N, K)
    got = cuda_lib.dequantize_dev(dt, t, N, K).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), O.dequantize(dt, b, N, K).view(np.uint32))


def test_dequantize_golden(cuda_lib, golden):
    for dt, name in ((O.Q4_K, "q4k"), (O.Q5_K, "q5k"), (O.Q6_K, "q6k")):
        rb = golden[f"{name}_rand_bytes"]
        t = upload(cuda_lib, dt, rb, rb.shape[0], 256)
        got = cuda_lib.dequantize_dev(dt, t, rb.shape[0], 256).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), golden[f"{name}_rand_dequant"].view(np.uint32))
    # Q4_1 / Q5_0 / Q5_1: gguf's decode and the reference's own dequantize, bit for bit
    N, K = golden["w"].shape
    for dt, name in ((O.Q4_1, "q4_1"), (O.Q5_0, "q5_0"), (O.Q5_1, "q5_1")):
        b = golden[f"{name}_bytes"]
        got = cuda_lib.dequantize_dev(dt, upload(cuda_lib, dt, b, N, K), N, K).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), golden[f"{name}_dequant"].view(np.uint32))
        assert np.array_equal(got.view(np.uint32), golden[f"ref_{name}_dequant"].view(np.uint32))


@pytest.mark.parametrize("dt", ALL)
@pytest.mark.parametrize("N,K", [(3, 256), (70, 512), (257, 1024)])
def test_quantize_weight_bit_exact(cuda_lib, dt, N, K):
    w = O.seeded_weights(N, K, seed=N * K)
    w[0, :32] = 0.0  # an all-zero block
    got = cuda_lib.quantize_weight(dt, to_dev(w)).cpu().numpy()
    assert np.array_equal(got, O.quantize(dt, w).reshape(-1))


def test_quantize_weight_golden(cuda_lib, golden):
    w = golden["w"]
    for dt, name in ((O.Q4_0, "q4_0"), (O.Q8_0, "q8_0"), (O.Q4_K, "q4k"), (O.Q5_K, "q5k"), (O.Q6_K, "q6k"),
                     (O.Q4_1, "q4_1"), (O.Q5_0, "q5_0"), (O.Q5_1, "q5_1")):
        got = cuda_lib.quantize_weight(dt, to_dev(w)).cpu().numpy()
        assert np.array_equal(got, golden[f"{name}_bytes"].reshape(-1))


# --------------------------------------------------------------------------
# activation quantisation
# --------------------------------------------------------------------------
@pytest.mark.parametrize("M,K", [(1, 4096), (3, 512), (2, 80), (5, 14336), (1, 33)])
def test_quantize_q8_0_bit_exact(cuda_lib, M, K):
    rng = np.random.default_rng(M * 1000 + K)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    x[0, : min(K, 32)] = 0.0  # an all-zero block (d = 0)
    if K > 64:
        x[0, 40] = 1e30  # huge value
        x[-1, 64:] *= 1e-30  # tiny values
    got = cuda_lib.quantize_q8_0(to_dev(x)).cpu().numpy()
    assert np.array_equal(got, O.quantize_q8_0_act(x))


def test_quantize_q8_0_golden(cuda_lib, golden):
    got = cuda_lib.quantize_q8_0(to_dev(golden["x"])).cpu().numpy()
    assert np.array_equal(got, golden["act_q8_0_bytes"])


def test_quantize_q8_0_ties_round_half_away(cuda_lib):
    # amax = 127 -> d = 1, id = 1: x*id are exact halves
    x = np.zeros((1, 32), np.float32)
    x[0, 0] = 127.0
    x[0, 1:9] = [2.5, -2.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5]
    got = cuda_lib.quantize_q8_0(to_dev(x)).cpu().numpy()
    assert np.array_equal(got, O.quantize_q8_0_act(x))
    q = got[0, 2:].view(np.int8)
    assert list(q[1:9]) == [3, -3, 1, -1, 2, -2, 127, -127]


# --------------------------------------------------------------------------
# the product
# --------------------------------------------------------------------------
def check_f32(dt, x, b, N, y):
    ref = O.matmul_ref(dt, x, b, N)
    bound = O.fp32_bound(dt, x, b, N)
    err = np.abs(y.astype(np.float64) - ref)
    assert np.isfinite(y).all()
    assert (err <= 2.0 * bound).all(), f"max err {err.max()} bound {bound.min()}"
    return err


def check_q8(dt, x, b, N, y):
    K = x.shape[1]
    yq, bact, mag = O.matmul_q8act(dt, x, b, N, with_mag=True)
    reorder = 2.0 * (K / 8 + 64) * U24 * mag.astype(np.float64)
    err = np.abs(y.astype(np.float64) - yq)
    assert np.isfinite(y).all()
    assert (err <= reorder).all(), f"vs q8 restatement: max err {err.max()}"
    ref = O.matmul_ref(dt, x, b, N)
    b32 = O.fp32_bound(dt, x, b, N)
    err_ref = np.abs(y.astype(np.float64) - ref)
    assert (err_ref <= bact + b32 + reorder).all()
    return err_ref


SMALL = [(1, 256), (33, 512), (64, 256), (100, 1280), (257, 2048)]


@pytest.mark.parametrize("dt", ALL)
@pytest.mark.parametrize("N,K", SMALL)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 7, 8])
def test_matmul_q8_small(cuda_lib, dt, N, K, M):
    b, x = make(dt, N, K, seed=N + K + M, M=M)
    t = upload(cuda_lib, dt, b, N, K)
    y, _ = run_matmul(cuda_lib, dt, t, x, N, K, cuda_lib.ACT_Q8)
    check_q8(dt, x, b, N, y)


@pytest.mark.parametrize("dt", ALL)
@pytest.mark.parametrize("N,K", SMALL)
@pytest.mark.parametrize("M", [1, 3, 8])
def test_matmul_f32_small(cuda_lib, dt, N, K, M):
    b, x = make(dt, N, K, seed=N + K + M, M=M)
    t = upload(cuda_lib, dt, b, N, K)
    y, _ = run_matmul(cuda_lib, dt, t, x, N, K, cuda_lib.ACT_F32)
    check_f32(dt, x, b, N, y)


@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0] + LEGACY)
@pytest.mark.parametrize("K", [32, 80, 300, 4000])
@pytest.mark.parametrize("mode", [0, 1])
def test_matmul_ragged_k(cuda_lib, dt, K, mode):
    N = 70
    b, x = make(dt, N, K, seed=K, M=2)
    t = upload(cuda_lib, dt, b, N, K)
    y, _ = run_matmul(cuda_lib, dt, t, x, N, K, mode)
    (check_f32 if mode else check_q8)(dt, x, b, N, y)


def test_matmul_golden_reference_outputs(cuda_lib, golden):
    """Against the unmodified reference CPUBackend::matmul outputs."""
    x = golden["x"]
    for dt, name in ((O.Q4_0, "q4_0"), (O.Q8_0, "q8_0")):
        b = golden[f"{name}_bytes"]
        N, K = golden["w"].shape
        t = upload(cuda_lib, dt, b, N, K)
        y, _ = run_matmul(cuda_lib, dt, t, x, N, K, cuda_lib.ACT_F32)
        ref = golden[f"ref_{name}_y"]
        bound = O.fp32_bound(dt, x, b, N)
        assert (np.abs(y - ref) <= 2 * bound).all()
    xr = golden["ragged_x"]
    for dt, name in ((O.Q4_0, "q4_0"), (O.Q8_0, "q8_0")):
        b = golden[f"ragged_{name}_bytes"]
        t = upload(cuda_lib, dt, b, 8, 80)
        y, _ = run_matmul(cuda_lib, dt, t, xr, 8, 80, cuda_lib.ACT_F32)
        bound = O.fp32_bound(dt, xr, b, 8)
        assert (np.abs(y - golden[f"ragged_ref_{name}_y"]) <= 2 * bound).all()


@pytest.mark.parametrize("dt", [O.Q4_K, O.Q8_0, O.Q6_K, O.Q5_K, O.Q4_0])
@pytest.mark.parametrize("M", [9, 13, 16, 32])
def test_matmul_multi_pass_tokens(cuda_lib, dt, M):
    N, K = 192, 1024
    b, x = make(dt, N, K, seed=M, M=M)
    t = upload(cuda_lib, dt, b, N, K)
    y, _ = run_matmul(cuda_lib, dt, t, x, N, K, cuda_lib.ACT_Q8)
    check_q8(dt, x, b, N, y)


# Llama-2-7B decode shapes (out x in) and the 4096 x 14336 headline shape.
FULL = [(O.Q4_K, 4096, 14336), (O.Q4_K, 4096, 4096), (O.Q4_K, 11008, 4096), (O.Q8_0, 4096, 4096),
        (O.Q8_0, 4096, 11008), (O.Q6_K, 32000, 4096), (O.Q6_K, 4096, 11008), (O.Q4_0, 4096, 4096),
        (O.Q5_K, 4096, 4096), (O.Q4_1, 4096, 4096), (O.Q5_0, 4096, 4096), (O.Q5_1, 4096, 11008),
        # Llama-3-70B shapes (clusters of 2 with 16-span chunks, multi-wave grids)
        (O.Q4_K, 128256, 8192), (O.Q4_K, 28672, 8192), (O.Q4_K, 8192, 28672)]


@pytest.mark.parametrize("dt,N,K", FULL)
@pytest.mark.parametrize("mode", [0, 1])
def test_matmul_full_size(cuda_lib, dt, N, K, mode):
    b, x = make(dt, N, K, seed=5, M=1)
    t = upload(cuda_lib, dt, b, N, K)
    y, _ = run_matmul(cuda_lib, dt, t, x, N, K, mode)
    (check_f32 if mode else check_q8)(dt, x, b, N, y)


def test_deterministic_and_pdl_identical(cuda_lib):
    dt, N, K = O.Q4_K, 4096, 14336
    b, x = make(dt, N, K, seed=9, M=1)
    t = upload(cuda_lib, dt, b, N, K)
    y1, ws = run_matmul(cuda_lib, dt, t, x, N, K, 0)
    y2, _ = run_matmul(cuda_lib, dt, t, x, N, K, 0, ws=ws)
    y3, _ = run_matmul(cuda_lib, dt, t, x, N, K, 0, flags=cuda_lib.FLAG_PDL, ws=ws)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    assert np.array_equal(y1.view(np.uint32), y3.view(np.uint32))


def test_zero_activations_give_zero(cuda_lib):
    dt, N, K = O.Q4_K, 128, 512
    b, _ = make(dt, N, K)
    t = upload(cuda_lib, dt, b, N, K)
    for mode in (0, 1):
        y, _ = run_matmul(cuda_lib, dt, t, np.zeros((2, K), np.float32), N, K, mode)
        assert (y == 0).all()


# --------------------------------------------------------------------------
# the Backend mirror (host buffers, reference argument semantics)
# --------------------------------------------------------------------------
def test_backend_matmul_host(cuda_lib):
    ob = cuda_lib
    be = ob.CudaBackend(0, act_mode=ob.ACT_F32)
    assert be.name() == "CUDA" and be.supports_dtype(ob.ODI_DTYPE_Q4_K)
    assert "sm_10" in be.device_info()
    N, K = 300, 1024
    for dt in ALL:
        b, x = make(dt, N, K, seed=dt, M=3)
        w = ob.QuantWeight(dt, (K, N), b)
        out = np.zeros((3, N), np.float32)
        be.matmul(out, x, w)
        check_f32(dt, x, b, N, out)
        out2 = np.zeros((3, N), np.float32)
        be.quantized_matmul(out2, x, w)
        assert np.array_equal(out, out2)
        deq = np.zeros((N, K), np.float32)
        be.dequantize(deq, w)
        assert np.array_equal(deq.view(np.uint32), O.dequantize(dt, b, N, K).view(np.uint32))
    be.sync()


def test_backend_errors(cuda_lib):
    ob = cuda_lib
    be = ob.CudaBackend(0)
    b, x = make(O.Q4_K, 64, 512, M=1)
    w = ob.QuantWeight(O.Q4_K, (512, 64), b)
    with pytest.raises(RuntimeError, match="dimension mismatch"):
        be.matmul(np.zeros((1, 64), np.float32), np.zeros((1, 256), np.float32), w)
    with pytest.raises(RuntimeError, match="require F32 activations"):
        be.matmul(np.zeros((1, 64), np.float32), np.zeros((1, 512), np.float16), w)


@pytest.mark.parametrize("dt,N,K,M", [(O.Q4_K, 4096, 14336, 1), (O.Q8_0, 300, 1024, 3), (O.Q6_K, 4096, 4096, 9)])
@pytest.mark.parametrize("offset", [0, 1], ids=["aligned", "offset4"])
def test_matmul_host_pinned_buffers(cuda_lib, dt, N, K, M, offset):
    """odi_cuda_matmul_host on page-locked host buffers (y stored by the
    product straight into host memory, the error word read from mapped
    memory) gives the results of the device-buffer product bit for bit;
    pageable buffers (the copy-engine path) too.  offset4 starts both buffers
    4 bytes into a pinned block."""
    import ctypes

    import torch

    ob = cuda_lib
    L = ob.lib()
    b, x = make(dt, N, K, seed=N + M, M=M)
    h = ctypes.c_void_p()
    bb = np.ascontiguousarray(b)
    ob.check(L.odi_cuda_weight_upload(bb.ctypes.data_as(ctypes.c_void_p), dt, N, K, ctypes.byref(h)))
    try:
        t = upload(ob, dt, b, N, K)
        want, _ = run_matmul(ob, dt, t, x, N, K, ob.ACT_AUTO)
        hx = torch.empty(M * K + 4, dtype=torch.float32).pin_memory()
        hy = torch.full((M * N + 4,), float("nan"), dtype=torch.float32).pin_memory()
        hx[offset:offset + M * K] = torch.from_numpy(x.reshape(-1))
        ob.check(L.odi_cuda_matmul_host(h, hx.data_ptr() + 4 * offset, hy.data_ptr() + 4 * offset, M, ob.ACT_AUTO,
                                        None))
        got = hy[offset:offset + M * N].numpy().reshape(M, N)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        yp = np.full((M, N), np.nan, np.float32)  # pageable
        ob.check(L.odi_cuda_matmul_host(h, x.ctypes.data_as(ctypes.c_void_p), yp.ctypes.data_as(ctypes.c_void_p), M,
                                        ob.ACT_AUTO, None))
        assert np.array_equal(yp.view(np.uint32), want.view(np.uint32))
    finally:
        L.odi_cuda_weight_free(h)


@pytest.mark.parametrize("dt,N,K,M", [(O.Q4_K, 4096, 14336, 1), (O.Q8_0, 300, 1024, 3), (O.Q6_K, 4096, 4096, 9),
                                      (O.Q4_K, 1024, 4096, 32)])
def test_matmul_host_async_queue(cuda_lib, dt, N, K, M):
    """A queue of odi_cuda_matmul_host_async products with distinct inputs,
    closed by one odi_cuda_host_sync, gives each product of the synchronous
    odi_cuda_matmul_host bit for bit: page-locked buffers (x pulled by the
    kernel that runs ahead of each product while the one before it runs, y
    stored by the product), pageable ones, and a page-locked x 4 bytes into
    its block (the 4-byte pull).  M = 1 reports into the mapped error word,
    M = 3 into the device workspace (Q8 records), M = 9 and 32 run on the
    tensor cores (y copied out)."""
    import ctypes

    import torch

    ob = cuda_lib
    L = ob.lib()
    b, _ = make(dt, N, K, seed=N + M, M=M)
    h = ctypes.c_void_p()
    bb = np.ascontiguousarray(b)
    ob.check(L.odi_cuda_weight_upload(bb.ctypes.data_as(ctypes.c_void_p), dt, N, K, ctypes.byref(h)))
    try:
        R = 6
        xs = [O.seeded_acts(M, K, seed=100 + r) for r in range(R)]
        want = []
        for x in xs:
            y = np.full((M, N), np.nan, np.float32)
            ob.check(L.odi_cuda_matmul_host(h, x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p),
                                            M, ob.ACT_AUTO, None))
            want.append(y)
        hx = torch.empty((R, M * K + 4), dtype=torch.float32).pin_memory()
        hy = torch.full((R, M * N), float("nan"), dtype=torch.float32).pin_memory()
        pageable = [np.full((M, N), np.nan, np.float32) for _ in range(R)]
        xo = [1 if r == 4 else 0 for r in range(R)]
        for r in range(R):
            hx[r, xo[r]:xo[r] + M * K] = torch.from_numpy(xs[r].reshape(-1))
        for r in range(R):
            if r % 3 == 2:  # pageable x and y
                rc = L.odi_cuda_matmul_host_async(h, xs[r].ctypes.data_as(ctypes.c_void_p),
                                                  pageable[r].ctypes.data_as(ctypes.c_void_p), M, ob.ACT_AUTO, None)
            else:
                rc = L.odi_cuda_matmul_host_async(h, hx[r].data_ptr() + 4 * xo[r], hy[r].data_ptr(), M,
                                                  ob.ACT_AUTO, None)
            ob.check(rc)
        ob.check(L.odi_cuda_host_sync(None))
        for r in range(R):
            got = pageable[r] if r % 3 == 2 else hy[r].numpy().reshape(M, N)
            assert np.array_equal(got.view(np.uint32), want[r].view(np.uint32)), r
        assert not np.array_equal(want[0], want[1])
    finally:
        L.odi_cuda_weight_free(h)


def _host_weight(ob, dt, N, K, seed):
    import ctypes

    b = np.ascontiguousarray(O.quantize(dt, O.seeded_weights(N, K, seed=seed)))
    h = ctypes.c_void_p()
    ob.check(ob.lib().odi_cuda_weight_upload(b.ctypes.data_as(ctypes.c_void_p), dt, N, K, ctypes.byref(h)))
    return h


@pytest.mark.parametrize("dt,N,K,M,n", [(O.Q8_0, 300, 1024, 1, 450), (O.Q6_K, 32000, 4096, 4, 140)])
def test_matmul_host_async_batches(cuda_lib, dt, N, K, M, n):
    """More queued products than one batch of parked outputs holds: 450
    one-token products cross the 200-entry gather table twice; 140 products
    of 4 x 32000 outputs fill the 64 MiB output ring after 128.  Every h_y
    equals the synchronous call's bit for bit after the one sync."""
    import ctypes

    import torch

    ob = cuda_lib
    L = ob.lib()
    h = _host_weight(ob, dt, N, K, seed=7)
    try:
        R = 5
        hx = torch.stack([torch.from_numpy(O.seeded_acts(M, K, seed=200 + r)) for r in range(R)]).pin_memory()
        want = []
        for r in range(R):
            y = torch.empty((M, N), dtype=torch.float32).pin_memory()
            ob.check(L.odi_cuda_matmul_host(h, hx[r].data_ptr(), y.data_ptr(), M, ob.ACT_AUTO, None))
            want.append(y.numpy().copy())
        hy = torch.full((n, M, N), float("nan"), dtype=torch.float32).pin_memory()
        for i in range(n):
            ob.check(L.odi_cuda_matmul_host_async(h, hx[i % R].data_ptr(), hy[i].data_ptr(), M, ob.ACT_AUTO, None))
        ob.check(L.odi_cuda_host_sync(None))
        got = hy.numpy()
        for i in range(n):
            assert np.array_equal(got[i].view(np.uint32), want[i % R].view(np.uint32)), i
    finally:
        L.odi_cuda_weight_free(h)


def test_matmul_host_async_two_streams(cuda_lib):
    """Products queued on one stream, then on another: the library's shared
    buffers make the second queue wait for the first (its parked outputs sent
    out on their own stream); each stream's sync then finds its results."""
    import torch

    ob = cuda_lib
    L = ob.lib()
    dt, N, K, M = O.Q4_K, 512, 2048, 2
    h = _host_weight(ob, dt, N, K, seed=9)
    try:
        s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
        xs = [torch.from_numpy(O.seeded_acts(M, K, seed=300 + r)).pin_memory() for r in range(6)]
        want = []
        for x in xs:
            y = torch.empty((M, N), dtype=torch.float32).pin_memory()
            ob.check(L.odi_cuda_matmul_host(h, x.data_ptr(), y.data_ptr(), M, ob.ACT_Q8, None))
            want.append(y.numpy().copy())
        ys = [torch.full((M, N), float("nan"), dtype=torch.float32).pin_memory() for _ in range(6)]
        for r in range(6):
            st = s1 if r < 3 else s2
            ob.check(L.odi_cuda_matmul_host_async(h, xs[r].data_ptr(), ys[r].data_ptr(), M, ob.ACT_Q8,
                                                  st.cuda_stream))
        ob.check(L.odi_cuda_host_sync(s2.cuda_stream))
        ob.check(L.odi_cuda_host_sync(s1.cuda_stream))
        for r in range(6):
            assert np.array_equal(ys[r].numpy().view(np.uint32), want[r].view(np.uint32)), r
    finally:
        L.odi_cuda_weight_free(h)
