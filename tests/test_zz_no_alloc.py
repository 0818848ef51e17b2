"""odi_cuda_matmul_host_noalloc: the host-buffer product that allocates nothing.

Some callers cannot allocate device memory once they are running: an engine
that reserved HBM for its weights and KV cache up front, a process whose
device memory belongs to another allocator's pool, a decode loop that cannot
take the synchronisation cudaMalloc may cause.  odi_cuda_matmul_host grows a
per-device buffer with cudaMalloc; this entry point stages x, y and the
kernels' error word in a static device array of NOALLOC_SCRATCH_BYTES per GPU
instead, and refuses calls that do not fit.

Checked through the C ABI against odi_cuda_matmul_host on the same uploaded
weight and host activations, two calls in a row (the second call must not see
the first one's leftovers).  Both run the same kernel with the same work
plan, so the tolerance is zero: the outputs must be identical bit for bit,
well inside the oracle bounds the parity tests use.

The file name makes pytest collect it last, so a run that stops at the first
failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    (O.Q4_K, 320, 2048, 1),
    (O.Q8_0, 200, 80, 3),
    (O.Q6_K, 4096, 4096, 8),
    (O.Q4_K, 128, 1024, 9),
    (O.Q4_0, 513, 4096, 32),
]


def _upload(ob, dt, N, K, seed):
    L = ob.lib()
    Kw = (K + O.BLOCK_ELEMS[dt] - 1) // O.BLOCK_ELEMS[dt] * O.BLOCK_ELEMS[dt]
    blocks = np.ascontiguousarray(O.quantize(dt, O.seeded_weights(N, Kw, seed=seed)))
    h = ctypes.c_void_p()
    ob.check(L.odi_cuda_weight_upload(blocks.ctypes.data_as(ctypes.c_void_p), dt, N, K, ctypes.byref(h)))
    return h


def _call(fn, ob, h, x, N, mode):
    y = np.full((x.shape[0], N), np.nan, dtype=np.float32)
    ob.check(fn(h, x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), x.shape[0], mode, None))
    return y


def _free_bytes(L):
    free, total = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.odi_cuda_memory_info(ctypes.byref(free), ctypes.byref(total)) == 0
    return free.value


@pytest.mark.parametrize("dt,N,K,M", CASES)
@pytest.mark.parametrize("mode", [0, 1], ids=["q8", "f32"])
def test_noalloc_matches_matmul_host_twice(cuda_lib, dt, N, K, M, mode):
    ob = cuda_lib
    L = ob.lib()
    h = _upload(ob, dt, N, K, seed=3)
    try:
        x1 = np.ascontiguousarray(O.seeded_acts(M, K, seed=11))
        x2 = np.ascontiguousarray(O.seeded_acts(M, K, seed=12))
        ref1 = _call(L.odi_cuda_matmul_host, ob, h, x1, N, mode)
        ref2 = _call(L.odi_cuda_matmul_host, ob, h, x2, N, mode)
        _call(L.odi_cuda_matmul_host_noalloc, ob, h, x2, N, mode)  # first call on the device: set-up
        # Free device memory is device-wide, so another process (or this one's
        # caching allocator) can move it; the library itself must take none:
        # the reading after the two calls may not fall below the lowest of
        # several readings taken before them.
        free0 = min(_free_bytes(L) for _ in range(3))
        y1 = _call(L.odi_cuda_matmul_host_noalloc, ob, h, x1, N, mode)
        y2 = _call(L.odi_cuda_matmul_host_noalloc, ob, h, x2, N, mode)
        assert max(_free_bytes(L) for _ in range(3)) >= free0, \
            "the no-allocation entry point took device memory"
        np.testing.assert_array_equal(y1, ref1)
        np.testing.assert_array_equal(y2, ref2)
        assert not np.array_equal(y1, y2)
    finally:
        L.odi_cuda_weight_free(h)


def test_noalloc_refuses_oversize_then_still_works(cuda_lib):
    ob = cuda_lib
    L = ob.lib()
    N, K = 4096, 4096
    h = _upload(ob, O.Q4_K, N, K, seed=5)
    try:
        M_big = ob.NOALLOC_SCRATCH_BYTES // (4 * (N + K)) + 1
        x = np.zeros((M_big, K), dtype=np.float32)
        y = np.full((M_big, N), 7.0, dtype=np.float32)
        rc = L.odi_cuda_matmul_host_noalloc(h, x.ctypes.data_as(ctypes.c_void_p),
                                            y.ctypes.data_as(ctypes.c_void_p), M_big, 0, None)
        assert rc == ob.ODI_ERROR_INVALID_ARGUMENT
        assert b"static scratch" in L.odi_cuda_last_error()
        assert np.all(y == 7.0)  # nothing ran
        xs = np.ascontiguousarray(O.seeded_acts(2, K, seed=13))
        ref = _call(L.odi_cuda_matmul_host, ob, h, xs, N, 0)
        np.testing.assert_array_equal(_call(L.odi_cuda_matmul_host_noalloc, ob, h, xs, N, 0), ref)
    finally:
        L.odi_cuda_weight_free(h)
