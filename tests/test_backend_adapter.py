"""odi::CUDABackend, the C++ drop-in for the reference's Backend, driven
through the same odi::Backend calls as the reference's own CPUBackend
(odiengine_b200/host/backend_c.cpp wraps both).

CPU tests: the adapter library loads, exports its facade, and its CPUBackend
(the reference's code) gives the compiled reference's results and errors.
GPU tests: CUDABackend against CPUBackend and the oracle -- the same product
within the bounds of tests/test_gpu_parity.py, the same shape rules and the
same exception messages, weights uploaded once.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle as O

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
ADAPTER = os.path.join(ROOT, "odiengine_b200", "host", "_build", "libodi_cuda_backend.so")
U24 = 2.0 ** -24
BACKEND_CPU, BACKEND_CUDA = 1, 4
F32, F16 = 0, 1
_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_shape = ctypes.POINTER(_i64)
FACADE = {
    "odi_be_last_error": (ctypes.c_char_p, []),
    "odi_be_create": (_vp, [_int, _int, _int, _int]),
    "odi_be_destroy": (None, [_vp]),
    "odi_be_matmul": (_int, [_vp, _vp, _int, _shape, _vp, _int, _int, _shape, _vp, _int, _int, _shape]),
    "odi_be_quantized_matmul": (_int, [_vp, _vp, _int, _shape, _vp, _int, _shape, _vp, _int, _int, _shape]),
    "odi_be_dequantize": (_int, [_vp, _vp, _vp, _int, _int, _shape]),
    "odi_be_sync": (_int, [_vp]),
    "odi_be_supports_dtype": (_int, [_vp, _int]),
    "odi_be_info": (_int, [_vp, ctypes.POINTER(_int), ctypes.c_char_p, _sz, ctypes.c_char_p, _sz,
                           ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "odi_be_cached_weights": (_i64, [_vp]),
    "odi_be_gguf_open": (_vp, [ctypes.c_char_p]),
    "odi_be_gguf_close": (None, [_vp]),
    "odi_be_gguf_tensor_count": (_i64, [_vp]),
    "odi_be_gguf_tensor": (_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(_int), ctypes.POINTER(_int),
                                  _shape]),
    "odi_be_upload_model": (_int, [_vp, _vp, ctypes.POINTER(_i64)]),
    "odi_be_create_via_factory": (_vp, [_int, _int]),
    "odi_be_factory_error": (_int, []),
    "odi_be_factory_message": (ctypes.c_char_p, []),
    "odi_be_cuda_available": (_int, []),
    "odi_be_decoder_from_gguf": (_vp, [_vp, _vp, _int, _int]),
    "odi_be_decoder_free": (None, [_vp]),
    "odi_be_decoder_reset": (_int, [_vp, _int, _int, _int]),
    "odi_be_decoder_prefill": (_int, [_vp, _vp, _int, _int]),
    "odi_be_decoder_generate": (_int, [_vp, _int, _vp]),
    "odi_be_decoder_time": (_int, [_vp, _int, ctypes.POINTER(ctypes.c_float)]),
    "odi_be_decoder_logits": (_int, [_vp, _vp]),
    "odi_be_decoder_config": (_int, [_vp, _vp]),
}
ODI_ERROR_BACKEND_UNAVAILABLE = 300
Q8_K = 15  # odi_dtype_t (include/odi/odi_types.h): a block type the CUDA library does not compute


class BackendError(RuntimeError):
    pass


def _shp(dims):
    return (_i64 * len(dims))(*dims)


class Backend:
    """An odi::Backend* behind the C facade."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            import odiengine_b200 as ob

            ob.lib()  # the adapter resolves libodi_cuda.so through its rpath; load it first
            if not os.path.exists(ADAPTER):
                raise FileNotFoundError(f"{ADAPTER} not built (make -C odiengine_b200/host)")
            L = ctypes.CDLL(ADAPTER)
            for n, (r, a) in FACADE.items():
                f = getattr(L, n)
                f.restype, f.argtypes = r, a
            cls._lib = L
        return cls._lib

    def __init__(self, kind, act_mode=0, threads=1, device=0):
        self.h = self.lib().odi_be_create(kind, threads, device, act_mode)
        if not self.h:
            raise BackendError(self.lib().odi_be_last_error().decode())

    def close(self):
        if self.h:
            self.lib().odi_be_destroy(self.h)
            self.h = None

    def _rc(self, rc):
        if rc:
            raise BackendError(self.lib().odi_be_last_error().decode())

    def matmul(self, out, a, b, b_dtype, b_shape, a_dtype=F32, quantized=False):
        """out/a numpy arrays; b a raw GGUF block array with its [K, N] shape."""
        if quantized:
            rc = self.lib().odi_be_quantized_matmul(self.h, out.ctypes.data, out.ndim, _shp(out.shape), a.ctypes.data,
                                                    a.ndim, _shp(a.shape), b.ctypes.data, b_dtype, len(b_shape),
                                                    _shp(b_shape))
        else:
            rc = self.lib().odi_be_matmul(self.h, out.ctypes.data, out.ndim, _shp(out.shape), a.ctypes.data, a_dtype,
                                          a.ndim, _shp(a.shape), b.ctypes.data, b_dtype, len(b_shape), _shp(b_shape))
        self._rc(rc)
        return out

    def dequantize(self, x, dtype, shape):
        n = int(np.prod(shape))
        out = np.full(n, np.nan, dtype=np.float32)
        self._rc(self.lib().odi_be_dequantize(self.h, out.ctypes.data, x.ctypes.data, dtype, len(shape), _shp(shape)))
        return out

    def info(self):
        t = _int()
        name = ctypes.create_string_buffer(64)
        dev = ctypes.create_string_buffer(256)
        used, avail = _sz(), _sz()
        self._rc(self.lib().odi_be_info(self.h, ctypes.byref(t), name, 64, dev, 256, ctypes.byref(used),
                                        ctypes.byref(avail)))
        return t.value, name.value.decode(), dev.value.decode(), used.value, avail.value

    def cached_weights(self):
        return int(self.lib().odi_be_cached_weights(self.h))

    def sync(self):
        self._rc(self.lib().odi_be_sync(self.h))


def weight(dt, N, K, seed=0):
    Kw = (K + O.BLOCK_ELEMS[dt] - 1) // O.BLOCK_ELEMS[dt] * O.BLOCK_ELEMS[dt]
    return np.ascontiguousarray(O.quantize(dt, O.seeded_weights(N, Kw, seed=seed)))


def need_adapter():
    if not os.path.exists(ADAPTER):
        pytest.skip("adapter not built: the reference tree was absent when building")


# --------------------------------------------------------------------------
# CPU: the facade and the reference CPUBackend behind it
# --------------------------------------------------------------------------
def test_adapter_exports_facade():
    need_adapter()
    L = Backend.lib()
    for n in FACADE:
        assert hasattr(L, n), n


@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0])
def test_cpu_backend_through_facade_is_the_reference(dt):
    need_adapter()
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    N, K, M = 96, 512, 3
    b = weight(dt, N, K)
    x = O.seeded_acts(M, K, seed=4)
    be = Backend(BACKEND_CPU)
    try:
        out = be.matmul(np.zeros((M, N), np.float32), x, b, dt, (K, N))
    finally:
        be.close()
    assert np.array_equal(out, O.matmul_reference_impl(dt, x, b, N))


def test_cpu_backend_errors_through_facade():
    need_adapter()
    be = Backend(BACKEND_CPU)
    try:
        b = weight(O.Q4_0, 32, 256)
        with pytest.raises(BackendError, match="matmul: dimension mismatch"):
            be.matmul(np.zeros((1, 32), np.float32), np.zeros((1, 128), np.float32), b, O.Q4_0, (256, 32))
        with pytest.raises(BackendError, match="Unsupported quantization type"):
            be.matmul(np.zeros((1, 32), np.float32), np.zeros((1, 256), np.float32), weight(O.Q4_K, 32, 256),
                      O.Q4_K, (256, 32))
    finally:
        be.close()


def test_factory_cuda_without_gpu_is_unavailable_not_cpu():
    """The integrated factory's CUDA case (create_cuda_backend): with no
    usable GPU it returns no backend and records ODI_ERROR_BACKEND_UNAVAILABLE
    -- it never hands out a CPUBackend for a CUDA request, as the reference's
    TODO case does (cpu_backend.cpp:1010-1013)."""
    need_adapter()
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = Backend.lib()
    assert not L.odi_be_create_via_factory(BACKEND_CUDA, 1)
    assert L.odi_be_factory_error() == ODI_ERROR_BACKEND_UNAVAILABLE
    assert b"CUDA" in L.odi_be_factory_message()
    assert L.odi_be_cuda_available() == 0
    h = L.odi_be_create_via_factory(BACKEND_CPU, 1)  # the CPU case is the reference's own
    assert h
    L.odi_be_destroy(h)


def test_cuda_backend_unavailable_without_gpu():
    need_adapter()
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(BackendError, match="CUDABackend"):
        Backend(BACKEND_CUDA)


# --------------------------------------------------------------------------
# GPU: CUDABackend vs CPUBackend / the oracle
# --------------------------------------------------------------------------
def _check_f32(dt, x, b, N, y):
    ref = O.matmul_ref(dt, x, b, N)
    bound = O.fp32_bound(dt, x, b, N)
    assert np.isfinite(y).all()
    assert (np.abs(y.astype(np.float64) - ref) <= 2.0 * bound).all()


def _check_q8(dt, x, b, N, y):
    K = x.shape[1]
    yq, bact, mag = O.matmul_q8act(dt, x, b, N, with_mag=True)
    reorder = 2.0 * (K / 8 + 64) * U24 * mag.astype(np.float64)
    assert np.isfinite(y).all()
    assert (np.abs(y.astype(np.float64) - yq) <= reorder).all()


@pytest.fixture(scope="module")
def cuda_backends(cuda_lib):
    need_adapter()
    q8, f32 = Backend(BACKEND_CUDA, act_mode=0), Backend(BACKEND_CUDA, act_mode=1)
    yield q8, f32
    q8.close()
    f32.close()


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K, O.Q4_1, O.Q5_0, O.Q5_1])
@pytest.mark.parametrize("N,K,M", [(96, 512, 1), (300, 1024, 5), (4096, 4096, 1), (512, 2048, 32)])
def test_cuda_backend_matmul(cuda_backends, dt, N, K, M):
    q8, f32 = cuda_backends
    b = weight(dt, N, K, seed=N + K)
    x = O.seeded_acts(M, K, seed=9)
    y8 = q8.matmul(np.full((M, N), np.nan, np.float32), x, b, dt, (K, N))
    yf = f32.matmul(np.full((M, N), np.nan, np.float32), x, b, dt, (K, N), quantized=True)
    _check_q8(dt, x, b, N, y8)
    _check_f32(dt, x, b, N, yf)
    if dt in (O.Q4_0, O.Q8_0) and O.ref_lib() is not None:
        ref = O.matmul_reference_impl(dt, x, b, N)
        assert (np.abs(yf.astype(np.float64) - ref) <= 2.0 * O.fp32_bound(dt, x, b, N)).all()


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K])
def test_cuda_backend_auto_mode(cuda_lib, dt):
    """The default (AUTO) backend: tensor cores from 9 tokens for the dtypes
    that have them, else the Q8 GEMV."""
    need_adapter()
    be = Backend(BACKEND_CUDA, act_mode=3)
    try:
        N, K = 320, 2048
        b = weight(dt, N, K, seed=21)
        for M in (1, 8, 9, 40):
            x = O.seeded_acts(M, K, seed=M)
            y = be.matmul(np.full((M, N), np.nan, np.float32), x, b, dt, (K, N))
            if M >= 9 and dt in (O.Q4_K, O.Q6_K):
                y16, b16 = O.matmul_f16(dt, x, b, N)
                assert (np.abs(y.astype(np.float64) - y16) <= b16 + 1e-30).all()
            else:
                _check_q8(dt, x, b, N, y)
    finally:
        be.close()


@pytest.mark.gpu
def test_cuda_backend_matches_cpu_backend_and_errors(cuda_backends):
    q8, f32 = cuda_backends
    cpu = Backend(BACKEND_CPU)
    try:
        N, K = 64, 512
        b = weight(O.Q4_0, N, K, seed=2)
        x = O.seeded_acts(2, K, seed=3)
        yc = cpu.matmul(np.zeros((2, N), np.float32), x, b, O.Q4_0, (K, N))
        yg = f32.matmul(np.zeros((2, N), np.float32), x, b, O.Q4_0, (K, N))
        assert (np.abs(yg.astype(np.float64) - yc) <= 2.0 * O.fp32_bound(O.Q4_0, x, b, N)).all()
        # the same exceptions, message for message
        for be in (cpu, f32):
            with pytest.raises(BackendError, match="^matmul: dimension mismatch"):
                be.matmul(np.zeros((1, N), np.float32), np.zeros((1, K // 2), np.float32), b, O.Q4_0, (K, N))
            with pytest.raises(BackendError, match="^matmul: quantized weights require F32 activations"):
                be.matmul(np.zeros((1, N), np.float32), np.zeros((1, K), np.float16), b, O.Q4_0, (K, N),
                          a_dtype=F16)
        # leading batch dimensions of `a` are not iterated (M = a.shape(-2)), as in the reference
        xb = O.seeded_acts(3 * 2, K, seed=5).reshape(3, 2, K)
        oc = cpu.matmul(np.zeros((3, 2, N), np.float32), xb, b, O.Q4_0, (K, N))
        og = f32.matmul(np.zeros((3, 2, N), np.float32), xb, b, O.Q4_0, (K, N))
        assert np.array_equal(oc[1:], og[1:])  # untouched by both
        assert (np.abs(og[0].astype(np.float64) - oc[0]) <= 2.0 * O.fp32_bound(O.Q4_0, xb[0], b, N)).all()
    finally:
        cpu.close()


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K])
def test_cuda_backend_dequantize(cuda_backends, dt):
    q8, _ = cuda_backends
    N, K = 70, 512
    b = weight(dt, N, K, seed=7)
    got = q8.dequantize(b, dt, (K, N))
    assert np.array_equal(got.reshape(N, K), O.dequantize(dt, b, N, K))


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [O.Q4_1, O.Q5_0, O.Q5_1])
def test_legacy_types_cuda_correct_where_cpu_backend_reads_transposed(cuda_backends, dt):
    """Q4_1 / Q5_0 / Q5_1: CUDABackend computes the product the block format
    defines; the reference CPUBackend's dequantize + matmul_f32 fallback
    reads the [N][K] dequantized weight as [K][N] (cpu_backend.cpp:211-216)
    and returns that product instead.  Same calls, same tensors."""
    _, f32 = cuda_backends
    N, K, M = 64, 512, 2
    b = weight(dt, N, K, seed=3)
    x = O.seeded_acts(M, K, seed=4)
    y = f32.matmul(np.full((M, N), np.nan, np.float32), x, b, dt, (K, N))
    _check_f32(dt, x, b, N, y)
    cpu = Backend(BACKEND_CPU)
    try:
        yc = cpu.matmul(np.full((M, N), np.nan, np.float32), x, b, dt, (K, N))
    finally:
        cpu.close()
    deq = O.dequantize(dt, b, N, K).astype(np.float64)
    transposed_read = x.astype(np.float64) @ deq.reshape(-1).reshape(K, N)
    assert np.abs(yc - transposed_read).max() <= 1e-4 * np.abs(transposed_read).max()
    assert np.abs(yc - y).max() > 0.1 * np.abs(y).max()


@pytest.mark.gpu
def test_cuda_backend_uploads_once_and_reports():
    need_adapter()
    be = Backend(BACKEND_CUDA)
    try:
        N, K = 256, 1024
        b = weight(O.Q4_K, N, K, seed=1)
        x = O.seeded_acts(1, K, seed=1)
        y1 = be.matmul(np.zeros((1, N), np.float32), x, b, O.Q4_K, (K, N))
        y2 = be.matmul(np.zeros((1, N), np.float32), x, b, O.Q4_K, (K, N))
        assert np.array_equal(y1, y2)
        assert be.cached_weights() == 1
        t, name, dev, used, avail = be.info()
        assert (t, name) == (BACKEND_CUDA, "CUDA")
        assert "sm_10" in dev and used > 0 and avail > 0
        be.sync()
    finally:
        be.close()


@pytest.mark.gpu
def test_factory_cuda_with_gpu_is_the_cuda_backend(cuda_lib):
    need_adapter()
    L = Backend.lib()
    assert L.odi_be_cuda_available() == 1
    h = L.odi_be_create_via_factory(BACKEND_CUDA, 1)
    assert h, L.odi_be_factory_message()
    be = Backend.__new__(Backend)
    be.h = h
    try:
        t, name, _, _, _ = be.info()
        assert (t, name) == (BACKEND_CUDA, "CUDA")
    finally:
        be.close()


@pytest.mark.gpu
def test_cuda_backend_refuses_unsupported_quantized_types(cuda_backends):
    """No CPU fallback in the quantized path: a block type the library does
    not compute is reported unsupported and refused by matmul and
    dequantize, where the reference CPUBackend would claim it
    (cpu_backend.cpp:123-143) and then throw or fall back."""
    q8, _ = cuda_backends
    L = Backend.lib()
    assert L.odi_be_supports_dtype(q8.h, O.Q4_K) == 1
    assert L.odi_be_supports_dtype(q8.h, F32) == 1
    assert L.odi_be_supports_dtype(q8.h, Q8_K) == 0
    K, N = 256, 64
    fake = np.zeros(N * 292, np.uint8)  # Q8_K is 292 bytes per 256 values
    with pytest.raises(BackendError, match="not supported by the CUDA backend"):
        q8.matmul(np.zeros((1, N), np.float32), np.zeros((1, K), np.float32), fake, Q8_K, (K, N))
    with pytest.raises(BackendError, match="not supported by the CUDA backend"):
        q8.dequantize(fake, Q8_K, (K, N))


_INJECT_SCRIPT = r"""
import ctypes, sys
sys.path.insert(0, {root!r})
sys.path.insert(0, {tests!r})
import test_backend_adapter as T
L = T.Backend.lib()
h = L.odi_be_create_via_factory(T.BACKEND_CUDA, 1)
print("handle", bool(h), "code", L.odi_be_factory_error(), L.odi_be_factory_message().decode())
"""


@pytest.mark.gpu
def test_factory_cuda_init_failure_maps_to_unavailable(cuda_lib):
    """A device that fails to initialise (host-side injection,
    ODI_CUDA_INJECT=init, in a child process) gives no backend and
    ODI_ERROR_BACKEND_UNAVAILABLE, on a machine that has a GPU."""
    import subprocess
    import sys

    need_adapter()
    env = dict(os.environ, ODI_CUDA_INJECT="init")
    code = _INJECT_SCRIPT.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "handle False code 300" in r.stdout, r.stdout
