"""CPU oracle for the quantized matrix product -- TEST INFRASTRUCTURE ONLY.

Thin ctypes bindings over two checker libraries:

* ``liboracle.so`` -- this project's C restatement (odi_oracle.c) of the
  reference path: the fp32 block loops of ``CPUBackend::matmul_q4_0`` /
  ``matmul_q8_0`` (src/compute/cpu/cpu_backend.cpp:786-854), the same loop
  order for Q4_1/Q5_0/Q5_1 (cpu_backend.cpp:704-767 decode) and
  Q4_K/Q5_K/Q6_K, the Q4_0/Q8_0/Q4_1/Q5_0/Q5_1 quantisers of gguf 0.19.0, the Q8_0
  activation quantiser, the Q8-activation integer dot and error bounds, and
  the tiled device layout.
* ``_ref/libodi_ref.so`` -- the reference's own, unmodified CPU backend
  (cpu_backend.cpp + tensor.cpp) behind ref_harness.cpp.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg use
this package; the product path never imports it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

Q8_0, Q4_0, Q4_1, Q5_0, Q5_1, Q4_K, Q5_K, Q6_K = 6, 7, 8, 9, 10, 11, 12, 13
DTYPES = {"Q8_0": Q8_0, "Q4_0": Q4_0, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K}
BLOCK_ELEMS = {Q8_0: 32, Q4_0: 32, Q4_1: 32, Q5_0: 32, Q5_1: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_1: 20, Q5_0: 22, Q5_1: 24, Q4_K: 144, Q5_K: 176, Q6_K: 210}

_lib = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64


def build() -> None:
    """Compile liboracle.so (and _ref when the reference tree is present)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.orc_fp16_to_fp32.restype = ctypes.c_float
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32_ref.restype = ctypes.c_float
        L.orc_fp16_to_fp32_ref.argtypes = [ctypes.c_uint16]
        L.orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.orc_row_bytes.restype = _i64
        L.orc_row_bytes.argtypes = [ctypes.c_int, _i64]
        L.orc_quantize.argtypes = [ctypes.c_int, _vp, _i64, _i64, _vp]
        L.orc_dequantize.argtypes = [ctypes.c_int, _vp, _i64, _i64, _vp, ctypes.c_int]
        L.orc_matmul_ref.argtypes = [ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_int]
        L.orc_quantize_q8_0_act.argtypes = [_vp, _i64, _i64, _vp]
        L.orc_quantize_act_planes.argtypes = [_vp, _i64, _i64, _vp, _vp]
        L.orc_matmul_q8act.argtypes = [ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp]
        L.orc_matmul_q8act_mt.argtypes = [ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, ctypes.c_int]
        L.orc_fp32_bound.argtypes = [ctypes.c_int, _vp, _vp, _i64, _i64, _i64, _vp]
        L.orc_fp32_bound_mt.argtypes = [ctypes.c_int, _vp, _vp, _i64, _i64, _i64, _vp, ctypes.c_int]
        L.orc_term_magnitude.argtypes = [ctypes.c_int, _vp, _i64, _i64, _vp]
        L.orc_block_factors.argtypes = [ctypes.c_int, _vp, _i64, _i64, _vp, _vp, _vp]
        L.orc_tiled_bytes.restype = _i64
        L.orc_tiled_bytes.argtypes = [ctypes.c_int, _i64, _i64]
        L.orc_unit_bytes.restype = _i64
        L.orc_unit_bytes.argtypes = [ctypes.c_int]
        L.orc_repack.argtypes = [ctypes.c_int, _vp, _vp, _i64, _i64]
        L.orc_unpack.argtypes = [ctypes.c_int, _vp, _vp, _i64, _i64]
        _lib = L
    return _lib


def ref_lib():
    """The unmodified reference CPU backend, or None if it was not built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libodi_ref.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.ref_matmul.argtypes = [ctypes.c_int, _vp, _vp, _vp, ctypes.c_longlong,
                                 ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int]
        L.ref_matmul_time.restype = ctypes.c_double
        L.ref_matmul_time.argtypes = L.ref_matmul.argtypes + [ctypes.c_int]
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_dequantize.argtypes = [ctypes.c_int, _vp, _vp, ctypes.c_longlong]
        _ref = L
    return _ref


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_vp)


def row_bytes(dtype: int, K: int) -> int:
    return int(lib().orc_row_bytes(dtype, K))


def quantize(dtype: int, w: np.ndarray) -> np.ndarray:
    """fp32 [N, K] -> GGUF blocks uint8 [N, row_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.zeros((N, row_bytes(dtype, K)), dtype=np.uint8)
    rc = lib().orc_quantize(dtype, _p(w), N, K, _p(out))
    if rc:
        raise ValueError(f"orc_quantize failed ({rc})")
    return out


def dequantize(dtype: int, blocks: np.ndarray, N: int, K: int, ref_fp16: bool = False) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.zeros((N, K), dtype=np.float32)
    rc = lib().orc_dequantize(dtype, _p(blocks), N, K, _p(out), int(ref_fp16))
    if rc:
        raise ValueError(f"orc_dequantize failed ({rc})")
    return out


def matmul_ref(dtype: int, x: np.ndarray, blocks: np.ndarray, N: int, nthreads: int = 0) -> np.ndarray:
    """Restated reference product: out[M,N] = x[M,K] . dequant(W)^T (rows
    split over nthreads host threads, 0: all; results do not depend on it)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.zeros((M, N), dtype=np.float32)
    rc = lib().orc_matmul_ref(dtype, _p(out), _p(x), _p(np.ascontiguousarray(blocks)), M, K, N,
                              nthreads or host_threads())
    if rc:
        raise ValueError(f"orc_matmul_ref failed ({rc})")
    return out


def matmul_reference_impl(dtype: int, x: np.ndarray, blocks: np.ndarray, N: int, nthreads: int = 1) -> np.ndarray:
    """The reference's own CPUBackend::matmul (oracle/_ref).  Raises
    RuntimeError with the reference's message when it throws."""
    L = ref_lib()
    if L is None:
        raise FileNotFoundError("oracle/_ref/libodi_ref.so not built")
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.zeros((M, N), dtype=np.float32)
    rc = L.ref_matmul(dtype, _p(out), _p(x), _p(np.ascontiguousarray(blocks)), M, K, N, nthreads)
    if rc:
        raise RuntimeError(L.ref_last_error().decode())
    return out


def dequantize_reference_impl(dtype: int, blocks: np.ndarray, n: int) -> np.ndarray:
    """The reference's own CPUBackend::dequantize (oracle/_ref) of n values."""
    L = ref_lib()
    if L is None:
        raise FileNotFoundError("oracle/_ref/libodi_ref.so not built")
    out = np.zeros(n, dtype=np.float32)
    if L.ref_dequantize(dtype, _p(out), _p(np.ascontiguousarray(blocks)), n):
        raise RuntimeError(L.ref_last_error().decode())
    return out


def quantize_q8_0_act(x: np.ndarray) -> np.ndarray:
    """fp32 [M, K] -> Q8_0 blocks uint8 [M, ceil(K/32)*34]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.zeros((M, (K + 31) // 32 * 34), dtype=np.uint8)
    lib().orc_quantize_q8_0_act(_p(x), M, K, _p(out))
    return out


def quantize_act_planes(x: np.ndarray):
    """fp32 [M, K] -> (xq int8 [M, Kp], xs records uint8 [M, Kp/32, 8])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    Kp = (K + 255) // 256 * 256
    xq = np.zeros((M, Kp), dtype=np.int8)
    xs = np.zeros((M, Kp // 32, 8), dtype=np.uint8)
    lib().orc_quantize_act_planes(_p(x), M, K, _p(xq), _p(xs))
    return xq, xs


def host_threads() -> int:
    """Host threads the checkers use by default (all cores this process may run on)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def matmul_q8act(dtype: int, x: np.ndarray, blocks: np.ndarray, N: int, with_mag: bool = False,
                 nthreads: int = 0):
    """Q8-activation product and its bound against the exact real product.
    With with_mag, also the sum of |block terms| (for fp32 reordering bounds).
    Rows are split over nthreads host threads (0: all); results do not
    depend on the thread count."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.zeros((M, N), dtype=np.float32)
    bound = np.zeros((M, N), dtype=np.float32)
    mag = np.zeros((M, N), dtype=np.float32)
    rc = lib().orc_matmul_q8act_mt(dtype, _p(out), _p(x), _p(np.ascontiguousarray(blocks)), M, K, N, _p(bound),
                                   _p(mag), nthreads or host_threads())
    if rc:
        raise ValueError(f"orc_matmul_q8act failed ({rc})")
    return (out, bound, mag) if with_mag else (out, bound)


def fp32_bound(dtype: int, x: np.ndarray, blocks: np.ndarray, N: int, nthreads: int = 0) -> np.ndarray:
    """Per-output bound on |y_fp32 - y_exact| for any fp32 summation order
    (rows split over nthreads host threads, 0: all)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    bound = np.zeros((M, N), dtype=np.float32)
    rc = lib().orc_fp32_bound_mt(dtype, _p(x), _p(np.ascontiguousarray(blocks)), M, K, N, _p(bound),
                                 nthreads or host_threads())
    if rc:
        raise ValueError(f"orc_fp32_bound failed ({rc})")
    return bound


def term_magnitude(dtype: int, blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    """|A_g*q| + |B_g| per weight element ([N, K]; >= |w|): the scale of the
    error of decoding a weight to fp16 from fp16-rounded factors."""
    out = np.zeros((N, K), dtype=np.float32)
    rc = lib().orc_term_magnitude(dtype, _p(np.ascontiguousarray(blocks)), N, K, _p(out))
    if rc:
        raise ValueError(f"orc_term_magnitude failed ({rc})")
    return out


def decode_f16(dtype: int, blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    """The fp16 weights the tensor-core path decodes ([N, K] float16):
    rne16(q * rne16(A) - rne16(B)) with value = A*q - B, one rounding of the
    exact result (an IEEE fp16 fma), A and B rounded from fp32."""
    A = np.zeros((N, K), dtype=np.float32)
    B = np.zeros((N, K), dtype=np.float32)
    q = np.zeros((N, K), dtype=np.int32)
    rc = lib().orc_block_factors(dtype, _p(np.ascontiguousarray(blocks)), N, K, _p(A), _p(B), _p(q))
    if rc:
        raise ValueError(f"orc_block_factors failed ({rc})")
    a16 = A.astype(np.float16).astype(np.float64)
    b16 = B.astype(np.float16).astype(np.float64)
    return (q.astype(np.float64) * a16 - b16).astype(np.float16)


def matmul_f16(dtype: int, x: np.ndarray, blocks: np.ndarray, N: int):
    """Restatement of the tensor-core product: fp16 activations times
    decode_f16 weights summed exactly (float64), and the fp32-summation
    bound 2 (K + 16) 2^-24 sum |x16 w16| that any summation order meets."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    x16 = x.astype(np.float16).astype(np.float64)
    w16 = decode_f16(dtype, blocks, N, K).astype(np.float64)
    y = x16 @ w16.T
    bound = 2.0 * (K + 16) * 2.0 ** -24 * (np.abs(x16) @ np.abs(w16).T)
    return y, bound


def f16_bound(dtype: int, x: np.ndarray, blocks: np.ndarray, N: int) -> np.ndarray:
    """Bound on |y - y_exact| for the tensor-core path (fp16 weights decoded
    as fp16(A)*q - fp16(B) in one fp16 fma, fp16-rounded activations, exact
    products, fp32 sums in any order), per output [M, N]:

        1.01 * (2^-10 * S_T + 2^-11 * S_W) + 2 (K + 16) 2^-24 * 1.01 * S_T
        + 2^-20 * sum|x| + 2^-24 * sum|w|

    S_T = sum_k |x_k| T_k (T = term_magnitude), S_W = sum_k |x_k| |w_k|.
    The first term: |fp16 w - w| <= 2^-11 (T + |w|) + 2^-21 and
    |fp16 x - x| <= 2^-11 |x| + 2^-25 (round to nearest, subnormals
    included); the second: fp32 reassociation of K terms of size
    <= 1.01 |x| T; the last two: the absolute (subnormal) parts."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    ax = np.abs(x).astype(np.float64)
    T = term_magnitude(dtype, blocks, N, K).astype(np.float64)
    W = np.abs(dequantize(dtype, blocks, N, K)).astype(np.float64)
    S_T = ax @ T.T
    S_W = ax @ W.T
    u = 2.0 ** -24
    return (1.01 * (2.0 ** -10 * S_T + 2.0 ** -11 * S_W) + 2.0 * (K + 16) * u * 1.01 * S_T
            + 2.0 ** -20 * ax.sum(1)[:, None] + u * W.sum(1)[None, :])


def tiled_bytes(dtype: int, N: int, K: int) -> int:
    return int(lib().orc_tiled_bytes(dtype, N, K))


def repack(dtype: int, blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    out = np.zeros(tiled_bytes(dtype, N, K), dtype=np.uint8)
    rc = lib().orc_repack(dtype, _p(np.ascontiguousarray(blocks)), _p(out), N, K)
    if rc:
        raise ValueError(f"orc_repack failed ({rc})")
    return out


def unpack(dtype: int, tiled: np.ndarray, N: int, K: int) -> np.ndarray:
    out = np.zeros((N, row_bytes(dtype, K)), dtype=np.uint8)
    rc = lib().orc_unpack(dtype, _p(np.ascontiguousarray(tiled)), _p(out), N, K)
    if rc:
        raise ValueError(f"orc_unpack failed ({rc})")
    return out


def seeded_weights(N: int, K: int, seed: int = 0, std: float = 0.02) -> np.ndarray:
    """W ~ N(0, std) fp32 [N, K] from numpy default_rng(seed)."""
    return np.random.default_rng(seed).normal(0.0, std, (N, K)).astype(np.float32)


def seeded_acts(M: int, K: int, seed: int = 1) -> np.ndarray:
    """x ~ N(0, 1) fp32 [M, K] from numpy default_rng(seed)."""
    return np.random.default_rng(seed).normal(0.0, 1.0, (M, K)).astype(np.float32)
