"""odiengine_b200 -- B200 (sm_100a) backend for ODIEngine's quantized matrix product.

The product is the C-ABI library ``libodi_cuda.so`` (declared in
include/odi_cuda.h).  This package is the host-side mirror of the reference's
compute-dispatch interface for that path (src/compute/backend.hpp:16-131):
:class:`CudaBackend` offers ``matmul`` / ``quantized_matmul`` / ``dequantize`` /
``sync`` with the reference's argument meaning and error behaviour, over the
C ABI via ctypes.  PyTorch is used only as the device-memory and stream
holder (plumbing); all arithmetic happens in the library's CUDA kernels.

There is no CPU fallback: importing the package without the built library,
or calling it without a B200, raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libodi_cuda.so")

# odi_dtype_t (include/odi/odi_types.h:32-49)
ODI_DTYPE_F32 = 0
ODI_DTYPE_Q8_0 = 6
ODI_DTYPE_Q4_0 = 7
ODI_DTYPE_Q4_1 = 8
ODI_DTYPE_Q5_0 = 9
ODI_DTYPE_Q5_1 = 10
ODI_DTYPE_Q4_K = 11
ODI_DTYPE_Q5_K = 12
ODI_DTYPE_Q6_K = 13
DTYPE_NAMES = {ODI_DTYPE_Q8_0: "Q8_0", ODI_DTYPE_Q4_0: "Q4_0", ODI_DTYPE_Q4_1: "Q4_1", ODI_DTYPE_Q5_0: "Q5_0",
               ODI_DTYPE_Q5_1: "Q5_1", ODI_DTYPE_Q4_K: "Q4_K", ODI_DTYPE_Q5_K: "Q5_K", ODI_DTYPE_Q6_K: "Q6_K"}
DTYPES = {v: k for k, v in DTYPE_NAMES.items()}
BLOCK_ELEMS = {ODI_DTYPE_Q8_0: 32, ODI_DTYPE_Q4_0: 32, ODI_DTYPE_Q4_1: 32, ODI_DTYPE_Q5_0: 32, ODI_DTYPE_Q5_1: 32,
               ODI_DTYPE_Q4_K: 256, ODI_DTYPE_Q5_K: 256, ODI_DTYPE_Q6_K: 256}
BLOCK_BYTES = {ODI_DTYPE_Q8_0: 34, ODI_DTYPE_Q4_0: 18, ODI_DTYPE_Q4_1: 20, ODI_DTYPE_Q5_0: 22, ODI_DTYPE_Q5_1: 24,
               ODI_DTYPE_Q4_K: 144, ODI_DTYPE_Q5_K: 176, ODI_DTYPE_Q6_K: 210}

ACT_Q8 = 0
ACT_F32 = 1
ACT_F16 = 2
ACT_AUTO = 3
TC_MIN_TOKENS = 9  # ODI_CUDA_TC_MIN_TOKENS
FLAG_PDL = 1

# odi_error_t values (include/odi/odi_error.h:11-48)
ODI_SUCCESS = 0
ODI_ERROR_INVALID_ARGUMENT = 2
ODI_ERROR_BACKEND_UNAVAILABLE = 300
ODI_ERROR_GPU_OUT_OF_MEMORY = 303

# Every symbol include/odi_cuda.h declares, with (restype, argtypes).
_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = {
    "odi_cuda_init": (_int, [_int]),
    "odi_cuda_device_count": (_int, []),
    "odi_cuda_device_info": (_int, [ctypes.c_char_p, _sz]),
    "odi_cuda_memory_info": (_int, [ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "odi_cuda_supports_dtype": (_int, [_int]),
    "odi_cuda_last_error": (ctypes.c_char_p, []),
    "odi_cuda_sync": (_int, [_vp]),
    "odi_cuda_gguf_bytes": (_i64, [_int, _i64, _i64]),
    "odi_cuda_tiled_bytes": (_i64, [_int, _i64, _i64]),
    "odi_cuda_repack": (_int, [_int, _vp, _vp, _i64, _i64, _vp]),
    "odi_cuda_unpack": (_int, [_int, _vp, _vp, _i64, _i64, _vp]),
    "odi_cuda_weight_upload": (_int, [_vp, _int, _i64, _i64, ctypes.POINTER(_vp)]),
    "odi_cuda_weight_free": (_int, [_vp]),
    "odi_cuda_weight_data": (_vp, [_vp]),
    "odi_cuda_weight_shape": (_int, [_vp, ctypes.POINTER(_int), ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "odi_cuda_quantize_weight": (_int, [_int, _vp, _vp, _i64, _i64, _vp]),
    "odi_cuda_quantize_q8_0": (_int, [_vp, _vp, _i64, _i64, _vp]),
    "odi_cuda_matmul_workspace_bytes": (_sz, [_int, _i64, _i64, _i64, _int]),
    "odi_cuda_gemv_plan_info": (_int, [_int, _i64, _i64, _i64, _int, _vp]),
    "odi_cuda_matmul": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _int, _vp]),
    "odi_cuda_matmul_fused": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _int, _vp, _vp]),
    "odi_cuda_workspace_status": (_int, [_vp, ctypes.POINTER(_int), _vp]),
    "odi_cuda_dequantize": (_int, [_int, _vp, _vp, _i64, _i64, _vp]),
    "odi_cuda_matmul_host": (_int, [_vp, _vp, _vp, _i64, _int, _vp]),
    "odi_cuda_matmul_host_async": (_int, [_vp, _vp, _vp, _i64, _int, _vp]),
    "odi_cuda_host_sync": (_int, [_vp]),
    "odi_cuda_matmul_host_noalloc": (_int, [_vp, _vp, _vp, _i64, _int, _vp]),
    "odi_cuda_dequantize_host": (_int, [_vp, _vp, _vp]),
    "odi_cuda_tc_supported": (_int, [_int]),
    "odi_cuda_embed": (_int, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "odi_cuda_rms_norm": (_int, [_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "odi_cuda_rope_kv": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int, ctypes.c_float, _vp]),
    "odi_cuda_attention_scratch_bytes": (_sz, [_int, _int, _int]),
    "odi_cuda_attention_decode": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int, ctypes.c_float, _vp, _sz,
                                         _vp]),
    "odi_cuda_rope_attention": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int,
                                       ctypes.c_float, ctypes.c_float, _vp, _sz, _vp]),
    "odi_cuda_q8_records_bytes": (_sz, [_i64, _i64]),
    "odi_cuda_quantize_records": (_int, [_vp, _i64, _i64, _vp, _vp, _int, _vp]),
    "odi_cuda_matmul_q8rec": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _int, _vp, _vp]),
    "odi_cuda_silu_mul": (_int, [_vp, _vp, _i64, _vp]),
    "odi_cuda_add": (_int, [_vp, _vp, _i64, _vp]),
    "odi_cuda_argmax": (_int, [_vp, _i64, _vp, _vp, _int, _vp]),
    "odi_cuda_scatter_signals": (_i64, [_int, _i64, _i64, _i64, _int]),
    "odi_cuda_matmul_scatter": (_int, [_int, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _int, _vp, _vp]),
    "odi_cuda_wait_peers": (_int, [_vp, _vp, _vp, _int, _vp, _vp]),
    "odi_cuda_wait_peers_timeout": (_int, [_vp, _vp, _vp, _int, ctypes.c_uint64, _vp, _vp]),
    "odi_cuda_decoder_create": (_int, [_vp, _vp, _vp, _vp, _vp, _int, ctypes.POINTER(_vp)]),
    "odi_cuda_decoder_free": (_int, [_vp]),
    "odi_cuda_decoder_reset": (_int, [_vp, _int, _int, _int]),
    "odi_cuda_decoder_prefill": (_int, [_vp, _vp, _int, _int]),
    "odi_cuda_decoder_generate": (_int, [_vp, _int, _vp]),
    "odi_cuda_decoder_time": (_int, [_vp, _int, ctypes.POINTER(ctypes.c_float)]),
    "odi_cuda_decoder_tokens": (_int, [_vp, _int, _int, _vp]),
    "odi_cuda_decoder_logits": (_int, [_vp, _vp]),
    "odi_cuda_decoder_launches_per_step": (_int, [_vp]),
    "odi_cuda_buffer_upload": (_int, [_vp, _sz, ctypes.POINTER(_vp)]),
    "odi_cuda_buffer_free": (_int, [_vp]),
    "odi_cuda_nccl_unique_id": (_int, [_vp]),
    "odi_cuda_nccl_init": (_int, [_vp, _int, _int, ctypes.POINTER(_vp)]),
    "odi_cuda_nccl_free": (_int, [_vp]),
    "odi_cuda_comm_ranks": (_int, [_vp, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
    "odi_cuda_sharded_workspace_bytes": (_sz, [_vp, _int, _i64, _i64, _i64, _int]),
    "odi_cuda_matmul_sharded": (_int, [_vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _sz, _int, _vp]),
    "odi_cuda_sym_alloc": (_int, [_sz, ctypes.POINTER(_vp), _vp]),
    "odi_cuda_sym_free": (_int, [_vp]),
    "odi_cuda_ipc_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "odi_cuda_ipc_close": (_int, [_vp]),
}

# ODI_CUDA_NOALLOC_SCRATCH_BYTES (include/odi_cuda.h): the static device
# array behind odi_cuda_matmul_host_noalloc.
NOALLOC_SCRATCH_BYTES = 8 << 20

MAX_PEERS = 8  # ODI_CUDA_MAX_PEERS
NCCL_ID_BYTES = 128  # ODI_CUDA_NCCL_ID_BYTES
IPC_HANDLE_BYTES = 64  # ODI_CUDA_IPC_HANDLE_BYTES


class MatmulOpts(ctypes.Structure):
    """odi_cuda_matmul_opts (include/odi_cuda.h)."""

    _fields_ = [("norm_weight", ctypes.c_void_p), ("norm_eps", ctypes.c_float), ("swiglu", ctypes.c_int),
                ("accumulate", ctypes.c_int), ("norm_ssq", ctypes.c_void_p), ("norm_ssq_count", ctypes.c_int),
                ("out_ssq", ctypes.c_void_p)]


class Q8RecOpts(ctypes.Structure):
    """odi_cuda_q8rec_opts (include/odi_cuda.h)."""

    _fields_ = [("accumulate", ctypes.c_int), ("out_ssq", ctypes.c_void_p), ("norm_ssq", ctypes.c_void_p),
                ("norm_ssq_count", ctypes.c_int), ("norm_eps", ctypes.c_float), ("out_records", ctypes.c_void_p),
                ("out_norm_weight", ctypes.c_void_p), ("out_swiglu", ctypes.c_int)]


class GemvPlan(ctypes.Structure):
    """odi_cuda_gemv_plan (include/odi_cuda.h)."""

    _fields_ = [("tokens_per_pass", ctypes.c_int), ("passes", ctypes.c_int), ("cluster", ctypes.c_int),
                ("spans_per_cta", ctypes.c_int), ("stages", ctypes.c_int), ("reduce_scatter", ctypes.c_int),
                ("ctas_per_sm", ctypes.c_int), ("ctas", ctypes.c_int64), ("shared_bytes", ctypes.c_size_t)]


def gemv_plan(dtype: int, M: int, N: int, K: int, act_mode: int = 0) -> "GemvPlan":
    """The streaming GEMV's work split for one product (host arithmetic)."""
    p = GemvPlan()
    check(lib().odi_cuda_gemv_plan_info(dtype, M, N, K, act_mode, ctypes.byref(p)))
    return p


class Scatter(ctypes.Structure):
    """odi_cuda_scatter (include/odi_cuda.h)."""

    _fields_ = [("out", ctypes.c_void_p * MAX_PEERS), ("counters", ctypes.c_void_p * MAX_PEERS),
                ("nranks", ctypes.c_int), ("rank", ctypes.c_int), ("row0", ctypes.c_int64), ("ld", ctypes.c_int64)]


_lib = None


class OdiCudaError(RuntimeError):
    """A non-zero odi_error_t status from the library, with its message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load libodi_cuda.so (build it first with ``python -m odiengine_b200.build``)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m odiengine_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise OdiCudaError(rc, lib().odi_cuda_last_error().decode(errors="replace"))


def _ptr(t) -> int:
    return t.data_ptr() if t is not None else 0


def _stream(stream) -> int:
    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def gguf_bytes(dtype: int, N: int, K: int) -> int:
    return int(lib().odi_cuda_gguf_bytes(dtype, N, K))


def tiled_bytes(dtype: int, N: int, K: int) -> int:
    return int(lib().odi_cuda_tiled_bytes(dtype, N, K))


def init(device: int = 0) -> None:
    check(lib().odi_cuda_init(device))


def repack(dtype: int, gguf_dev, N: int, K: int, stream=None):
    """Device GGUF blocks (uint8 tensor) -> new device uint8 tensor in the tiled layout."""
    import torch

    out = torch.empty(tiled_bytes(dtype, N, K), dtype=torch.uint8, device=gguf_dev.device)
    check(lib().odi_cuda_repack(dtype, _ptr(gguf_dev), _ptr(out), N, K, _stream(stream)))
    return out


def unpack(dtype: int, tiled_dev, N: int, K: int, stream=None):
    import torch

    out = torch.empty(gguf_bytes(dtype, N, K), dtype=torch.uint8, device=tiled_dev.device)
    check(lib().odi_cuda_unpack(dtype, _ptr(tiled_dev), _ptr(out), N, K, _stream(stream)))
    return out


def quantize_q8_0(x_dev, stream=None):
    """fp32 [M, K] device tensor -> GGUF Q8_0 blocks uint8 [M, ceil(K/32)*34]."""
    import torch

    M, K = x_dev.shape
    out = torch.empty((M, (K + 31) // 32 * 34), dtype=torch.uint8, device=x_dev.device)
    check(lib().odi_cuda_quantize_q8_0(_ptr(x_dev), _ptr(out), M, K, _stream(stream)))
    return out


def quantize_weight(dtype: int, w_dev, stream=None):
    """fp32 [N, K] device tensor -> GGUF blocks uint8 [N * row bytes] on the device."""
    import torch

    N, K = w_dev.shape
    out = torch.empty(gguf_bytes(dtype, N, K), dtype=torch.uint8, device=w_dev.device)
    check(lib().odi_cuda_quantize_weight(dtype, _ptr(w_dev), _ptr(out), N, K, _stream(stream)))
    return out


def workspace_bytes(dtype: int, M: int, N: int, K: int, act_mode: int = ACT_Q8) -> int:
    return int(lib().odi_cuda_matmul_workspace_bytes(dtype, M, N, K, act_mode))


def new_workspace(nbytes: int, device="cuda"):
    """A zero-filled device workspace (the library keeps it valid between calls)."""
    import torch

    return torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)


def matmul_dev(dtype: int, w_tiled, x, y, N: int, K: int, act_mode: int = ACT_Q8, workspace=None,
               flags: int = 0, stream=None):
    """y[M,N] = x[M,K] . dequant(W)^T on device tensors (asynchronous)."""
    M = x.shape[0]
    need = workspace_bytes(dtype, M, N, K, act_mode)
    if workspace is None:
        workspace = new_workspace(need, x.device)
    check(lib().odi_cuda_matmul(dtype, _ptr(w_tiled), _ptr(x), _ptr(y), M, N, K, act_mode,
                                _ptr(workspace), workspace.numel(), flags, _stream(stream)))
    return y


def workspace_status(workspace, stream=None) -> int:
    st = ctypes.c_int(0)
    check(lib().odi_cuda_workspace_status(_ptr(workspace), ctypes.byref(st), _stream(stream)))
    return st.value


def dequantize_dev(dtype: int, w_tiled, N: int, K: int, stream=None):
    import torch

    out = torch.empty((N, K), dtype=torch.float32, device=w_tiled.device)
    check(lib().odi_cuda_dequantize(dtype, _ptr(w_tiled), _ptr(out), N, K, _stream(stream)))
    return out


# ---------------------------------------------------------------------------
# Mirror of the reference's Backend interface for the quantized-matmul path.
# ---------------------------------------------------------------------------

@dataclass
class QuantWeight:
    """A GGUF weight as the reference sees it: shape [K, N] (ne0 = K inputs,
    ne1 = N outputs), dtype an odi_dtype_t, host bytes of N rows of blocks
    (gguf_parser.cpp:614-628 hands out exactly such views)."""

    dtype: int
    shape: tuple  # (K, N)
    data: object  # numpy uint8 array of GGUF blocks

    @property
    def K(self) -> int:
        return self.shape[0]

    @property
    def N(self) -> int:
        return self.shape[1]


class DeviceWeight:
    """A weight uploaded once to HBM (odi_cuda_weight_upload): owns the tiled copy."""

    def __init__(self, w: QuantWeight):
        import numpy as np

        buf = np.ascontiguousarray(w.data, dtype=np.uint8)
        if buf.nbytes != gguf_bytes(w.dtype, w.N, w.K):
            raise ValueError(f"weight bytes {buf.nbytes} != expected {gguf_bytes(w.dtype, w.N, w.K)}")
        h = ctypes.c_void_p()
        check(lib().odi_cuda_weight_upload(buf.ctypes.data_as(ctypes.c_void_p), w.dtype, w.N, w.K, ctypes.byref(h)))
        self.handle = h
        self.tiled = None
        self.dtype, self.N, self.K = w.dtype, w.N, w.K

    @classmethod
    def from_tiled(cls, dtype: int, N: int, K: int, tiled) -> "DeviceWeight":
        """Wrap a device uint8 tensor already in the tiled layout (e.g. made by
        quantize_weight + repack on the device); the tensor is kept alive."""
        if tiled.numel() != tiled_bytes(dtype, N, K):
            raise ValueError("tiled tensor size does not match the shape")
        self = cls.__new__(cls)
        self.handle, self.tiled = None, tiled
        self.dtype, self.N, self.K = dtype, N, K
        return self

    @property
    def data_ptr(self) -> int:
        if self.tiled is not None:
            return self.tiled.data_ptr()
        return lib().odi_cuda_weight_data(self.handle)

    def _ws_for(self, M: int, act_mode: int, device):
        """The weight's cached workspace, grown to what M tokens need."""
        need = workspace_bytes(self.dtype, M, self.N, self.K, act_mode)
        ws = getattr(self, "_ws", None)
        if ws is None or ws.numel() < need or ws.device != device:
            ws = self._ws = new_workspace(need, device)
        return ws

    def matmul(self, x, y=None, act_mode: int = None, flags: int = 0, stream=None):
        """y[M, N] = x[M, K] . W^T for device fp32 tensors (asynchronous on
        `stream`); the workspace is cached on the weight and grown on demand."""
        import torch

        if act_mode is None:
            act_mode = ACT_AUTO
        M = x.shape[0]
        if y is None:
            y = torch.empty((M, self.N), dtype=torch.float32, device=x.device)
        ws = self._ws_for(M, act_mode, x.device)
        check(lib().odi_cuda_matmul(self.dtype, self.data_ptr, _ptr(x), _ptr(y), M, self.N, self.K, act_mode,
                                    _ptr(ws), ws.numel(), flags, _stream(stream)))
        return y

    def free(self) -> None:
        self.tiled = None
        if getattr(self, "handle", None):
            check(lib().odi_cuda_weight_free(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class CudaBackend:
    """Host mirror of ``odi::Backend`` (src/compute/backend.hpp:16-131) for the
    quantized matrix product, backed by libodi_cuda.so.

    * ``matmul(out, a, b)`` -- backend.hpp:38 / cpu_backend.cpp:177-227: a is
      fp32 [M, K] (or [K]), b a :class:`QuantWeight` of shape [K, N], out fp32
      [M, N].  Same checks and messages as the reference: "matmul: dimension
      mismatch", "matmul: quantized weights require F32 activations".
    * ``quantized_matmul`` forwards to ``matmul`` (cpu_backend.cpp:650-653).
    * ``dequantize(out, x)`` -- backend.hpp:111.
    * ``sync()`` -- backend.hpp:130.
    Weights are uploaded to HBM once, on first use, and cached by identity.
    """

    def __init__(self, device: int = 0, act_mode: int = ACT_Q8):
        init(device)
        self.device = device
        self.act_mode = act_mode
        self._cache = {}

    # Backend info (backend.hpp:21-30)
    def type(self) -> int:
        return 4  # ODI_BACKEND_CUDA (odi_types.h:57)

    def name(self) -> str:
        return "CUDA"

    def device_info(self) -> str:
        buf = ctypes.create_string_buffer(256)
        check(lib().odi_cuda_device_info(buf, 256))
        return buf.value.decode()

    def available_memory(self) -> int:
        f, t = ctypes.c_size_t(), ctypes.c_size_t()
        check(lib().odi_cuda_memory_info(ctypes.byref(f), ctypes.byref(t)))
        return f.value

    def used_memory(self) -> int:
        f, t = ctypes.c_size_t(), ctypes.c_size_t()
        check(lib().odi_cuda_memory_info(ctypes.byref(f), ctypes.byref(t)))
        return t.value - f.value

    def supports_dtype(self, dtype: int) -> bool:
        return bool(lib().odi_cuda_supports_dtype(dtype))

    def device_weight(self, b: QuantWeight) -> DeviceWeight:
        """The HBM copy of a weight, uploaded on first use.  Keyed like the
        reference's stable mmap views (gguf_parser.cpp:614-628): by host data
        address, dtype and shape; the cache holds the host array so the
        address cannot be recycled while the entry lives."""
        import numpy as np

        arr = np.asarray(b.data)
        key = (arr.__array_interface__["data"][0], arr.nbytes, b.dtype, b.shape)
        hit = self._cache.get(key)
        if hit is None:
            hit = (DeviceWeight(b), arr)
            self._cache[key] = hit
        return hit[0]

    def matmul(self, out, a, b) -> None:
        import numpy as np

        if not isinstance(b, QuantWeight):
            raise RuntimeError("matmul: unsupported dtype combination")
        a = np.asarray(a)
        if a.ndim < 1:
            raise RuntimeError("matmul: invalid tensor dimensions")
        M = 1 if a.ndim == 1 else int(np.prod(a.shape[:-1]))
        K = a.shape[-1]
        if K != b.K:
            raise RuntimeError("matmul: dimension mismatch")
        if a.dtype != np.float32:
            raise RuntimeError("matmul: quantized weights require F32 activations")
        if not self.supports_dtype(b.dtype):
            raise RuntimeError("Unsupported quantization type for dequantize")
        if out.dtype != np.float32 or out.size != M * b.N or not out.flags["C_CONTIGUOUS"]:
            raise RuntimeError("matmul: output must be contiguous F32 [M, N]")
        dw = self.device_weight(b)
        x = np.ascontiguousarray(a.reshape(M, K))
        check(lib().odi_cuda_matmul_host(dw.handle, x.ctypes.data_as(ctypes.c_void_p),
                                         out.ctypes.data_as(ctypes.c_void_p), M, self.act_mode, None))

    def quantized_matmul(self, out, a, b_quant) -> None:
        self.matmul(out, a, b_quant)

    def dequantize(self, out, x: QuantWeight) -> None:
        import numpy as np
        import torch

        dw = self.device_weight(x)
        ptr = dw.data_ptr
        dev = torch.empty((x.N, x.K), dtype=torch.float32, device=f"cuda:{self.device}")
        check(lib().odi_cuda_dequantize(x.dtype, ptr, dev.data_ptr(), x.N, x.K, None))
        check(lib().odi_cuda_sync(None))
        np.copyto(out.reshape(x.N, x.K), dev.cpu().numpy())

    def sync(self) -> None:
        check(lib().odi_cuda_sync(None))
