"""Failure detection without faulting a GPU.

* A bounded device wait that runs out: odi_cuda_wait_peers_timeout on one
  GPU, with an arrival counter that nothing advances.  The kernel gives up
  after its timeout, sets ODI_CUDA_WS_ERR_PEER_WAIT in the workspace error
  word and returns; the context stays usable (a product afterwards is
  correct).
* Host-side injection (ODI_CUDA_INJECT, read once per process, so each case
  runs in a child process): allocation failures map to
  ODI_CUDA_ERR_GPU_OUT_OF_MEMORY (odi_error_t ODI_ERROR_GPU_OUT_OF_MEMORY,
  include/odi/odi_error.h:41), and a product whose error word reports a wait
  that gave up fails with ODI_CUDA_ERR_OPERATION_FAILED instead of handing
  back its output (the reference's backends throw on failure,
  src/compute/cpu/cpu_backend.cpp:177-227).
"""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
ERR_PEER_WAIT = 32  # ODI_CUDA_WS_ERR_PEER_WAIT


def test_peer_wait_times_out_and_reports(cuda_lib):
    import torch

    ob = cuda_lib
    L = ob.lib()
    cnt = torch.zeros(8, dtype=torch.int64, device="cuda")       # nobody ever arrives
    consumed = torch.zeros(8, dtype=torch.int64, device="cuda")
    ws = ob.new_workspace(256)
    inc = (ctypes.c_uint64 * 1)(1)
    t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t[0].record()
    ob.check(L.odi_cuda_wait_peers_timeout(cnt.data_ptr(), consumed.data_ptr(), inc, 1, 20000, ws.data_ptr(), None))
    t[1].record()
    torch.cuda.synchronize()
    assert t[0].elapsed_time(t[1]) >= 15.0  # it did wait (about 20 ms), then gave up
    assert ob.workspace_status(ws) == ERR_PEER_WAIT
    assert ob.workspace_status(ws) == 0  # read and cleared
    assert int(consumed[0]) == 1
    # the context is still good
    N, K = 128, 512
    b = O.quantize(O.Q4_K, O.seeded_weights(N, K, seed=1))
    x = O.seeded_acts(1, K, seed=2)
    w = ob.repack(O.Q4_K, torch.from_numpy(b.reshape(-1)).cuda(), N, K)
    y = torch.empty((1, N), device="cuda")
    ob.matmul_dev(O.Q4_K, w, torch.from_numpy(x).cuda(), y, N, K, ob.ACT_F32)
    ref = O.matmul_ref(O.Q4_K, x, b, N)
    assert (np.abs(y.cpu().numpy() - ref) <= 2 * O.fp32_bound(O.Q4_K, x, b, N)).all()


def test_peer_wait_timeout_bounds_checked(cuda_lib):
    ob = cuda_lib
    L = ob.lib()
    inc = (ctypes.c_uint64 * 1)(1)
    with pytest.raises(ob.OdiCudaError, match="timeout"):
        ob.check(L.odi_cuda_wait_peers_timeout(8, 8, inc, 1, 0, 8, None))


_CHILD = r"""
import ctypes, sys
import numpy as np
sys.path.insert(0, {root!r})
import odiengine_b200 as ob
import oracle as O
L = ob.lib()
out = {{}}
out["init"] = L.odi_cuda_init(0)
N, K = 96, 512
b = np.ascontiguousarray(O.quantize(O.Q4_K, O.seeded_weights(N, K, seed=3)))
h = ctypes.c_void_p()
out["upload"] = L.odi_cuda_weight_upload(b.ctypes.data_as(ctypes.c_void_p), O.Q4_K, N, K, ctypes.byref(h))
out["upload_msg"] = L.odi_cuda_last_error().decode()
p = ctypes.c_void_p()
hd = ctypes.create_string_buffer(64)
out["sym"] = L.odi_cuda_sym_alloc(4096, ctypes.byref(p), hd)
if out["upload"] == 0:
    x = O.seeded_acts(2, K, seed=4)
    y = np.zeros((2, N), np.float32)
    for fn in ("odi_cuda_matmul_host", "odi_cuda_matmul_host_noalloc"):
        out[fn] = getattr(L, fn)(h, x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), 2, 0, None)
        out[fn + "_msg"] = L.odi_cuda_last_error().decode()
    out["async"] = L.odi_cuda_matmul_host_async(h, x.ctypes.data_as(ctypes.c_void_p),
                                                y.ctypes.data_as(ctypes.c_void_p), 2, 0, None)
    out["host_sync"] = L.odi_cuda_host_sync(None)
    out["host_sync_msg"] = L.odi_cuda_last_error().decode()
    L.odi_cuda_weight_free(h)
print(repr(out))
"""


def _child(inject):
    env = dict(os.environ, ODI_CUDA_INJECT=inject)
    r = subprocess.run([sys.executable, "-c", _CHILD.format(root=ROOT)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    import ast

    return ast.literal_eval(r.stdout.strip().splitlines()[-1])


def test_injected_allocation_failure_maps_to_gpu_out_of_memory(cuda_lib):
    out = _child("alloc")
    assert out["init"] == 0
    assert out["upload"] == 303, out  # ODI_CUDA_ERR_GPU_OUT_OF_MEMORY = ODI_ERROR_GPU_OUT_OF_MEMORY
    assert "cudaMalloc" in out["upload_msg"]
    assert out["sym"] == 303


def test_injected_wait_failure_fails_the_host_product(cuda_lib):
    out = _child("wait")
    assert out["init"] == 0 and out["upload"] == 0 and out["sym"] == 0
    for fn in ("odi_cuda_matmul_host", "odi_cuda_matmul_host_noalloc"):
        assert out[fn] == 6, out  # ODI_CUDA_ERR_OPERATION_FAILED
        assert "wait gave up" in out[fn + "_msg"]
    # a queued product reports at the sync that closes the queue
    assert out["async"] == 0, out
    assert out["host_sync"] == 6 and "wait gave up" in out["host_sync_msg"], out


def test_injected_init_failure_is_backend_unavailable(cuda_lib):
    out = _child("init")
    assert out["init"] == 300  # ODI_CUDA_ERR_BACKEND_UNAVAILABLE
