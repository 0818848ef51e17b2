"""The C-ABI library loads and exports every symbol include/odi_cuda.h
declares; host-only layout helpers agree with the oracle.  No GPU needed and
no kernel is launched."""
import os
import re

import pytest

import odiengine_b200 as ob
import oracle as O

HEADER = os.path.join(os.path.dirname(__file__), "..", "include", "odi_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(odi_cuda_\w+)\s*\(", src)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    for s in ("odi_cuda_init", "odi_cuda_matmul", "odi_cuda_quantize_q8_0", "odi_cuda_repack",
              "odi_cuda_weight_upload", "odi_cuda_matmul_host", "odi_cuda_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = ob.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing


def test_python_signatures_cover_header():
    assert set(declared_symbols()) <= set(ob.SIGNATURES)


@pytest.mark.parametrize("dt", [O.Q4_0, O.Q8_0, O.Q4_K, O.Q5_K, O.Q6_K, O.Q4_1, O.Q5_0, O.Q5_1])
@pytest.mark.parametrize("N,K", [(1, 256), (65, 512), (4096, 14336), (32000, 4096)])
def test_layout_sizes_match_oracle(dt, N, K):
    assert ob.tiled_bytes(dt, N, K) == O.tiled_bytes(dt, N, K)
    assert ob.gguf_bytes(dt, N, K) == O.row_bytes(dt, K) * N


def test_supports_dtype():
    L = ob.lib()
    for dt in (6, 7, 8, 9, 10, 11, 12, 13):
        assert L.odi_cuda_supports_dtype(dt) == 1
    for dt in (0, 1, 2, 5, 14):
        assert L.odi_cuda_supports_dtype(dt) == 0


def test_bad_arguments_report_odi_error_codes():
    L = ob.lib()
    assert L.odi_cuda_gguf_bytes(99, 1, 1) == -1
    rc = L.odi_cuda_matmul(11, None, None, None, 1, 64, 300, 0, None, 0, 0, None)
    assert rc == ob.ODI_ERROR_INVALID_ARGUMENT  # K-quant K % 256 != 0
    assert b"256" in L.odi_cuda_last_error()
    rc = L.odi_cuda_matmul(14, None, None, None, 1, 64, 256, 0, None, 0, 0, None)
    assert rc == 202  # ODI_ERROR_MODEL_UNSUPPORTED_DTYPE for Q8_K


# The shapes the bench times on the streaming GEMV: the 7B decode sweep (M = 1
# and 8), the headline, its 8-token pass, and the 70B one-token shapes.
SWEEP = [(dt, N, K, M) for dt in (O.Q8_0, O.Q4_K, O.Q6_K)
         for N, K in ((4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)) for M in (1, 8)]
SWEEP += [(O.Q4_K, 4096, 14336, 1), (O.Q4_K, 4096, 14336, 8), (O.Q4_K, 28672, 8192, 1),
          (O.Q4_K, 8192, 28672, 1), (O.Q4_K, 128256, 8192, 1)]


@pytest.mark.parametrize("dt,N,K,M", SWEEP)
def test_gemv_plan_fits_four_ctas_per_sm(dt, N, K, M):
    """Every timed GEMV configuration keeps four CTAs per SM: a plan whose
    shared memory exceeded the quarter of an SM ran its grid in 1.15 waves
    (the 8-token passes before the reduce-scatter).  Host arithmetic only."""
    p = ob.gemv_plan(dt, M, N, K, ob.ACT_Q8)
    assert p.ctas_per_sm == 4, (p.shared_bytes, p.cluster, p.spans_per_cta)
    assert p.shared_bytes <= 56 * 1024
    assert p.stages >= 2 and p.stages % 2 == 0
    assert p.tokens_per_pass == (1 if M == 1 else 8) and p.passes == 1
    # the split covers the row tiles and the spans exactly
    assert p.ctas == -(-N // 64) * p.cluster
    assert (p.cluster - 1) * p.spans_per_cta < -(-K // 256) <= p.cluster * p.spans_per_cta
    assert p.reduce_scatter == (1 if M > 1 and p.cluster > 1 else 0)


def test_gemv_plan_refuses_other_modes():
    with pytest.raises(ob.OdiCudaError):
        ob.gemv_plan(O.Q4_K, 32, 4096, 4096, ob.ACT_F16)
    with pytest.raises(ob.OdiCudaError):
        ob.gemv_plan(O.Q4_K, 1, 4096, 100, ob.ACT_Q8)  # K-quant rows are whole super-blocks
    p = ob.gemv_plan(O.Q4_K, 13, 4096, 4096, ob.ACT_Q8)
    assert p.tokens_per_pass == 8 and p.passes == 2
