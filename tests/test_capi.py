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
