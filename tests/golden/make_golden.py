"""Generate the golden fixtures in tests/golden/golden.npz.

Run in a container that has both the `gguf` Python package (0.19.0) and the
reference tree (for oracle/_ref):

    make -C oracle && python tests/golden/make_golden.py

What each array pins:
  w / x                  seeded inputs: W ~ N(0, 0.02) from default_rng(0),
                         x ~ N(0, 1) from default_rng(1)
  q4_0_bytes, q8_0_bytes gguf 0.19.0 quants.quantize(W, Q4_0 / Q8_0)
  act_q8_0_bytes         gguf 0.19.0 quants.quantize(x, Q8_0)
  <t>_dequant            gguf 0.19.0 quants.dequantize of the <t> bytes
  q4k/q5k/q6k_bytes      this project's K-quant quantiser output (gguf has no
                         K-quant quantiser); pinned through <t>_dequant
  <t>_rand_bytes/_dequant random K-quant blocks (normal fp16 scales) decoded by gguf
  ref_q4_0_y, ref_q8_0_y the UNMODIFIED reference CPUBackend::matmul
                         (oracle/_ref) on x and the gguf-quantised W
  ragged_*               K = 80 (not a multiple of 32): reference matmul over
                         3 blocks per row, only the first 80 values used
  q4_1/q5_0/q5_1_bytes   gguf 0.19.0 quants.quantize(W, Q4_1 / Q5_0 / Q5_1)
  <t>_dequant            gguf 0.19.0 quants.dequantize of those bytes
  ref_<t>_dequant        the UNMODIFIED reference CPUBackend::dequantize
                         (cpu_backend.cpp:704-767) of the same bytes
  ref_<t>_y              the UNMODIFIED reference CPUBackend::matmul on them:
                         its dequantize + matmul_f32 fallback reads the
                         [N][K] dequantized buffer as [K][N]
                         (cpu_backend.cpp:211-216), kept as evidence of that
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

import oracle as O  # noqa: E402
from gguf import quants  # noqa: E402
from gguf.constants import GGMLQuantizationType as T  # noqa: E402

N, K, M = 32, 512, 3


def rand_kquant_blocks(rng, dtype, nblocks):
    bb = O.BLOCK_BYTES[dtype]
    b = rng.integers(0, 256, (nblocks, bb), dtype=np.uint8)
    # fp16 scale fields: normal, moderate magnitude (exponent 5..20)
    def normal_f16(n):
        e = rng.integers(5, 21, n).astype(np.uint16)
        m = rng.integers(0, 1024, n).astype(np.uint16)
        s = rng.integers(0, 2, n).astype(np.uint16)
        return ((s << 15) | (e << 10) | m).view(np.uint8).reshape(n, 2)
    if dtype in (O.Q4_K, O.Q5_K):
        b[:, 0:2] = normal_f16(nblocks)
        b[:, 2:4] = normal_f16(nblocks)
    else:
        b[:, 208:210] = normal_f16(nblocks)
    return b


def main():
    w = O.seeded_weights(N, K, seed=0)
    x = O.seeded_acts(M, K, seed=1)
    out = {"w": w, "x": x}
    gt = {O.Q4_0: T.Q4_0, O.Q8_0: T.Q8_0, O.Q4_K: T.Q4_K, O.Q5_K: T.Q5_K, O.Q6_K: T.Q6_K}
    names = {O.Q4_0: "q4_0", O.Q8_0: "q8_0", O.Q4_K: "q4k", O.Q5_K: "q5k", O.Q6_K: "q6k"}
    for dt in (O.Q4_0, O.Q8_0):
        b = quants.quantize(w, gt[dt])
        out[f"{names[dt]}_bytes"] = b
        out[f"{names[dt]}_dequant"] = quants.dequantize(b, gt[dt])
        out[f"ref_{names[dt]}_y"] = O.matmul_reference_impl(dt, x, b, N)
    out["act_q8_0_bytes"] = quants.quantize(x, T.Q8_0)
    for dt, gtype, nm in ((O.Q4_1, T.Q4_1, "q4_1"), (O.Q5_0, T.Q5_0, "q5_0"), (O.Q5_1, T.Q5_1, "q5_1")):
        b = quants.quantize(w, gtype)
        out[f"{nm}_bytes"] = b
        out[f"{nm}_dequant"] = quants.dequantize(b, gtype)
        out[f"ref_{nm}_dequant"] = O.dequantize_reference_impl(dt, b, N * K).reshape(N, K)
        out[f"ref_{nm}_y"] = O.matmul_reference_impl(dt, x, b, N)
    rng = np.random.default_rng(7)
    for dt in (O.Q4_K, O.Q5_K, O.Q6_K):
        b = O.quantize(dt, w)
        out[f"{names[dt]}_bytes"] = b
        out[f"{names[dt]}_dequant"] = quants.dequantize(b, gt[dt])
        rb = rand_kquant_blocks(rng, dt, 16)
        out[f"{names[dt]}_rand_bytes"] = rb
        out[f"{names[dt]}_rand_dequant"] = quants.dequantize(rb, gt[dt])
    # ragged K (reference handles K % 32 != 0 inside the last block)
    Kr = 80
    wr = O.seeded_weights(8, 96, seed=3)
    xr = O.seeded_acts(2, Kr, seed=4)
    for dt in (O.Q4_0, O.Q8_0):
        b = quants.quantize(wr, gt[dt])
        out[f"ragged_{names[dt]}_bytes"] = b
        out[f"ragged_ref_{names[dt]}_y"] = O.matmul_reference_impl(dt, xr, b, 8)
    out["ragged_x"] = xr
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
