"""Run-to-run reproducibility of the products: the same call repeated gives
bit-identical outputs.

Every reduction in the CUDA path has a fixed order (unit parities, then the
cluster ranks in rank order), so any difference between repeats is a race --
e.g. a ring slot refilled by a bulk copy while a thread's reads of it were
still outstanding.  The shapes cover each split the plan picks for the
streaming GEMV (one CTA per row tile up to clusters of 8), the 8-token
mma.sync units, the on-chip staging and the Q8-records staging.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

CASES = [
    (O.Q8_0, 32000, 4096, 8),   # split 4, 8-token units, two ring stages
    (O.Q8_0, 11008, 4096, 8),
    (O.Q8_0, 4096, 11008, 8),
    (O.Q4_0, 11008, 4096, 8),
    (O.Q6_K, 32000, 4096, 8),
    (O.Q4_K, 4096, 14336, 1),   # split 8, one token, on-chip staging
    (O.Q4_K, 32000, 4096, 1),
    (O.Q5_K, 4096, 4096, 4),
    (O.Q8_0, 4096, 4096, 2),
]


def _weights(ob, dt, N, K, seed):
    import torch

    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    wf = torch.empty((N, K), dtype=torch.float32, device="cuda").normal_(0.0, 0.02, generator=gen)
    tiled = ob.repack(dt, ob.quantize_weight(dt, wf), N, K)
    x = torch.empty((8, K), dtype=torch.float32, device="cuda").normal_(0.0, 1.0, generator=gen)
    return tiled, x


@pytest.mark.parametrize("dt,N,K,M", CASES)
def test_repeats_bit_identical(cuda_lib, dt, N, K, M):
    import torch

    ob = cuda_lib
    tiled, x8 = _weights(ob, dt, N, K, seed=N + K + M)
    x = x8[:M].contiguous()
    ws = ob.new_workspace(ob.workspace_bytes(dt, M, N, K, ob.ACT_Q8))
    ys = []
    for _ in range(40):
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        ob.matmul_dev(dt, tiled, x, y, N, K, ob.ACT_Q8, ws)
        ys.append(y)
    torch.cuda.synchronize()
    assert ob.workspace_status(ws) == 0
    Y = torch.stack(ys).cpu().numpy()
    assert np.isfinite(Y).all()
    differ = (Y != Y[:1]).any(axis=0)
    assert not differ.any(), f"{int(differ.sum())} outputs differ between repeats"
