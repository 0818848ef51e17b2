"""The Q8_0 activation quantiser's division-free arithmetic equals the gguf
quantiser's IEEE operations (d = amax / 127, q = roundf(v * (1 / d))).

The device helpers (q8_scale, q8_round in odiengine_b200/csrc/common.cuh)
replace the division by 127 with one residual correction of amax * RN(1/127)
and roundf with trunc(t + copysign(0.5 - 2^-25, t)).  tests/q8_math_check.c
restates both in host fp32 and compares them with the host's division and
roundf: here over a regular subset of the fp32 bit patterns (every 61st), and
over all of them when ODI_EXHAUSTIVE=1 (about 80 s on one core).  The GPU
side is covered by the bit-exact quantisation parity tests.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_q8_scale_and_round_match_ieee(tmp_path):
    exe = str(tmp_path / "q8_math_check")
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-std=c11", "-o", exe,
                    os.path.join(HERE, "q8_math_check.c"), "-lm"], check=True)
    stride = "1" if os.environ.get("ODI_EXHAUSTIVE") == "1" else "61"
    out = subprocess.run([exe, stride], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 mismatches; " in out.stdout and out.stdout.rstrip().endswith(" 0 mismatches")
