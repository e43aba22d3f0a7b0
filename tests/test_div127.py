"""The q8_0 quantizers divide amax by 127 with Markstein's correction step
(kvm_quant.cuh div127) instead of an IEEE division; this checks the identity
on the host over a dense sample of all non-negative finite floats (the full
sweep is `div127_check 1`)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_div127_matches_ieee_division(tmp_path):
    exe = tmp_path / "div127_check"
    # -mfma: fmaf must be the fused instruction; no contraction of a * r
    subprocess.run(["gcc", "-O2", "-mfma", "-ffp-contract=off", "-o", str(exe),
                    os.path.join(HERE, "cpp", "div127_check.c"), "-lm"], check=True)
    out = subprocess.run([str(exe), "13"], check=True, capture_output=True, text=True).stdout
    assert "mismatches 0" in out, out
