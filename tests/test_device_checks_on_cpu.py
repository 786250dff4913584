"""The optional device-check build (``VO_DEVICE_CHECKS=1``): kernels that use ``VO_DCHECK`` compile for sm_100a
with the checks in and with them compiled out (nvcc cross-compiles without a GPU)."""

import os
import shutil
import subprocess

import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "verl_omni_b200", "csrc")


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not installed")
@pytest.mark.parametrize("checks", [False, True])
def test_decode_kernel_compiles_with_and_without_device_checks(tmp_path, checks):
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-I", CSRC, "-c",
           os.path.join(CSRC, "decode_attn_sm100.cu"), "-o", str(tmp_path / "k.o")]
    if checks:
        cmd.insert(1, "-DVO_DEVICE_CHECKS")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert (tmp_path / "k.o").stat().st_size > 0


def test_device_check_macro_evaluates_to_its_condition():
    src = open(os.path.join(CSRC, "dcheck.cuh")).read()
    assert "#define VO_DCHECK(cond) (static_cast<bool>(cond))" in src  # compiled-out form keeps the condition
    assert "atomicCAS(&vo_dcheck_site_" in src  # checked form records the first failing line, never traps
    assert "__trap" not in src and "assert(" not in src
