"""Host-side checks of native logic that needs no GPU."""

import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, REPO

CSRC = os.path.join(REPO, "blockstreamer_b200", "csrc")


@pytest.fixture(scope="module")
def e2m1_check(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("native") / "e2m1_host_check")
    src = os.path.join(REPO, "tests", "native", "e2m1_host_check.cu")
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-I", os.path.join(REPO, "include"), "-I", CSRC,
                    src, "-o", exe], check=True)
    res = subprocess.run([exe], capture_output=True, text=True)
    return res


def test_e2m1_decode_matches_reference_sweep(e2m1_check):
    """The library's general e2m1 decode equals the reference dequant for every
    byte under every e8m0 scale (golden sweep from dequantize_expert)."""
    lines = e2m1_check.stdout.splitlines()
    tab = np.array([[int(v, 16) for v in ln.split()] for ln in lines[: 256 * 256]], dtype=np.uint16)
    tab = tab.reshape(256, 256, 2)  # [scale][byte][lo/hi]
    golden = np.load(os.path.join(GOLDEN, "dequant_sweep.npz"))["bits"]  # [512 k, 256 rows=scale]
    # golden row r uses scale r; element k comes from byte k//2 (low nibble for even k)
    k = np.arange(512)
    byte = k // 2
    half = k % 2
    for s in range(256):
        assert np.array_equal(tab[s, byte, half], golden[:, s]), f"scale {s}"


def test_e2m1_fast_decode_equals_general(e2m1_check):
    last = e2m1_check.stdout.splitlines()[-1]
    assert last.startswith("MISMATCHES 0"), last
    assert e2m1_check.returncode == 0
