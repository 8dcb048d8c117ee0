"""The drop-in check: silarray's own doctest suite (test/test_array.cpp,
test_examples.cpp, test_perceptron.cpp), compiled against the B200 backend
headers (include/sil_b200: gpu.h, unified_memory.h, device.h) and
libsilcu.so, run in GPU mode on the device.  The reference's array.h front-end
is unchanged except for the mechanical g++-13 rewrite of its seven
explicit-object members (oracle/patch_ref.py); the binary is built by
`make -C oracle dropin` where the reference sources are present."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "ref_tests_b200")


@pytest.mark.parametrize("mode", ["--gpu", ""])
def test_reference_suite_on_b200(cuda, mode):
    if not os.path.exists(BIN):
        pytest.skip("drop-in test binary not built (reference sources were absent at build time)")
    args = [BIN] + ([mode] if mode else [])
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "Status: SUCCESS" in r.stdout


def test_chain_fusion_through_sil_api(cuda):
    """tests/dropin/chain_fusion.cpp: chains of elementwise nodes evaluated
    through sil:: run as one fused launch (intermediates the caller holds are
    stored too), equal to the reference CPU path; the binary is built by
    `make -C oracle dropin`."""
    path = os.path.join(ROOT, "oracle", "_ref", "chain_fusion_b200")
    if not os.path.exists(path):
        pytest.skip("chain fusion program not built (reference sources were absent at build time)")
    r = subprocess.run([path], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "PASSED" in r.stdout
