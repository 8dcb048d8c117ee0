"""The drop-in host layer (include/sil_b200/gpu.h) on the CPU: silarray's own
array.h front-end over a host-memory test double of the CUDA runtime and of
libsilcu (tests/dropin/hostmock/), running tests/dropin/chain_fusion.cpp.
This checks the host logic of the chain fusion -- which nodes join a chain,
register allocation, which intermediates are still referenced and stored,
the launch count -- without a GPU; tests/test_dropin.py runs the same
program on the B200 against the real library.  Needs the reference sources
(SILARRAY_REF) for array.h."""
import os
import subprocess
import sysconfig

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("SILARRAY_REF", "/root/reference")


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "include", "array.h")),
                    reason="reference sources not present (set SILARRAY_REF)")
def test_chain_fusion_host_logic(tmp_path):
    gen = tmp_path / "gen"
    gen.mkdir()
    subprocess.run(["python", os.path.join(ROOT, "oracle", "patch_ref.py"), os.path.join(REF, "include"),
                    str(gen / "array.h"), "--dropin"], check=True)
    blasdir = os.path.join(sysconfig.get_paths()["purelib"], "opencv_python_headless.libs")
    blas = [os.path.join(blasdir, f) for f in os.listdir(blasdir) if f.startswith("libopenblasp-")]
    exe = tmp_path / "chain_fusion_host"
    inc = lambda p: ["-I", os.path.join(ROOT, p)]  # noqa: E731
    cmd = (["g++", "-std=c++23", "-O1", "-w"] + inc("tests/dropin/hostmock") + inc("include/sil_b200") +
           inc("include") + ["-I", str(gen)] + inc("include/sil_b200/compat") +
           ["-I", os.path.join(REF, "include"), "-o", str(exe),
            os.path.join(ROOT, "tests/dropin/chain_fusion.cpp"),
            os.path.join(ROOT, "tests/dropin/hostmock/silcu_host.cpp")] + blas[:1] +
           [f"-Wl,-rpath,{blasdir}"])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    env = dict(os.environ, LD_LIBRARY_PATH=blasdir)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and "PASSED" in r.stdout, r.stdout[-3000:] + r.stderr[-2000:]
