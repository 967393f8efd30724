"""The reference's own test programs, compiled unchanged against libhxq.so.

`make -C oracle reftests` builds test/test_hxq.c, test/test_affine.c,
test/test_lloyd.c, test/test_polarquant.c and test/test_affine_cuda.cu from
the reference tree with only this repository's headers on the include path
and links them with -lhxq (reference: test/test_hxq.c:40-326,
test/test_affine.c:69-462, test/test_lloyd.c, test/test_polarquant.c,
test/test_affine_cuda.cu:52-338).  A caller of the reference library that
relinks against this one sees exactly these results.  The programs live in
oracle/_ref (built where the reference tree is present; they travel with the
repository like the reference library).

test_hxq and test_affine exercise host-pointer paths (the CPU backend) and
run without a GPU.  Lloyd and PolarQuant compute on the GPU here, and
test_affine_cuda is the reference's GPU test, so those three are gpu tests.
"""
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(REPO, "oracle", "_ref")


def _binary(name):
    path = os.path.join(REF_BIN, name)
    if not os.path.exists(path):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "reftests"], check=False)
    if not os.path.exists(path):
        pytest.skip("reference test programs not built (no reference tree to compile them from)")
    return path


def _run(name, timeout=600):
    r = subprocess.run([_binary(name)], capture_output=True, text=True, timeout=timeout, cwd=REF_BIN)
    out = r.stdout + r.stderr
    m = re.findall(r"(\d+)/(\d+)\s+(?:tests\s+)?passed", out)
    assert m, out[-2000:]
    passed, total = (int(v) for v in m[-1])
    return r.returncode, passed, total, out


@pytest.mark.parametrize("name,expect", [("test_hxq", 41), ("test_affine", 32)])
def test_reference_cpu_suite(H, name, expect):
    rc, passed, total, out = _run(name)
    assert (passed, total) == (expect, expect), out[-3000:]
    assert rc == 0, out[-3000:]


@pytest.mark.gpu
@pytest.mark.parametrize("name,expect", [("test_lloyd", 14), ("test_polarquant", 37), ("test_affine_cuda", None)])
def test_reference_gpu_suite(H, cuda, name, expect):
    rc, passed, total, out = _run(name)
    print(out)
    assert passed == total, out[-3000:]
    if expect is not None:
        assert total == expect, out[-3000:]
    assert rc == 0, out[-3000:]
