"""The reference's unit-test cases (tests/test_tensor.cpp, test_nn.cpp,
test_rope.cpp, test_quant.cpp) run against the C++ Tensor/nn API of the host
layer on the GPU: turbo.cpp_b200/host/tests/test_host.cpp."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "turbo.cpp_b200", "host", "tests", "test_host")


def test_host_api_reference_cases():
    if not os.path.exists(BIN):
        pytest.fail("test_host is not built (python turbo.cpp_b200/build.py)")
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
