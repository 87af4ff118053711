"""GPU parity of the C++ host layer: runs tests/cpp/test_device_runners.cpp, which drives every
operator through the harness's C++ runners (host/include/harness/device_ops.hpp -> the C ABI ->
the CUDA kernels) on the reference test suites' cases and compares with the CPU oracle."""
from __future__ import annotations

import pytest

from test_cpp_host import build_cpp_tests, run_binary

pytestmark = pytest.mark.gpu


def test_device_runners_cpp(cuda, hc_lib):
    import build

    build.build_host()
    build_cpp_tests(hc_lib)
    r = run_binary("test_device_runners", 900)
    print(r.stdout[-4000:])
    assert r.returncode == 0, r.stdout[-8000:] + r.stderr[-2000:]
    assert "FAILED" not in r.stdout
