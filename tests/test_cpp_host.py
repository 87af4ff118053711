"""Runs the C++ tests of the host layer on CPU (tests/cpp/test_host_layer.cpp): the accuracy pass
rule, host-side argument validation of the C++ runners, and that without a device every runner
throws harness::DeviceError instead of computing anything on the CPU."""
from __future__ import annotations

import subprocess
from pathlib import Path

CPP = Path(__file__).resolve().parent / "cpp"
ROOT = CPP.parents[1]


def build_cpp_tests(hc_lib) -> None:
    """libhc_b200.so + libhc_harness.so (hc_lib fixture / build.py), the oracle, then the test binaries."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True,
                   capture_output=True)
    r = subprocess.run(["make", "-s", "-C", str(CPP)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def run_binary(name: str, timeout: int) -> subprocess.CompletedProcess:
    return subprocess.run([str(CPP / "_bin" / name)], capture_output=True, text=True, timeout=timeout)


def test_host_layer_cpp(hc_lib):
    import build  # noqa: F401  (the package dir is on sys.path via conftest)

    build.build_host()
    build_cpp_tests(hc_lib)
    r = run_binary("test_host_layer", 120)
    assert r.returncode == 0, r.stdout[-6000:] + r.stderr[-2000:]
    assert "[  PASSED  ]" in r.stdout


def test_cmake_configures(tmp_path):
    """The CMake route (CMakeLists.txt: CUDA sm_100a library, host layer, oracle, CTest) configures here."""
    import shutil

    if shutil.which("cmake") is None:
        import pytest

        pytest.skip("cmake not installed")
    r = subprocess.run(["cmake", "-S", str(ROOT), "-B", str(tmp_path / "b"), "-G", "Ninja"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    ninja = (tmp_path / "b" / "build.ninja").read_text()
    assert "arch=compute_100a" in ninja and "test_device_runners" in ninja
