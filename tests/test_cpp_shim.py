"""The C++ drop-in headers (include/quantized.hpp, matmul_q4.hpp,
layer_moe.hpp) and their shim sources: they compile against libqmoe here,
and on a GPU the driver tests/cpp/shim_test.cpp checks them against the CPU
oracle and the reference's error messages."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
BIN = HERE / "cpp" / "_build" / "shim_test"


def _build():
    r = subprocess.run(["bash", str(HERE / "cpp" / "build.sh")], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_cpp_headers_and_shims_build():
    _build()
    assert BIN.exists()


@pytest.mark.gpu
def test_cpp_shim_driver_on_gpu():
    _build()
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
