"""The C++ host mirror (go-whistle_b200/host/whistle.hpp: cq::New, Matrix,
GEMMs, needle::QuantizeRow, Int8Rows, AttendInt8Spans) through its test
program tests/cpp/test_host.cpp, written like the reference's Go tests:
validation and panics on the CPU, parity with the oracle on the GPU."""

from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

CPP = Path(__file__).resolve().parent / "cpp"


def _program(wb, orc) -> Path:
    """Builds (make) and returns the test program; the fixtures built the
    product and the oracle it links."""
    r = subprocess.run(["make", "-C", str(CPP)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return CPP / "_build" / "test_host"


def _run(prog: Path, mode: str):
    r = subprocess.run([str(prog), mode], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout and "FAIL" not in r.stdout, r.stdout


def test_host_mirror_cpu(wb, orc):
    _run(_program(wb, orc), "--cpu")


@pytest.mark.gpu
def test_host_mirror_gpu(wb, orc, cuda):
    _run(_program(wb, orc), "--gpu")
