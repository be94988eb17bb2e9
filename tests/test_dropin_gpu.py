"""Runs oracle/_ref/dropin_test: the reference's own C++ API, CPU code and
weight-upload path, with its GPU quant path replaced by
mini-llama_b200/cpp/cuda_quant_mlq.cc + libmlq.so (built by `make -C oracle
dropin` where the reference checkout exists; the binary ships with the
repository snapshot)."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
BIN = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "dropin_test"


def test_reference_api_runs_on_mlq():
    if not BIN.exists():
        pytest.skip("drop-in test binary not built (needs the reference checkout)")
    r = subprocess.run([str(BIN)], capture_output=True, text=True, timeout=600)
    print(r.stdout, r.stderr)
    if r.returncode == 2:
        pytest.skip("no CUDA device")
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("[PASS]") == 6
