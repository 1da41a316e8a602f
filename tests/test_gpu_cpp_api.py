"""The C++ QuasarML layer (qsml:: / QuasarML::Ops over libqsml_cuda.so) run
on the GPU: tests/cpp/test_qsml_api.cpp restates the reference's unit-test
known answers and checks the ops this backend adds; it exits nonzero on any
failed check."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "quasarml_b200", "cpp", "_build", "test_qsml_api")


@pytest.mark.gpu
def test_cpp_api_program():
    assert os.path.exists(BIN), "build the C++ layer first (make -C quasarml_b200/cpp)"
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "failed 0" in r.stdout
