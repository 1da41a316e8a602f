"""CPU checks of the C++ QuasarML layer: it is built, links only the C ABI
library (no torch, no CUDA runtime of its own) and exports the reference's
op names."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "quasarml_b200", "cpp", "libquasarml.so")


def _built():
    return os.path.exists(LIB)


@pytest.mark.skipif(not _built(), reason="C++ layer not built")
def test_exports_reference_op_names():
    out = subprocess.run(["nm", "-DC", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    for name in ("QuasarML::Ops::add(", "QuasarML::Ops::subtract(", "QuasarML::Ops::multiply(",
                 "QuasarML::Ops::divide(", "QuasarML::Ops::relu(", "QuasarML::Ops::sum(", "QuasarML::Ops::mean(",
                 "QuasarML::Ops::max(", "QuasarML::Ops::min(", "QuasarML::Ops::matmul(",
                 "QuasarML::Ops::batch_matmul(", "QuasarML::Ops::transpose(", "QuasarML::Ops::slice(",
                 "QuasarML::Ops::copy(", "QuasarML::Ops::reshape(", "QuasarML::Ops::pow(",
                 "QuasarML::Ops::layer_norm(", "QuasarML::Tensor::download(", "QuasarML::DeviceManager::instance("):
        assert name in out, name


@pytest.mark.skipif(not _built(), reason="C++ layer not built")
def test_links_only_the_c_abi():
    out = subprocess.run(["ldd", LIB], capture_output=True, text=True).stdout
    assert "libqsml_cuda.so" in out
    assert "libtorch" not in out and "libcudart" not in out
