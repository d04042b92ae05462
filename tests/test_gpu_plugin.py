"""GPU: the C++ plugin (blocktensor_b200/cpp: CudaBackend, CudaTransformerEngine)
driven through the reference's own importer, MemoryManager, KVCache and engine.

The test binary is built here by `make -C oracle plugin` against the reference
sources (tests/cpp/plugin_test.cpp) and travels prebuilt; it compares the CUDA
engine with the reference TransformerEngine on its CPUBackend, dispatches the
pipelines by shader name, and checks the exception contract.
"""
import os
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

BIN = os.path.join(ROOT, "oracle", "_ref", "bt_plugin_test")


def test_plugin_through_reference_interfaces(cuda, tmp_path):
    if not os.path.exists(BIN):
        pytest.skip("oracle/_ref/bt_plugin_test not built (needs the reference source tree)")
    r = subprocess.run([BIN, str(tmp_path / "plugin.btmodel")], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    print(r.stderr)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PLUGIN TEST PASSED" in r.stdout
