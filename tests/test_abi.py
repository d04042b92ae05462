"""CPU: the C-ABI library loads and exports exactly what include/bt_cuda.h declares."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "bt_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^BT_API\s+[\w\s\*]+?\b(bt_\w+)\s*\(", src, flags=re.M)))


def exported_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return sorted({line.split()[-1] for line in out.splitlines() if " T " in line})


def test_header_declares_symbols():
    syms = declared_symbols()
    assert "bt_engine_forward_token" in syms and "bt_cuda_quantize_q8_0" in syms
    assert len(syms) >= 25


def test_library_exports_every_declared_symbol():
    import blocktensor_b200.native as nat
    assert os.path.exists(nat.LIB_PATH), "build with python -m blocktensor_b200.build"
    exported = set(exported_symbols(nat.LIB_PATH))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    extra = [s for s in exported if s.startswith("bt_") and s not in declared_symbols()]
    assert not extra, f"exported but not declared: {extra}"


def test_python_binding_matches_header():
    import blocktensor_b200.native as nat
    assert sorted(nat.SIGNATURES) == declared_symbols()


def test_library_loads_without_gpu():
    import blocktensor_b200 as bt
    lib = bt.load()
    assert lib.bt_cuda_abi_version() == 1
    # no compute here: only argument validation that never reaches the device
    assert lib.bt_cuda_quantize_q8_0(None, None, 33, None) == bt.native.BT_ERR_INVALID_ARGUMENT
    assert "multiple of block size" in bt.native.last_error()


def test_status_mapping():
    import blocktensor_b200.native as nat
    with pytest.raises(IndexError):
        nat.check(nat.BT_ERR_OUT_OF_RANGE)
    with pytest.raises(ValueError):
        nat.check(nat.BT_ERR_INVALID_ARGUMENT)
    with pytest.raises(RuntimeError):
        nat.check(nat.BT_ERR_RUNTIME)
    with pytest.raises(nat.CudaBackendError):
        nat.check(nat.BT_ERR_CUDA)
    nat.check(nat.BT_OK)


def test_config_layout_matches_reference():
    """bt_model_config is byte-compatible with the reference ModelConfig (36 bytes)."""
    import blocktensor_b200 as bt
    from oracle import oracle as O
    c = bt.model_config(32000, 4096, 11008, 32, 32, 32, 128, 1024)
    o = O.make_config(32000, 4096, 11008, 32, 32, 32, 128, 1024)
    assert bytes(c) == bytes(o) and ctypes.sizeof(c) == 36
    if O.ref_available():
        assert O.RefLib().btr_sizeof_config() == 36
        assert O.RefLib().btr_sizeof_block_q8_0() == 36
