"""GPU: tensor-parallel decode (2 GPUs, more when present) against the
single-GPU engine, through blocktensor_b200.tp_check under torchrun.

Bars: the greedy tokens of the whole run identical, and the last step's
per-layer activations within the engine tests' 1e-2 relative bar (the ranks'
partial sums are added in a different order than the single-GPU GEMV's).
Skipped on a box with one GPU.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,shape", [(2, "mha"), (4, "mha"), (8, "mha"), (2, "gqa"), (4, "gqa")])
def test_tp_decode_matches_single_gpu(cuda, world, shape, tmp_path):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           "-m", "blocktensor_b200.tp_check", str(out), shape]
    r = subprocess.run(["timeout", "-k", "30", "240"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = json.loads(out.read_text())
    assert res["tokens"] == res["want"], "tensor-parallel greedy tokens differ from the single-GPU engine"
    assert res["tap_err_max"] <= 1e-2
