"""GPU parity at full size: the Llama-2-7B-shaped int8 model (seed 0) generated on
the device against the golden tokens, logits and residual taps of the oracle
(pinned to the reference engine for the first steps; tests/golden/make_golden.py).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = 1e-2


def close(gpu, ref, what):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(gpu - ref) > TOL * (1.0 + np.abs(ref))
    assert not bad.any(), f"{what}: {bad.sum()} outside 1e-2, worst {np.abs(gpu - ref).max()}"
    rel = np.linalg.norm(gpu - ref) / np.linalg.norm(ref)
    assert rel <= TOL, f"{what}: relative L2 {rel}"


@pytest.fixture(scope="module")
def golden():
    path = os.path.join(GOLDEN, "llama7b_c2.npz")
    if not os.path.exists(path):
        pytest.skip("llama7b_c2.npz not generated")
    return np.load(path)


@pytest.fixture(scope="module")
def engine7b(cuda, golden):
    from blocktensor_b200 import synthetic
    cfg = synthetic.config("llama2-7b", 1024)
    assert bytes(cfg) == golden["config"].tobytes()
    eng = cuda.TransformerEngine(cfg)
    eng.generate(seed=0, sigma=0.02)
    yield eng
    eng.close()


@pytest.mark.parametrize("kv", ["kv32", "kv16"])
def test_7b_greedy_tokens_and_activations(cuda, golden, engine7b, kv):
    eng = engine7b
    prompt = golden["prompt"]
    want = golden[f"{kv}_tokens"]
    n_prompt, n_gen = len(prompt), len(want) - len(prompt)
    kvc = cuda.KVCache(eng, n_prompt + n_gen + 1, cuda.BT_KV_FP32 if kv == "kv32" else cuda.BT_KV_FP16)
    # logits and taps at the last prompt position
    eng.set_taps(True)
    try:
        for p in range(n_prompt):
            lg = eng.forward_single_token(int(prompt[p]), p, kvc)
        taps = eng.read_taps()
    finally:
        eng.set_taps(False)
    close(lg, golden[f"{kv}_logits_last_prompt"], "logits at the last prompt position")
    for i, l in enumerate([0, 1, 15, 31]):
        close(taps[l], golden[f"{kv}_taps_last_prompt"][i], f"residual after layer {l}")
    np.testing.assert_allclose(np.linalg.norm(taps, axis=1), golden[f"{kv}_tap_norms_last_prompt"], rtol=TOL)
    # greedy decode on the device: the first 32 generated tokens are identical
    kvc2 = cuda.KVCache(eng, n_prompt + n_gen + 1, kvc.kv_dtype)
    got = eng.decode(kvc2, prompt, n_gen=n_gen - 1)
    assert np.array_equal(got[: len(want)], want[: len(got)]), (got, want)
