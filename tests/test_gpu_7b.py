"""GPU parity at full size: the Llama-2-7B-shaped int8 model (seed 0) generated on
the device against the golden tokens, logits and residual taps of the oracle
(pinned to the reference engine for the first steps; tests/golden/make_golden.py).

Bars: the first 32 generated greedy tokens identical; per-layer residual
activations within 1e-2 relative error (L2 norm of the difference over the
norm of the oracle's vector).  With the fp32 KV cache, the configuration the
reference engine itself runs, the elementwise form of the reference's tests
(|a - b| <= 1e-2 (1 + |b|)) must hold as well; with the fp16 cache, rounding
K/V to fp16 turns last-bit fp32 differences into occasional 1-ulp fp16 steps,
which 32 layers amplify past the elementwise form on a few elements of the
last layers while the relative error stays far inside 1e-2.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = 1e-2


def rel_l2(gpu, ref):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.linalg.norm(gpu - ref) / np.linalg.norm(ref)


def elementwise_ok(gpu, ref):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(gpu - ref) <= TOL * (1.0 + np.abs(ref))


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
def test_7b_greedy_tokens(cuda, golden, engine7b, kv):
    eng = engine7b
    prompt = golden["prompt"]
    want = golden[f"{kv}_tokens"]
    n_prompt, n_steps = len(prompt), len(want) - 1
    kvc = cuda.KVCache(eng, n_steps + 1, cuda.BT_KV_FP32 if kv == "kv32" else cuda.BT_KV_FP16)
    got = eng.decode(kvc, prompt, n_gen=n_steps - n_prompt)
    assert len(got) == len(want)
    first = n_prompt + 32
    assert np.array_equal(got[:first], want[:first]), (got, want)
    kvc.close()


@pytest.mark.parametrize("kv", ["kv32", "kv16"])
def test_7b_layer_activations(cuda, golden, engine7b, kv):
    eng = engine7b
    prompt = golden["prompt"]
    kvc = cuda.KVCache(eng, len(prompt) + 1, cuda.BT_KV_FP32 if kv == "kv32" else cuda.BT_KV_FP16)
    eng.set_taps(True)
    try:
        for p in range(len(prompt)):
            lg = eng.forward_single_token(int(prompt[p]), p, kvc)
        taps = eng.read_taps()
    finally:
        eng.set_taps(False)
    ref_logits = golden[f"{kv}_logits_last_prompt"]
    assert rel_l2(lg, ref_logits) <= TOL
    assert int(np.argmax(lg)) == int(np.argmax(ref_logits))
    for i, l in enumerate([0, 1, 15, 31]):
        ref = golden[f"{kv}_taps_last_prompt"][i]
        assert rel_l2(taps[l], ref) <= TOL, f"layer {l}: relative error {rel_l2(taps[l], ref)}"
        if kv == "kv32":
            ok = elementwise_ok(taps[l], ref)
            assert ok.all(), f"layer {l}: {(~ok).sum()} elements outside the elementwise 1e-2 form"
    if kv == "kv32":
        assert elementwise_ok(lg, ref_logits).all()
    np.testing.assert_allclose(np.linalg.norm(taps, axis=1), golden[f"{kv}_tap_norms_last_prompt"], rtol=TOL)
    kvc.close()


# ---------------------------------------------------------------- the benchmarked configuration
# A 512-token prompt, then greedy decode at contexts 513-544, as bench.py runs it (fp16 KV),
# and with the fp32 cache the reference engine itself uses.

@pytest.fixture(scope="module")
def golden512():
    path = os.path.join(GOLDEN, "llama7b_c2_p512.npz")
    if not os.path.exists(path):
        pytest.skip("llama7b_c2_p512.npz not generated")
    return np.load(path)


def _check_taps(taps, logits, g, kv, tag):
    layers = [int(l) for l in g["tap_layers"]]
    ref_logits = g[f"{kv}_logits_{tag}"]
    assert rel_l2(logits, ref_logits) <= TOL, f"{tag}: logits relative error {rel_l2(logits, ref_logits)}"
    assert int(np.argmax(logits)) == int(np.argmax(ref_logits))
    for i, l in enumerate(layers):
        ref = g[f"{kv}_taps_{tag}"][i]
        assert rel_l2(taps[l], ref) <= TOL, f"{tag} layer {l}: relative error {rel_l2(taps[l], ref)}"
        if kv == "kv32":
            ok = elementwise_ok(taps[l], ref)
            assert ok.all(), f"{tag} layer {l}: {(~ok).sum()} elements outside the elementwise 1e-2 form"
    np.testing.assert_allclose(np.linalg.norm(taps, axis=1), g[f"{kv}_tap_norms_{tag}"], rtol=TOL)


@pytest.mark.parametrize("kv", ["kv16", "kv32"])
def test_7b_prompt512_tokens_and_taps(cuda, golden512, engine7b, kv):
    """Positions 0-510 as one device decode, position 511 (last prompt token) through
    forward_single_token with taps, 512-542 as a second device decode continuing the
    same cache, and 543 through forward_single_token with taps: the 32 generated
    tokens and the final argmax must equal the oracle's, the taps and logits at 511
    and 543 be within 1e-2."""
    eng, g = engine7b, golden512
    prompt = g["prompt"]
    want = g[f"{kv}_tokens"]
    n_prompt = len(prompt)
    n_gen = len(want) - 1 - n_prompt
    assert n_prompt == 512 and n_gen == 32
    kvc = cuda.KVCache(eng, n_prompt + n_gen + 1, cuda.BT_KV_FP32 if kv == "kv32" else cuda.BT_KV_FP16)
    got = list(eng.decode(kvc, prompt[:n_prompt - 1], n_gen=0)[:n_prompt - 1])
    eng.set_taps(True)
    try:
        lg = eng.forward_single_token(int(prompt[n_prompt - 1]), n_prompt - 1, kvc)
        _check_taps(eng.read_taps(), lg, g, kv, "last_prompt")
        got.append(int(prompt[n_prompt - 1]))
        first = eng.last_argmax
        eng.set_taps(False)
        mid = eng.decode(kvc, [first], n_gen=n_gen - 2, pos0=n_prompt)  # positions 512 .. 542
        got.extend(int(t) for t in mid[:-1])
        last = int(mid[-1])
        eng.set_taps(True)
        lg = eng.forward_single_token(last, n_prompt + n_gen - 1, kvc)
        _check_taps(eng.read_taps(), lg, g, kv, "last_gen")
        got.append(last)
        got.append(eng.last_argmax)
    finally:
        eng.set_taps(False)
    got = np.array(got, np.uint32)
    assert len(got) == len(want)
    assert np.array_equal(got[:n_prompt], prompt)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"greedy tokens differ at positions {bad[:8]} (margins {g[f'{kv}_margins'][bad[:8] - 1]})"
    kvc.close()


@pytest.mark.parametrize("kv", ["kv16", "kv32"])
def test_7b_prompt512_prefill(cuda, golden512, engine7b, kv):
    """The 512-token prompt through prefill (positions 0-510 as batched GEMMs), the last
    prompt position through the decode step with taps, then 32 greedy steps: taps and
    logits at position 511 within 1e-2 and the 32 generated tokens identical."""
    eng, g = engine7b, golden512
    prompt = g["prompt"]
    want = g[f"{kv}_tokens"]
    n_prompt, n_gen = 512, 32
    kvc = cuda.KVCache(eng, n_prompt + n_gen + 1, cuda.BT_KV_FP32 if kv == "kv32" else cuda.BT_KV_FP16)
    eng.prefill(kvc, prompt)
    eng.set_taps(True)
    try:
        eng.steps(kvc, 1)
        taps = eng.read_taps()
    finally:
        eng.set_taps(False)
    layers = [int(l) for l in g["tap_layers"]]
    for i, l in enumerate(layers):
        ref = g[f"{kv}_taps_last_prompt"][i]
        assert rel_l2(taps[l], ref) <= TOL, f"layer {l}: relative error {rel_l2(taps[l], ref)}"
    np.testing.assert_allclose(np.linalg.norm(taps, axis=1), g[f"{kv}_tap_norms_last_prompt"], rtol=TOL)
    eng.steps(kvc, n_gen)  # positions 512 .. 543
    got = kvc.read_tokens(0, n_prompt + n_gen + 1)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"greedy tokens differ at positions {bad[:8]} (margins {g[f'{kv}_margins'][bad[:8] - 1]})"
    kvc.close()
