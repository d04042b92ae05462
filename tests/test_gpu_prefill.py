"""GPU parity of the multi-token tensor-core GEMM and of prompt prefill.

The reference runs a prompt one position at a time through
forward_single_token (benchmarks/bench_runner.cpp:107-109); prefill runs all
but the last prompt position as batched GEMMs with causal attention, and the
decode step takes over at the last prompt token.  Bars: the GEMM per token row
within 1e-5 of sum |s q x| of the oracle's matvec (the GEMV bar); K/V rows and
per-layer activations within 1e-2; greedy tokens identical to the oracle's
(the reference engine's for the tiny config) for the first 32 generated tokens.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = 1e-2


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.mark.parametrize("M,K,T", [(4096, 4096, 1), (4096, 4096, 33), (1000, 11008, 64), (288, 288, 5),
                                   (864, 288, 100), (33, 2816, 17), (22016, 4096, 32)])
def test_gemm_units_vs_oracle(cuda, oracle, M, K, T):
    import torch
    rng = np.random.default_rng(M + 7 * K + T)
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    x = rng.standard_normal((T, K)).astype(np.float32)
    units = cuda.pack_q8_units(dev(torch, b.view(np.uint8)), M, K)
    got = cuda.gemm_q8_units(units, dev(torch, x), M, K).cpu().numpy()
    nb = K // 32
    sq = np.abs(b["scale"].reshape(M, nb, 1) * b["qs"].reshape(M, nb, 32).astype(np.float64))
    for t in range(T):
        want = oracle.matvec_q8_0(b, x[t], M, K, nthreads=8)
        mag = (sq * np.abs(x[t].reshape(1, nb, 32))).sum(axis=(1, 2))
        err = np.abs(got[t].astype(np.float64) - want)
        assert (err <= 1e-5 * mag + 1e-30).all(), f"token {t}: worst relative error {np.max(err / (mag + 1e-30))}"


def test_gemm_units_outlier_blocks(cuda, oracle):
    """Per-token, per-block exponents: outlier blocks of one token cost neither its other
    blocks nor the other tokens precision."""
    import torch
    from test_gpu_kernels import outlier_case
    M, K = 4096, 4096
    b, x1, want1, mag1 = outlier_case(oracle, M, K, seed=5)
    rng = np.random.default_rng(6)
    x0 = rng.standard_normal(K).astype(np.float32)
    x = np.stack([x0, x1, x0 * 1e-3])
    units = cuda.pack_q8_units(dev(torch, b.view(np.uint8)), M, K)
    got = cuda.gemm_q8_units(units, dev(torch, x), M, K).cpu().numpy()
    nb = K // 32
    sq = np.abs(b["scale"].reshape(M, nb, 1) * b["qs"].reshape(M, nb, 32).astype(np.float64))
    for t in range(3):
        want = oracle.matvec_q8_0(b, x[t], M, K, nthreads=8)
        mag = (sq * np.abs(x[t].reshape(1, nb, 32))).sum(axis=(1, 2))
        err = np.abs(got[t].astype(np.float64) - want)
        assert (err <= 1e-5 * mag + 1e-30).all(), f"token {t}: worst relative error {np.max(err / (mag + 1e-30))}"


def test_gemm_zero_and_scaling(cuda, oracle):
    """Zero rows give exact zeros; a power-of-two scale of a token scales its row exactly."""
    import torch
    M, K = 512, 1024
    rng = np.random.default_rng(8)
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    units = cuda.pack_q8_units(dev(torch, b.view(np.uint8)), M, K)
    x = rng.standard_normal((4, K)).astype(np.float32)
    x[1] = 0.0
    x[2] = x[0] * 4.0
    got = cuda.gemm_q8_units(units, dev(torch, x), M, K).cpu().numpy()
    assert (got[1] == 0).all()
    assert np.array_equal(got[2], got[0] * 4.0)


# ---------------------------------------------------------------- prefill on the tiny config

@pytest.fixture(scope="module")
def tiny_engine(cuda):
    from blocktensor_b200 import synthetic
    eng = cuda.TransformerEngine(synthetic.config("tiny", 256))
    eng.generate(seed=0, sigma=0.02)
    yield eng
    eng.close()


@pytest.mark.parametrize("kv_dtype", ["fp32", "fp16"])
def test_tiny_prefill_greedy_tokens(cuda, tiny_engine, kv_dtype):
    """16-token prompt prefilled, then 128 greedy steps: the reference's greedy tokens."""
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    want = g["tokens"] if kv_dtype == "fp32" else g["tokens_kv16"]
    kv = cuda.KVCache(tiny_engine, 256, cuda.BT_KV_FP32 if kv_dtype == "fp32" else cuda.BT_KV_FP16)
    got = tiny_engine.generate_tokens(kv, g["prompt"], n_gen=128)
    assert len(got) == 16 + 128 + 1
    assert np.array_equal(got[:16], g["prompt"])
    first = 16 + 32
    assert np.array_equal(got[:first], want[:first]), "first 32 generated tokens differ"
    bad = np.nonzero(got[: len(want)] != want[: len(got)])[0]
    assert bad.size == 0, f"greedy tokens diverge at positions {bad[:5]} (margins {g['margins'][bad[:5] - 1]})"
    kv.close()


def test_tiny_prefill_kv_and_taps(cuda, oracle, tiny_engine):
    """After prefill the cache holds the oracle's K/V rows of the 15 prefilled positions, and
    the step at the last prompt position gives the oracle's taps and logits."""
    from blocktensor_b200 import synthetic
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    prompt = g["prompt"]
    cfg = tiny_engine.config
    ocfg = oracle.make_config(*synthetic.SHAPES["tiny"], 256)
    m = oracle.Model(ocfg, seed=0)
    okv = oracle.KV(ocfg, 256)
    for p in range(15):
        oracle.forward_token(m, okv, int(prompt[p]), p)
    kv = cuda.KVCache(tiny_engine, 256)
    tiny_engine.prefill(kv, prompt)
    n = 15 * cfg.num_kv_heads * cfg.head_dim
    for l in range(cfg.num_layers):
        k, v = kv.read_layer(l)
        ok, ov = okv.layer(l)
        assert rel_l2(k[:n], ok[:n]) <= TOL and rel_l2(v[:n], ov[:n]) <= TOL, f"layer {l} K/V rows"
        np.testing.assert_allclose(k[:n], ok[:n], rtol=TOL, atol=TOL)
        np.testing.assert_allclose(v[:n], ov[:n], rtol=TOL, atol=TOL)
    lo, otaps = oracle.forward_token(m, okv, int(prompt[15]), 15, want_taps=True)
    tiny_engine.set_taps(True)
    try:
        tiny_engine.steps(kv, 1)
        taps = tiny_engine.read_taps()
    finally:
        tiny_engine.set_taps(False)
    for l in range(cfg.num_layers):
        assert rel_l2(taps[l], otaps[l]) <= TOL, f"layer {l}: {rel_l2(taps[l], otaps[l])}"
    pos, tok, am = kv.state()
    assert pos == 16 and am == oracle.sample_greedy(lo)
    kv.close()
    m.close()


def test_prefill_multi_chunk_matches_decode_loop(cuda, oracle):
    """A 1100-token prompt (three prefill chunks, the later ones attending to the earlier
    chunks' cache) against the oracle run position by position: K/V rows within 1e-2 and
    the greedy continuation identical."""
    d = dict(vocab=512, dim=256, hidden=512, layers=2, heads=4, kv_heads=2, head_dim=64, max_seq=1200)
    cfg = cuda.model_config(*d.values())
    ocfg = oracle.make_config(*d.values())
    m = oracle.Model(ocfg, seed=3)
    eng = cuda.TransformerEngine(cfg)
    eng.load_pointers([(t.ptr, t.nbytes) for t in m.tensors()])
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, 512, 1100).astype(np.uint32)
    n_gen = 40
    kv = cuda.KVCache(eng, 1200)
    got = eng.generate_tokens(kv, prompt, n_gen=n_gen)
    okv = oracle.KV(ocfg, 1200)
    toks = [int(prompt[0])]
    for p in range(1100 + n_gen):
        lo = oracle.forward_token(m, okv, toks[p], p)
        toks.append(int(prompt[p + 1]) if p + 1 < 1100 else oracle.sample_greedy(lo))
    n = 1099 * cfg.num_kv_heads * cfg.head_dim
    for l in range(cfg.num_layers):
        k, v = kv.read_layer(l)
        ok, ov = okv.layer(l)
        assert rel_l2(k[:n], ok[:n]) <= TOL and rel_l2(v[:n], ov[:n]) <= TOL, f"layer {l}"
    assert np.array_equal(got, np.array(toks, np.uint32)[: len(got)])
    kv.close()
    eng.close()
    m.close()


def test_prefill_errors(cuda, tiny_engine):
    kv = cuda.KVCache(tiny_engine, 8)
    with pytest.raises(ValueError):
        tiny_engine.prefill(kv, [])
    with pytest.raises(IndexError):
        tiny_engine.prefill(kv, list(range(9)))          # 9 positions > 8
    with pytest.raises(IndexError):
        tiny_engine.prefill(kv, [1, 2, 32000])            # token >= vocab
    tiny_engine.prefill(kv, [1, 2, 3])
    assert kv.state()[0] == 2
    kv.close()
