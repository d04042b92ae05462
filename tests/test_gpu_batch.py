"""GPU parity of batched decode (bt_batch_*): independent sequences decoded together.

The reference decodes one sequence per KVCache (runtime/src/kv_cache.cpp:6-15);
a batch is n independent forward_single_token loops.  Every sequence of a batch
must therefore produce the oracle's own single-sequence greedy tokens (the first
32 generated tokens identical) and logits within 1e-2,
whatever the other sequences and their positions.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-2


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def oracle_run(oracle, m, ocfg, prompt, n_gen, max_seq, fp16):
    """Greedy tokens of one sequence on the oracle (prompt, then n_gen argmax tokens) and the
    logits of its last step."""
    okv = oracle.KV(ocfg, max_seq, fp16=fp16)
    toks = [int(prompt[0])]
    lo = None
    for p in range(len(prompt) + n_gen - 1):
        lo = oracle.forward_token(m, okv, toks[p], p)
        toks.append(int(prompt[p + 1]) if p + 1 < len(prompt) else oracle.sample_greedy(lo))
    okv.close()
    return np.array(toks, np.uint32), lo


def run_batch(cuda, eng, prompts, n_gen, max_seq, kv_dtype):
    b = cuda.Batch(eng, len(prompts), max_seq, kv_dtype)
    for s, p in enumerate(prompts):
        b.prefill(s, p)
    b.steps(n_gen)
    toks = [b.read_tokens(s, 0, len(p) + n_gen) for s, p in enumerate(prompts)]
    # the serving read-back: every sequence's newest token in one copy
    assert np.array_equal(b.read_current(), np.array([t[-1] for t in toks], np.uint32))
    logits = b.read_logits()
    b.close()
    return toks, logits


@pytest.mark.parametrize("kv_dtype", ["fp32", "fp16"])
def test_batch_gqa_ragged_vs_oracle(cuda, oracle, kv_dtype):
    """Six sequences with prompts of 1 to 100 tokens (ragged positions), GQA (2 query heads
    per KV head), 40 greedy steps each, against six independent oracle runs."""
    d = dict(vocab=1000, dim=256, hidden=512, layers=2, heads=4, kv_heads=2, head_dim=64, max_seq=160)
    cfg = cuda.model_config(*d.values())
    ocfg = oracle.make_config(*d.values())
    m = oracle.Model(ocfg, seed=21)
    eng = cuda.TransformerEngine(cfg)
    eng.load_pointers([(t.ptr, t.nbytes) for t in m.tensors()])
    rng = np.random.default_rng(22)
    prompts = [rng.integers(0, 1000, n).astype(np.uint32) for n in (5, 17, 33, 64, 100, 1)]
    n_gen = 40
    fp16 = kv_dtype == "fp16"
    toks, logits = run_batch(cuda, eng, prompts, n_gen, 160, cuda.BT_KV_FP16 if fp16 else cuda.BT_KV_FP32)
    for s, p in enumerate(prompts):
        want, lo = oracle_run(oracle, m, ocfg, p, n_gen, 160, fp16)
        got = toks[s]
        assert np.array_equal(got[: len(p)], p)
        first = len(p) + 32
        assert np.array_equal(got[:first], want[:first]), f"sequence {s}: first 32 generated tokens differ"
        assert rel_l2(logits[s], lo) <= TOL, f"sequence {s}: logits relative error {rel_l2(logits[s], lo)}"
    eng.close()
    m.close()


def test_batch_tiny_matches_golden_and_single(cuda, oracle):
    """The tiny config: sequence 0 is the golden prompt (the reference's greedy tokens),
    sequences 1-3 other prompts, each equal to the single-sequence engine's tokens."""
    import os
    from conftest import GOLDEN
    from blocktensor_b200 import synthetic
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    cfg = synthetic.config("tiny", 256)
    eng = cuda.TransformerEngine(cfg)
    eng.generate(seed=0, sigma=0.02)
    rng = np.random.default_rng(5)
    prompts = [g["prompt"]] + [rng.integers(0, 32000, n).astype(np.uint32) for n in (3, 40, 77)]
    n_gen = 64
    toks, _ = run_batch(cuda, eng, prompts, n_gen, 256, cuda.BT_KV_FP32)
    first = 16 + 32
    assert np.array_equal(toks[0][:first], g["tokens"][:first])
    for s in range(1, 4):
        kv = cuda.KVCache(eng, 256)
        single = eng.generate_tokens(kv, prompts[s], n_gen=n_gen)
        kv.close()
        n = len(prompts[s]) + 32
        assert np.array_equal(toks[s][:n], single[:n]), f"sequence {s}"
    eng.close()


def test_batch_tinyllama_width_two_layers(cuda, oracle):
    """The TinyLlama-1.1B width (D2048 F5632 H32 KVH4 hd64, vocab 32000) on two layers:
    four sequences at contexts 20-232 against the oracle."""
    d = dict(vocab=32000, dim=2048, hidden=5632, layers=2, heads=32, kv_heads=4, head_dim=64, max_seq=240)
    cfg = cuda.model_config(*d.values())
    ocfg = oracle.make_config(*d.values())
    m = oracle.Model(ocfg, seed=0)
    eng = cuda.TransformerEngine(cfg)
    eng.load_pointers([(t.ptr, t.nbytes) for t in m.tensors()])
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 32000, n).astype(np.uint32) for n in (20, 64, 130, 200)]
    n_gen = 32
    toks, logits = run_batch(cuda, eng, prompts, n_gen, 240, cuda.BT_KV_FP16)
    for s, p in enumerate(prompts):
        want, lo = oracle_run(oracle, m, ocfg, p, n_gen, 240, True)
        assert np.array_equal(toks[s], want[: len(toks[s])]), f"sequence {s}"
        assert rel_l2(logits[s], lo) <= TOL
    eng.close()
    m.close()


@pytest.mark.parametrize("kv_dtype", ["fp16", "fp32"])
def test_batch_gqa_head_dim_128(cuda, oracle, kv_dtype):
    """Eight query heads per KV head with head_dim 128 (the 70B shape's grouping): three
    sequences with contexts up to ~270, so their keys span several attention splits, against
    the oracle (fp16 caches on f16 tensor-core MMAs, fp32 caches on tf32)."""
    d = dict(vocab=1000, dim=1024, hidden=2048, layers=2, heads=8, kv_heads=1, head_dim=128, max_seq=300)
    cfg = cuda.model_config(*d.values())
    ocfg = oracle.make_config(*d.values())
    m = oracle.Model(ocfg, seed=17)
    eng = cuda.TransformerEngine(cfg)
    eng.load_pointers([(t.ptr, t.nbytes) for t in m.tensors()])
    rng = np.random.default_rng(18)
    prompts = [rng.integers(0, 1000, n).astype(np.uint32) for n in (3, 131, 240)]
    n_gen = 32
    fp16 = kv_dtype == "fp16"
    toks, logits = run_batch(cuda, eng, prompts, n_gen, 300, cuda.BT_KV_FP16 if fp16 else cuda.BT_KV_FP32)
    for s, p in enumerate(prompts):
        want, lo = oracle_run(oracle, m, ocfg, p, n_gen, 300, fp16)
        assert np.array_equal(toks[s], want[: len(toks[s])]), f"sequence {s}"
        assert rel_l2(logits[s], lo) <= TOL, f"sequence {s}: logits relative error {rel_l2(logits[s], lo)}"
    eng.close()
    m.close()


def test_batch_errors(cuda):
    d = dict(vocab=64, dim=64, hidden=128, layers=1, heads=2, kv_heads=2, head_dim=32, max_seq=16)
    eng = cuda.TransformerEngine(cuda.model_config(*d.values()))
    eng.generate(seed=1)
    b = cuda.Batch(eng, 2, 16)
    b.prefill(0, [1, 2, 3])
    with pytest.raises(IndexError):
        b.steps(1)                      # sequence 1 was never started
    b.prefill(1, [4])
    with pytest.raises(IndexError):
        b.prefill(2, [1])               # no sequence 2
    with pytest.raises(IndexError):
        b.steps(15)                     # sequence 0 would pass max_seq
    b.steps(13)
    assert len(b.read_tokens(0, 0, 16)) == 16
    b.close()
    eng.close()
