"""GPU parity of paged KV (bt_batch_create_paged): the K/V of a batch's sequences
in one pool of fixed-size pages instead of one contiguous buffer per sequence.

The reference KV cache is one contiguous single-sequence buffer per layer
(runtime/src/kv_cache.cpp:6-15).  A paged cache changes only where the rows
live, so a paged batch must give exactly the results of the contiguous batch
(same arithmetic, same order: tokens and logits bit-identical), and through it
the oracle's single-sequence greedy tokens, also when pages freed by one
sequence are reused, in another order, by the next.
"""
import numpy as np
import pytest

from test_gpu_batch import TOL, oracle_run, rel_l2

pytestmark = pytest.mark.gpu

SHAPE = dict(vocab=1000, dim=256, hidden=512, layers=2, heads=4, kv_heads=2, head_dim=64, max_seq=192)


def _model(cuda, oracle, seed):
    cfg = cuda.model_config(*SHAPE.values())
    ocfg = oracle.make_config(*SHAPE.values())
    m = oracle.Model(ocfg, seed=seed)
    eng = cuda.TransformerEngine(cfg)
    eng.load_pointers([(t.ptr, t.nbytes) for t in m.tensors()])
    return eng, m, ocfg


def _run(cuda, eng, prompts, n_gen, kv_dtype, page_tokens=0, n_pages=0):
    b = cuda.Batch(eng, len(prompts), SHAPE["max_seq"], kv_dtype, page_tokens=page_tokens, n_pages=n_pages)
    for s, p in enumerate(prompts):
        b.prefill(s, p)
    b.steps(n_gen)
    toks = [b.read_tokens(s, 0, len(p) + n_gen) for s, p in enumerate(prompts)]
    logits = b.read_logits()
    return b, toks, logits


@pytest.mark.parametrize("page_tokens", [16, 64])
@pytest.mark.parametrize("kv_dtype", ["fp32", "fp16"])
def test_paged_equals_contiguous_and_oracle(cuda, oracle, page_tokens, kv_dtype):
    """Five ragged sequences (prompts of 1 to 120 tokens, 40 greedy steps): the paged batch's
    tokens and logits are bit-identical to the contiguous batch's, and every sequence's first
    32 generated tokens are the oracle's."""
    eng, m, ocfg = _model(cuda, oracle, seed=31)
    dt = cuda.BT_KV_FP16 if kv_dtype == "fp16" else cuda.BT_KV_FP32
    rng = np.random.default_rng(32)
    prompts = [rng.integers(0, 1000, n).astype(np.uint32) for n in (7, 120, 1, 45, 64)]
    n_gen = 40
    bc, want_toks, want_logits = _run(cuda, eng, prompts, n_gen, dt)
    bc.close()
    # a sequence writes positions 0 .. len + n_gen - 2
    pages = sum(-(-(len(p) + n_gen - 1) // page_tokens) for p in prompts)
    bp, toks, logits = _run(cuda, eng, prompts, n_gen, dt, page_tokens, pages)
    assert bp.pages() == (0, pages)  # exactly the pages the sequences' positions need
    for s in range(len(prompts)):
        assert np.array_equal(toks[s], want_toks[s]), f"sequence {s}: paged tokens differ from contiguous"
    assert np.array_equal(logits, want_logits), "paged logits differ from contiguous"
    for s, p in enumerate(prompts):
        want, lo = oracle_run(oracle, m, ocfg, p, n_gen, SHAPE["max_seq"], kv_dtype == "fp16")
        first = len(p) + 32
        assert np.array_equal(toks[s][:first], want[:first]), f"sequence {s}: first 32 generated tokens differ"
        assert rel_l2(logits[s], lo) <= TOL
    bp.close()
    eng.close()
    m.close()


def test_pages_reused_by_the_next_sequence(cuda, oracle):
    """A pool too small for every sequence at once: two sequences run, one is released and a
    third starts in its slot on the freed pages (taken back in another order, interleaved
    with the survivor's new pages).  Every sequence decodes the oracle's tokens."""
    eng, m, ocfg = _model(cuda, oracle, seed=41)
    P = 16
    rng = np.random.default_rng(42)
    pa, pb, pc = (rng.integers(0, 1000, n).astype(np.uint32) for n in (50, 30, 70))
    b = cuda.Batch(eng, 2, SHAPE["max_seq"], cuda.BT_KV_FP16, page_tokens=P, n_pages=12)
    b.prefill(0, pa)
    b.prefill(1, pb)
    b.steps(20)  # a: positions to 69 (5 pages), b: to 49 (4 pages)
    assert b.pages() == (3, 12)
    ta = b.read_tokens(0, 0, len(pa) + 20)
    b.release(0)
    assert b.pages() == (8, 12)
    b.prefill(0, pc)  # c takes a's freed pages (5 of them)
    b.steps(26)  # c: to 95 (6 pages), b: to 75 (5 pages): 11 of 12
    assert b.pages() == (1, 12)
    tb = b.read_tokens(1, 0, len(pb) + 46)
    tc = b.read_tokens(0, 0, len(pc) + 26)
    for p, got, n in ((pa, ta, 20), (pb, tb, 46), (pc, tc, 26)):
        want, _ = oracle_run(oracle, m, ocfg, p, n, SHAPE["max_seq"], True)
        assert np.array_equal(got, want[: len(p) + n])
    b.steps(1)  # positions 95 (c) and 75 (b) are on pages they hold: nothing taken
    free, _ = b.pages()
    assert free == 1
    # 40 more steps need 6 new pages and 1 is free: refused, and nothing is taken
    with pytest.raises(MemoryError):
        b.steps(40)
    assert b.pages()[0] == free
    b.release(0)
    b.release(1)
    assert b.pages() == (12, 12)
    b.close()
    eng.close()
    m.close()


def test_paged_arguments(cuda, oracle):
    eng, m, _ = _model(cuda, oracle, seed=5)
    with pytest.raises(ValueError):
        cuda.Batch(eng, 2, 64, cuda.BT_KV_FP16, page_tokens=24, n_pages=4)  # not a power of two
    with pytest.raises(ValueError):
        cuda.Batch(eng, 2, 64, cuda.BT_KV_FP16, page_tokens=16, n_pages=0)
    b = cuda.Batch(eng, 2, 64, cuda.BT_KV_FP16, page_tokens=16, n_pages=2)
    with pytest.raises(MemoryError):
        b.prefill(0, np.arange(40, dtype=np.uint32))  # 3 pages needed, 2 in the pool
    assert b.pages() == (2, 2)
    c = cuda.Batch(eng, 1, 64, cuda.BT_KV_FP16)
    with pytest.raises(ValueError):
        c.release(0)  # no page pool
    c.close()
    b.close()
    eng.close()
    m.close()
