"""CPU: pin the oracle restatement (oracle/bt_oracle.c).

Two anchors:
* the committed golden vectors (tests/golden/*.npz, made by
  tests/golden/make_golden.py from the reference's own sources) -- always run;
* the reference library itself (oracle/_ref/libbtref.so) -- run where it was
  built, bit-for-bit.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN


@pytest.fixture(scope="module")
def gk():
    return np.load(os.path.join(GOLDEN, "ref_kernels.npz"))


def test_known_answer_q8_error(oracle, gk):
    """calc_numerical_errors.cpp:27-44: Q8_0 matvec vs fp32, max 1.710196e-01 mean 6.168072e-02."""
    raw, x = gk["mv_raw"], gk["mv_x"]
    blocks = oracle.quantize_q8_0(raw)
    assert np.array_equal(blocks.view(np.uint8), gk["mv_blocks"])
    yq = oracle.matvec_q8_0(blocks, x, 16, 256)
    assert np.array_equal(yq, gk["mv_y"])
    yf = np.zeros(16, np.float32)
    for r in range(16):
        acc = np.float32(0.0)
        for c in range(256):
            acc = np.float32(acc + np.float32(raw[r * 256 + c] * x[c]))
        yf[r] = acc
    err = np.abs(yf - yq)
    assert f"{err.max():.6e}" == "1.710196e-01"
    assert f"{err.sum(dtype=np.float32) / np.float32(16):.6e}" == "6.168072e-02"


@pytest.mark.parametrize("name", ["qn", "qu", "qedge"])
def test_quantizer_golden_bit_exact(oracle, gk, name):
    x = gk[f"{name}_x"]
    b = oracle.quantize_q8_0(x)
    assert np.array_equal(b.view(np.uint8), gk[f"{name}_blocks"])
    assert np.array_equal(oracle.dequantize_q8_0(b).view(np.uint32), gk[f"{name}_deq"].view(np.uint32))


def test_quantize_rejects_ragged(oracle):
    with pytest.raises(ValueError):
        oracle.quantize_q8_0(np.zeros(33, np.float32))


def test_zero_block(oracle, gk):
    """test_stage7_edge_cases.cpp:20-28: zeros -> scale 0, dequant 0."""
    b = oracle.quantize_q8_0(np.zeros(32, np.float32))
    assert b["scale"][0] == 0.0 == gk["zero_scale"]
    assert (oracle.dequantize_q8_0(b) == 0).all()


def test_kernels_golden(oracle, gk):
    rms = oracle.rmsnorm(gk["rms_x"], gk["rms_w"], 4, 512, 1e-5)
    assert np.array_equal(rms, gk["rms_y"])
    for pos in (0, 7, 300):
        assert np.array_equal(oracle.rope(gk["rope_x"], 2, 4, 64, pos), gk[f"rope_y_pos{pos}"])
    assert np.array_equal(oracle.softmax(gk["softmax_x"], 4, 256), gk["softmax_y"])
    assert np.array_equal(oracle.silu(gk["silu_x"]), gk["silu_y"])
    assert oracle.sample_greedy(gk["greedy_logits"]) == int(gk["greedy_id"]) == 3


def test_greedy_first_max_wins(oracle):
    assert oracle.sample_greedy(np.array([1.0, 5.0, 5.0, 2.0], np.float32)) == 1


def test_tiny_engine_golden(oracle):
    """Config 0 (D288 L6, seed 0): restated engine == reference engine logits (golden)."""
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    cfg = oracle.make_config(32000, 288, 768, 6, 6, 6, 48, 256)
    assert bytes(cfg) == g["config"].tobytes()
    m = oracle.Model(cfg, seed=0)
    prompt = oracle.gen_tokens(0, oracle.STREAM_PROMPT, 16, 32000)
    assert np.array_equal(prompt, g["prompt"])
    kv = oracle.KV(cfg, 256)
    toks = g["tokens"]
    keep = set(int(p) for p in g["keep_pos"])
    last = 48  # positions checked here (the golden holds 144)
    for p in range(last):
        lo, taps = oracle.forward_token(m, kv, int(toks[p]), p, want_taps=True)
        if p in keep:
            assert np.array_equal(lo, g[f"logits_p{p}"]), p
            assert np.array_equal(taps, g[f"taps_p{p}"]), p
        nxt = int(prompt[p + 1]) if p + 1 < 16 else oracle.sample_greedy(lo)
        assert nxt == int(toks[p + 1]), p


def test_generator_reproducible(oracle):
    a = oracle.gen_normal(7, 123, 1000, 0.02)
    b = oracle.gen_normal(7, 123, 600, 0.02, offset=400)
    assert np.array_equal(a[400:], b)
    assert abs(float(a.std()) - 0.02) < 0.002 and abs(float(a.mean())) < 0.002
    t = oracle.gen_tokens(0, oracle.STREAM_PROMPT, 1000, 32000)
    assert t.max() < 32000


# ---------------------------------------------------------------- against the reference library

def test_ref_quantize_bit_exact(oracle, ref):
    rng = np.random.default_rng(0)
    for scale in (1e-3, 0.02, 1.0, 300.0):
        x = (rng.standard_normal(32 * 997) * scale).astype(np.float32)
        assert np.array_equal(oracle.quantize_q8_0(x).view(np.uint8), ref.quantize_q8_0(x).view(np.uint8))


def test_ref_matvec_bit_exact(oracle, ref):
    rng = np.random.default_rng(1)
    M, N = 37, 32 * 9
    b = ref.quantize_q8_0((rng.standard_normal(M * N) * 0.02).astype(np.float32))
    x = rng.standard_normal(N).astype(np.float32)
    assert np.array_equal(oracle.matvec_q8_0(b, x, M, N), ref.matvec_q8_0(b, x, M, N))
    assert np.array_equal(oracle.matvec_q8_0(b, x, M, N, nthreads=4), ref.matvec_q8_0(b, x, M, N))


def test_ref_engine_bit_exact_gqa(oracle, ref):
    """A GQA shape (H8 KVH2 hd16): restatement == reference engine for 12 steps."""
    cfg = oracle.make_config(500, 128, 256, 2, 8, 2, 16, 32)
    m = oracle.Model(cfg, seed=5)
    eng = oracle.RefEngine(ref, m, kv_max_seq=32)
    kv = oracle.KV(cfg, 32)
    tok = 3
    for p in range(12):
        lr = eng.forward(tok, p)
        lo = oracle.forward_token(m, kv, tok, p)
        assert np.array_equal(lr, lo), p
        tok = oracle.sample_greedy(lo)


def test_ref_errors(ref):
    """Reference exception behaviour the CUDA path mirrors."""
    # KVCache overflow at pos == max_seq -> out_of_range (test_stage7_edge_cases.cpp:45-60)
    assert ref.btr_kv_update_probe(1, 4, 2, 8, 0, 3) == 0
    assert ref.btr_kv_update_probe(1, 4, 2, 8, 0, 4) == -2
    # ragged quantize -> invalid_argument
    with pytest.raises(ValueError):
        ref.quantize_q8_0(np.zeros(33, np.float32))


def test_ref_btmodel_roundtrip(oracle, ref, tmp_path):
    """.btmodel written by the reference exporter is read by our reader byte-for-byte."""
    from blocktensor_b200 import btmodel
    cfg = oracle.make_config(100, 64, 128, 2, 4, 4, 16, 32)
    m = oracle.Model(cfg, seed=3)
    eng = oracle.RefEngine(ref, m, kv_max_seq=32)
    path = str(tmp_path / "m.btmodel")
    eng.export(path)
    bm = btmodel.read_btmodel(path)
    assert bytes(bm.config) == bytes(cfg)
    assert bm.quant_type == btmodel.DT_INT8
    ts = m.tensors()
    assert len(bm.tensors) == len(ts)
    for a, t in zip(bm.tensors, ts):
        assert np.array_equal(a, m.tensor_array(t).view(np.uint8))
    assert [t.nbytes for t in bm.tensors] == bm.expected_sizes()
    # our writer produces a file the reference importer accepts
    path2 = str(tmp_path / "m2.btmodel")
    btmodel.write_btmodel(path2, bm.config, bm.tensors)
    eng2 = oracle.RefEngine.from_file(ref, path2, kv_max_seq=32)
    assert np.array_equal(eng2.forward(5, 0), eng.forward(5, 0))


def test_ref_bad_magic(ref, tmp_path):
    """Malformed file -> runtime_error (test_stage7_edge_cases.cpp:62-84)."""
    from blocktensor_b200 import btmodel
    bad = tmp_path / "corrupted.btmodel"
    bad.write_bytes((0xDEADBEEF).to_bytes(4, "little"))
    with pytest.raises(RuntimeError):
        btmodel.read_btmodel(str(bad))
    from oracle import oracle as O
    with pytest.raises(RuntimeError):
        O.RefEngine.from_file(ref, str(bad))
