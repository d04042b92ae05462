"""GPU parity of the decode engine (through the C ABI) against the oracle.

Bars (the north-star criteria): per-layer residual activations within 1e-2
relative error (elementwise |gpu - ref| <= 1e-2 * (1 + |ref|), and the
relative L2 error <= 1e-2); greedy tokens identical for the first 32
generated tokens; quantized weights bit-exact (device-generated == host
quantized).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = 1e-2


def assert_close_act(gpu, ref, what=""):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(gpu - ref) > TOL * (1.0 + np.abs(ref))
    assert not bad.any(), f"{what}: {bad.sum()} elements outside 1e-2, worst {np.abs(gpu - ref).max()}"
    rel = np.linalg.norm(gpu - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= TOL, f"{what}: relative L2 error {rel}"


TINY = dict(vocab=32000, dim=288, hidden=768, layers=6, heads=6, kv_heads=6, head_dim=48, max_seq=256)


def configs(bt, oracle, d):
    args = (d["vocab"], d["dim"], d["hidden"], d["layers"], d["heads"], d["kv_heads"], d["head_dim"], d["max_seq"])
    return bt.model_config(*args), oracle.make_config(*args)


@pytest.fixture(scope="module")
def tiny(cuda, oracle):
    cfg, ocfg = configs(cuda, oracle, TINY)
    m = oracle.Model(ocfg, seed=0)
    eng = cuda.TransformerEngine(cfg)
    eng.generate(seed=0, sigma=0.02)
    yield cfg, ocfg, m, eng
    eng.close()
    m.close()


def test_device_generator_matches_oracle_weights(cuda, oracle, tiny):
    """Weights generated+quantized on the device == oracle weights loaded from the host (bit-exact logits)."""
    cfg, ocfg, m, eng = tiny
    eng2 = cuda.TransformerEngine(cfg)
    eng2.load_pointers([(t.ptr, t.nbytes) for t in m.tensors()])
    kv1 = cuda.KVCache(eng, 32)
    kv2 = cuda.KVCache(eng2, 32)
    for p, tok in enumerate([5, 77, 31999, 0]):
        a = eng.forward_single_token(tok, p, kv1)
        b = eng2.forward_single_token(tok, p, kv2)
        assert np.array_equal(a, b), p
    eng2.close()


def test_tiny_layers_and_logits_vs_oracle(cuda, oracle, tiny):
    cfg, ocfg, m, eng = tiny
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    toks = g["tokens"]
    kv = cuda.KVCache(eng, 256)
    okv = oracle.KV(ocfg, 256)
    eng.set_taps(True)
    try:
        for p in range(48):
            lg = eng.forward_single_token(int(toks[p]), p, kv)
            taps = eng.read_taps()
            lo, otaps = oracle.forward_token(m, okv, int(toks[p]), p, want_taps=True)
            for l in range(cfg.num_layers):
                assert_close_act(taps[l], otaps[l], f"pos {p} layer {l}")
            assert_close_act(lg, lo, f"logits pos {p}")
            assert eng.last_argmax == int(np.argmax(lg))
    finally:
        eng.set_taps(False)
    # KV cache contents in the reference layout
    k, v = kv.read_layer(0)
    ok, ov = okv.layer(0)
    n = 48 * cfg.num_kv_heads * cfg.head_dim
    assert_close_act(k[:n], ok[:n], "K cache layer 0")
    assert_close_act(v[:n], ov[:n], "V cache layer 0")


@pytest.mark.parametrize("kv_dtype", ["fp32", "fp16"])
def test_tiny_greedy_tokens(cuda, tiny, kv_dtype):
    """16 prompt ids + 128 greedy steps on the device == the reference's greedy tokens."""
    cfg, ocfg, m, eng = tiny
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    want = g["tokens"] if kv_dtype == "fp32" else g["tokens_kv16"]
    kv = cuda.KVCache(eng, 256, cuda.BT_KV_FP32 if kv_dtype == "fp32" else cuda.BT_KV_FP16)
    got = eng.decode(kv, g["prompt"], n_gen=128)
    assert len(got) == 16 + 128 + 1
    first = 16 + 32
    assert np.array_equal(got[:first], want[:first]), "first 32 generated tokens differ"
    diverged = np.nonzero(got[: len(want)] != want[: len(got)])[0]
    assert diverged.size == 0, f"greedy tokens diverge at positions {diverged[:5]} (margins {g['margins'][diverged[:5] - 1]})"


def test_tiny_forward_matches_decode_path(cuda, tiny):
    cfg, ocfg, m, eng = tiny
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    kv = cuda.KVCache(eng, 64)
    toks = [int(g["prompt"][0])]
    for p in range(24):
        eng.forward_single_token(toks[p], p, kv, want_logits=False)
        toks.append(int(g["prompt"][p + 1]) if p + 1 < 16 else eng.last_argmax)
    kv2 = cuda.KVCache(eng, 64)
    got = eng.decode(kv2, g["prompt"], n_gen=8)
    assert list(got) == toks[:25]


def test_engine_errors(cuda, tiny):
    cfg, ocfg, m, eng = tiny
    kv = cuda.KVCache(eng, 8)
    with pytest.raises(IndexError):                 # token >= vocab (transformer_engine.cpp:229-231)
        eng.forward_single_token(cfg.vocab_size, 0, kv)
    with pytest.raises(IndexError):                 # pos >= max_seq (kv_cache.cpp:18-19)
        eng.forward_single_token(1, 8, kv)
    eng.forward_single_token(1, 7, kv)              # last slot is fine
    with pytest.raises(IndexError):
        eng.decode(kv, [1, 2, 3], n_gen=6)          # 9 positions > 8
    with pytest.raises(ValueError):
        cuda.KVCache(eng, 0)
    bad = cuda.model_config(100, 100, 128, 1, 4, 4, 25, 16)   # dim not a multiple of 32
    with pytest.raises(ValueError):
        cuda.TransformerEngine(bad)


def test_kv_outliving_engine(cuda):
    """Destroying the engine first detaches its caches; using one then fails cleanly."""
    d = dict(vocab=64, dim=64, hidden=128, layers=1, heads=2, kv_heads=2, head_dim=32, max_seq=8)
    cfg = cuda.model_config(*d.values())
    eng = cuda.TransformerEngine(cfg)
    eng.generate(seed=1)
    kv = cuda.KVCache(eng, 8)
    eng.forward_single_token(3, 0, kv)
    eng.close()
    with pytest.raises(ValueError):
        kv.read_layer(0)
    kv.close()


def test_btmodel_file_drives_engine(cuda, oracle, tmp_path):
    """A .btmodel file (reference format) loaded into the CUDA engine matches the reference engine."""
    from blocktensor_b200 import btmodel
    d = dict(vocab=1000, dim=256, hidden=512, layers=4, heads=4, kv_heads=4, head_dim=64, max_seq=128)
    cfg, ocfg = configs(cuda, oracle, d)
    m = oracle.Model(ocfg, seed=11)
    path = str(tmp_path / "bench.btmodel")
    btmodel.write_btmodel(path, ocfg, [m.tensor_array(t).view(np.uint8) for t in m.tensors()])
    bm = btmodel.read_btmodel(path)
    eng = cuda.TransformerEngine(bm.config)
    eng.load(bm.tensors)
    kv = cuda.KVCache(eng, 128)
    if oracle.ref_available():
        ref = oracle.RefEngine.from_file(oracle.RefLib(), path, kv_max_seq=128)
        step = lambda t, p: ref.forward(t, p)
    else:
        okv = oracle.KV(ocfg, 128)
        step = lambda t, p: oracle.forward_token(m, okv, t, p)
    tok = 7
    for p in range(20):
        a = eng.forward_single_token(tok, p, kv)
        b = step(tok, p)
        assert_close_act(a, b, f"pos {p}")
        assert int(np.argmax(a)) == int(np.argmax(b))
        tok = int(np.argmax(b))


@pytest.mark.parametrize("kv_fp16", [False, True])
def test_gqa_theta_vs_oracle(cuda, oracle, kv_fp16):
    """GQA (8 query heads per KV head, as the 70B shape) with RoPE base 500000 and hd 128."""
    d = dict(vocab=2048, dim=1024, hidden=2816, layers=2, heads=8, kv_heads=1, head_dim=128, max_seq=300)
    cfg, ocfg = configs(cuda, oracle, d)
    m = oracle.Model(ocfg, seed=21)
    eng = cuda.TransformerEngine(cfg, rope_theta=500000.0)
    eng.generate(seed=21, sigma=0.02)
    kv = cuda.KVCache(eng, 300, cuda.BT_KV_FP16 if kv_fp16 else cuda.BT_KV_FP32)
    assert kv.step_info(1)[0] == 1, "the persistent step kernel (query heads in groups of 16 / NV) runs this shape"
    okv = oracle.KV(ocfg, 300, fp16=kv_fp16)
    eng.set_taps(True)
    tok = 3
    for p in range(260):
        lg = eng.forward_single_token(tok, p, kv)
        if p % 37 == 0 or p == 259:
            lo, otaps = oracle.forward_token(m, okv, tok, p, theta=500000.0, want_taps=True)
            taps = eng.read_taps()
            for l in range(cfg.num_layers):
                assert_close_act(taps[l], otaps[l], f"pos {p} layer {l}")
            assert_close_act(lg, lo, f"logits pos {p}")
        else:
            oracle.forward_token(m, okv, tok, p, theta=500000.0)
        tok = int(np.argmax(lg)) % 2048


def test_tinyllama_shape_gqa(cuda, oracle):
    """TinyLlama head layout (32 query / 4 KV heads, hd 64), 2 layers, fp16 KV."""
    d = dict(vocab=1024, dim=2048, hidden=5632, layers=2, heads=32, kv_heads=4, head_dim=64, max_seq=600)
    cfg, ocfg = configs(cuda, oracle, d)
    m = oracle.Model(ocfg, seed=4)
    eng = cuda.TransformerEngine(cfg)
    eng.generate(seed=4, sigma=0.02)
    kv = cuda.KVCache(eng, 600, cuda.BT_KV_FP16)
    okv = oracle.KV(ocfg, 600, fp16=True)
    tok = 9
    for p in range(530):
        lg = eng.forward_single_token(tok, p, kv, want_logits=(p % 131 == 0 or p == 529))
        lo = oracle.forward_token(m, okv, tok, p)
        if lg is not None:
            assert_close_act(lg, lo, f"logits pos {p}")
        tok = int(np.argmax(lo))


def test_device_wait_expiry_reports_timeout(cuda, tiny):
    """Failure detection without a GPU fault: the host makes the phase barriers
    of the next step unreachable (bt_kv_inject_stall), the step's bounded
    device waits expire after 2 s, the kernel finishes, and the host reads
    BT_ERR_DEVICE_TIMEOUT.  The context stays usable: a fresh sequence on the
    same engine then decodes the same tokens as before the injection."""
    import time
    from blocktensor_b200 import native

    cfg, ocfg, m, eng = tiny
    g = np.load(os.path.join(GOLDEN, "tiny_c0.npz"))
    prompt = [int(t) for t in g["prompt"]]
    kv = cuda.KVCache(eng, 64)
    clean = eng.decode(kv, prompt, n_gen=8)

    eng.begin(kv, prompt)
    kv.inject_stall()
    t0 = time.time()
    eng.steps(kv, 1)
    with pytest.raises(native.CudaBackendError) as ei:
        kv.state()
    assert ei.value.code == native.BT_ERR_DEVICE_TIMEOUT
    assert 1.5 < time.time() - t0 < 30.0, "the expiry should come from the 2 s device wait limit"

    again = eng.decode(kv, prompt, n_gen=8)  # begin() resets the state and its error flag
    assert list(again) == list(clean)
    kv.state()


def test_btmodel_v2_from_converter_drives_engine(cuda, oracle, ref, tmp_path):
    """A safetensors checkpoint converted to .btmodel v2 loads into the CUDA engine and
    matches the reference engine on the same tensors (its v1 copy)."""
    import json
    from blocktensor_b200 import btmodel, convert
    D, F, L, H, KVH, V = 128, 256, 2, 4, 2, 512
    rng = np.random.default_rng(3)
    t = {"model.embed_tokens.weight": rng.standard_normal((V, D)) * 0.02, "model.norm.weight": np.ones(D)}
    for l in range(L):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = np.ones(D)
        t[p + "post_attention_layernorm.weight"] = np.ones(D)
        for n, shape in (("self_attn.q_proj", (D, D)), ("self_attn.k_proj", (KVH * 32, D)),
                         ("self_attn.v_proj", (KVH * 32, D)), ("self_attn.o_proj", (D, D)),
                         ("mlp.gate_proj", (F, D)), ("mlp.up_proj", (F, D)), ("mlp.down_proj", (D, F))):
            t[p + n + ".weight"] = rng.standard_normal(shape) * 0.05
    d = tmp_path / "ckpt"
    d.mkdir()
    convert.write_safetensors(str(d / "model.safetensors"), t)
    json.dump({"hidden_size": D, "intermediate_size": F, "num_hidden_layers": L, "num_attention_heads": H,
               "num_key_value_heads": KVH, "vocab_size": V, "rope_theta": 10000.0,
               "max_position_embeddings": 64}, open(d / "config.json", "w"))
    out = str(tmp_path / "m.btmodel")
    convert.convert(str(d), out, kv_dtype="fp32")
    eng = cuda.TransformerEngine.from_btmodel(out)
    m = btmodel.read_btmodel_v2(out)
    v1 = str(tmp_path / "m1.btmodel")
    btmodel.write_btmodel(v1, m.config, m.tensors)
    r = oracle.RefEngine.from_file(ref, v1, kv_max_seq=64)
    kv = cuda.KVCache(eng, 64)
    tok = 7
    for p in range(24):
        a = eng.forward_single_token(tok, p, kv)
        b = r.forward(tok, p)
        assert_close_act(a, b, f"pos {p}")
        assert int(np.argmax(a)) == int(np.argmax(b))
        tok = int(np.argmax(b))
    r.close()
    kv.close()
    eng.close()
