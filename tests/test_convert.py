"""CPU: the checkpoint converter and the .btmodel v2 format.

The quantizer must be quantization::quantize_q8_0 bit for bit (the reference's
own outputs in tests/golden/ref_kernels.npz, edge cases included); a converted
checkpoint must read back with its config, RoPE base, KV type, names and shapes,
every matrix equal to the quantizer's blocks, and load into the reference's own
engine through a v1 copy.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

from blocktensor_b200 import btmodel, convert


@pytest.mark.parametrize("name", ["qn", "qu", "qedge", "mv"])
def test_quantizer_matches_reference_goldens(name):
    g = np.load(os.path.join(GOLDEN, "ref_kernels.npz"))
    x = g["mv_raw"] if name == "mv" else g[f"{name}_x"]
    want = g["mv_blocks"] if name == "mv" else g[f"{name}_blocks"]
    got = convert.quantize_q8_0(x).view(np.uint8).reshape(-1)
    assert np.array_equal(got, want.reshape(-1))


def test_quantizer_matches_oracle(oracle):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(32 * 4099) * rng.choice([1e-3, 1.0, 1e3], 32 * 4099)).astype(np.float32)
    x[::977] = 0.0
    assert np.array_equal(convert.quantize_q8_0(x).view(np.uint8), oracle.quantize_q8_0(x).view(np.uint8))
    with pytest.raises(ValueError):
        convert.quantize_q8_0(np.zeros(33, np.float32))


def _checkpoint(tmp_path, tied=False, theta=500000.0):
    D, F, L, H, KVH, V = 64, 96, 2, 4, 2, 100
    hd = D // H
    rng = np.random.default_rng(1)
    t = {"model.embed_tokens.weight": rng.standard_normal((V, D)) * 0.02,
         "model.norm.weight": 1.0 + rng.standard_normal(D) * 0.01}
    if not tied:
        t["lm_head.weight"] = rng.standard_normal((V, D)) * 0.02
    for l in range(L):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = 1.0 + rng.standard_normal(D) * 0.01
        t[p + "post_attention_layernorm.weight"] = 1.0 + rng.standard_normal(D) * 0.01
        t[p + "self_attn.q_proj.weight"] = rng.standard_normal((H * hd, D)) * 0.02
        t[p + "self_attn.k_proj.weight"] = rng.standard_normal((KVH * hd, D)) * 0.02
        t[p + "self_attn.v_proj.weight"] = rng.standard_normal((KVH * hd, D)) * 0.02
        t[p + "self_attn.o_proj.weight"] = rng.standard_normal((D, H * hd)) * 0.02
        t[p + "mlp.gate_proj.weight"] = rng.standard_normal((F, D)) * 0.02
        t[p + "mlp.up_proj.weight"] = rng.standard_normal((F, D)) * 0.02
        t[p + "mlp.down_proj.weight"] = rng.standard_normal((D, F)) * 0.02
    t = {k: v.astype(np.float32) for k, v in t.items()}
    d = tmp_path / "ckpt"
    d.mkdir()
    convert.write_safetensors(str(d / "model.safetensors"), t)
    with open(d / "config.json", "w") as f:
        json.dump({"hidden_size": D, "intermediate_size": F, "num_hidden_layers": L, "num_attention_heads": H,
                   "num_key_value_heads": KVH, "vocab_size": V, "rms_norm_eps": 1e-5, "rope_theta": theta,
                   "max_position_embeddings": 64}, f)
    return str(d), t


@pytest.mark.parametrize("tied", [False, True])
def test_convert_roundtrip(tmp_path, tied):
    src, t = _checkpoint(tmp_path, tied=tied)
    out = str(tmp_path / "m.btmodel")
    cfg = convert.convert(src, out, kv_dtype="fp16")
    m = btmodel.read_btmodel_any(out)
    assert isinstance(m, btmodel.BtModelV2)
    assert bytes(m.config) == bytes(cfg)
    assert (cfg.dim, cfg.hidden_dim, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim) == (64, 96, 2, 4, 2, 16)
    assert m.rope_theta == 500000.0 and m.kv_dtype == 1 and m.quant_type == btmodel.DT_INT8
    assert m.names[:3] == ["embed_tokens", "output_norm", "output_head"] and m.names[3] == "layers.0.attn_norm"
    assert tuple(m.dims[5]) == (64, 64) and tuple(m.dims[6]) == (32, 64)
    assert np.array_equal(m.tensors[0].view(np.float32), t["model.embed_tokens.weight"].reshape(-1))
    head = t["model.embed_tokens.weight"] if tied else t["lm_head.weight"]
    assert np.array_equal(m.tensors[2], convert.quantize_q8_0(head).view(np.uint8))
    for l in range(2):
        p = f"model.layers.{l}."
        base = 3 + 9 * l
        assert np.array_equal(m.tensors[base].view(np.float32), t[p + "input_layernorm.weight"])
        for j, n in enumerate(("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")):
            assert np.array_equal(m.tensors[base + 2 + j], convert.quantize_q8_0(t[p + n + ".weight"]).view(np.uint8))
    # v2 tensors are 64-byte aligned in the file
    assert all((t.ctypes.data - m.tensors[0].ctypes.data) % 64 == 0 for t in m.tensors)


def test_v2_rejects_bad_files(tmp_path):
    src, _ = _checkpoint(tmp_path)
    out = tmp_path / "m.btmodel"
    convert.convert(src, str(out))
    data = out.read_bytes()
    (tmp_path / "bad.btmodel").write_bytes(b"XXXX" + data[4:])
    with pytest.raises(RuntimeError):
        btmodel.read_btmodel_any(str(tmp_path / "bad.btmodel"))
    (tmp_path / "short.btmodel").write_bytes(data[: len(data) // 2])
    with pytest.raises(RuntimeError):
        btmodel.read_btmodel_v2(str(tmp_path / "short.btmodel"))


def test_converted_model_runs_in_reference_engine(tmp_path, ref, oracle):
    """The converted tensors, written in the reference's v1 layout, load into the
    reference's own importer and TransformerEngine (RoPE base 10000 there)."""
    src, _ = _checkpoint(tmp_path, theta=10000.0)
    out = str(tmp_path / "m.btmodel")
    convert.convert(src, out)
    m = btmodel.read_btmodel_v2(out)
    v1 = str(tmp_path / "m1.btmodel")
    btmodel.write_btmodel(v1, m.config, m.tensors)
    eng = oracle.RefEngine.from_file(ref, v1, kv_max_seq=16)
    lg = eng.forward(3, 0)
    assert lg.shape == (100,) and np.isfinite(lg).all()
    eng.close()
