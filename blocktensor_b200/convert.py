"""Safetensors checkpoints (the Hugging Face Llama layout) to .btmodel v2.

    python -m blocktensor_b200.convert --input <dir with config.json and *.safetensors> \
        --output model.btmodel [--kv fp16|fp32]

The reference's converter (tools/convert_to_btmodel.py:66-101) stops after
parsing the safetensors header, and its quantizer rounds half to even in double
precision, which is not the engine's arithmetic.  This one writes every tensor:
embeddings and norms as fp32, projection matrices as 36-byte Q8_0 blocks
quantized exactly as quantization::quantize_q8_0 (quant_types.cpp:8-34): per
block of 32, amax = max |x| (NaN ignored, as std::max), scale = amax / 127 and
inv = 1 / scale in fp32 (0 for a zero block), q = (int) std::round(x * inv)
rounding half away from zero, clamped to [-128, 127]; a product that is not a
finite int converts to INT_MIN on x86, so it clamps to -128, as the reference
binary does.  The RoPE base and the KV-cache type, which v1 cannot record,
go into the v2 header.

Tensor names: model.embed_tokens.weight, model.norm.weight, lm_head.weight
(the embedding when tied), model.layers.{i}.input_layernorm.weight,
post_attention_layernorm.weight, self_attn.{q,k,v,o}_proj.weight,
mlp.{gate,up,down}_proj.weight.  The q/k rows stay in the checkpoint's order:
its rotary convention pairs dims (i, i + hd/2), which is cpu_ref::rope's
(kernels/cpu_ref.hpp:30-53).
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import struct

import numpy as np

from .btmodel import DT_INT8, write_btmodel_v2
from .native import ModelConfig

Q8_DTYPE = np.dtype([("scale", "<f4"), ("qs", "i1", (32,))])


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """quantization::quantize_q8_0 bit for bit; x fp32 with len % 32 == 0."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if x.size % 32:
        raise ValueError("quantize_q8_0: num_elements must be a multiple of block size")
    b = x.reshape(-1, 32)
    with np.errstate(all="ignore"):
        amax = np.fmax.reduce(np.abs(b), axis=1, initial=np.float32(0.0)).astype(np.float32)
        scale = (amax / np.float32(127.0)).astype(np.float32)
        inv = np.where(scale != 0, np.float32(1.0) / np.where(scale != 0, scale, np.float32(1.0)), np.float32(0.0))
        v = (b * inv.astype(np.float32)[:, None]).astype(np.float32).astype(np.float64)
        r = np.sign(v) * np.floor(np.abs(v) + 0.5)
        bad = ~np.isfinite(r) | (np.abs(r) > 2147483647.0)
        q = np.where(bad, -128.0, np.clip(r, -128.0, 127.0)).astype(np.int8)
    out = np.zeros(b.shape[0], Q8_DTYPE)
    out["scale"] = scale
    out["qs"] = q
    return out


# ---------------------------------------------------------------- safetensors

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": "bf16", "F64": np.float64}


def read_safetensors(path: str) -> dict:
    """name -> fp32 numpy array (F32, F16, BF16 and F64 tensors)."""
    out = {}
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n).decode())
        base = 8 + n
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            dt = _ST_DTYPES.get(meta["dtype"])
            if dt is None:
                raise ValueError(f"{path}: tensor {name} has unsupported dtype {meta['dtype']}")
            s, e = meta["data_offsets"]
            f.seek(base + s)
            raw = f.read(e - s)
            if dt == "bf16":
                a = (np.frombuffer(raw, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
            else:
                a = np.frombuffer(raw, dtype=dt).astype(np.float32)
            out[name] = a.reshape(meta["shape"])
    return out


def write_safetensors(path: str, tensors: dict) -> None:
    """fp32 tensors to a safetensors file (for tests and tools)."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, dtype=np.float32)
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# ---------------------------------------------------------------- conversion

def convert(src: str, out_path: str, kv_dtype: str = "fp16", max_seq: int | None = None) -> ModelConfig:
    """src: a directory with config.json and *.safetensors (or one .safetensors file with
    config.json beside it).  Returns the model's config."""
    d = src if os.path.isdir(src) else os.path.dirname(os.path.abspath(src))
    files = sorted(glob.glob(os.path.join(d, "*.safetensors"))) if os.path.isdir(src) else [src]
    with open(os.path.join(d, "config.json")) as f:
        hc = json.load(f)
    W = {}
    for p in files:
        W.update(read_safetensors(p))
    D, F, L = hc["hidden_size"], hc["intermediate_size"], hc["num_hidden_layers"]
    H = hc["num_attention_heads"]
    KVH = hc.get("num_key_value_heads", H)
    hd = hc.get("head_dim", D // H)
    V = hc["vocab_size"]
    cfg = ModelConfig(V, D, F, L, H, KVH, hd, int(max_seq or hc.get("max_position_embeddings", 2048)),
                      float(hc.get("rms_norm_eps", 1e-5)))
    theta = float(hc.get("rope_theta", 10000.0))

    def get(name):
        if name not in W:
            raise KeyError(f"checkpoint has no tensor {name}")
        return W[name]

    embed = get("model.embed_tokens.weight")
    head = W.get("lm_head.weight", embed)
    tensors = [embed.astype(np.float32), get("model.norm.weight").astype(np.float32), quantize_q8_0(head)]
    dims = [(V, D), (D,), (V, D)]
    for l in range(L):
        p = f"model.layers.{l}."
        tensors += [get(p + "input_layernorm.weight"), get(p + "post_attention_layernorm.weight")]
        dims += [(D,), (D,)]
        for n, shape in (("self_attn.q_proj", (H * hd, D)), ("self_attn.k_proj", (KVH * hd, D)),
                         ("self_attn.v_proj", (KVH * hd, D)), ("self_attn.o_proj", (D, H * hd)),
                         ("mlp.gate_proj", (F, D)), ("mlp.up_proj", (F, D)), ("mlp.down_proj", (D, F))):
            w = get(p + n + ".weight")
            if tuple(w.shape) != shape:
                raise ValueError(f"{p + n}: shape {w.shape}, expected {shape}")
            tensors.append(quantize_q8_0(w))
            dims.append(shape)
    write_btmodel_v2(out_path, cfg, [np.asarray(t) for t in tensors], dims, rope_theta=theta,
                     kv_dtype=1 if kv_dtype == "fp16" else 0, quant_type=DT_INT8)
    return cfg


def main():
    ap = argparse.ArgumentParser(description="safetensors (Llama layout) -> .btmodel v2 with Q8_0 matrices")
    ap.add_argument("--input", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--kv", choices=["fp16", "fp32"], default="fp16")
    ap.add_argument("--max-seq", type=int, default=None)
    a = ap.parse_args()
    cfg = convert(a.input, a.output, a.kv, a.max_seq)
    print(f"wrote {a.output}: {cfg}")


if __name__ == "__main__":
    main()
