""".btmodel v1 reader/writer (the format of models/model_importer.cpp:10-88).

Layout: u32 magic 0x42544d44, the raw 36-byte ModelConfig, u32 quant type
(blocktensor::DataType, INT8 = 3), then per tensor ``u64 size`` + ``size`` bytes
in the order embed, out_norm, head, then for each layer attn_norm, ffn_norm,
q, k, v, o, gate, up, down.  Embeddings and norms are fp32; matrices are arrays
of 36-byte BlockQ8_0.  The reader raises RuntimeError on a bad magic or a
truncated file, as import_btmodel does (model_importer.cpp:46,50).
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass, field

import numpy as np

from .native import ModelConfig

MAGIC = 0x42544D44
DT_INT8 = 3  # blocktensor::DataType::INT8 (runtime/include/blocktensor/backend.hpp:11-17)
LAYER_TENSORS = ("attn_norm", "ffn_norm", "q", "k", "v", "o", "gate", "up", "down")


@dataclass
class BtModel:
    config: ModelConfig
    quant_type: int
    tensors: list = field(default_factory=list)  # uint8 numpy arrays in file order

    def expected_sizes(self):
        c = self.config
        D, F, V = c.dim, c.hidden_dim, c.vocab_size
        KV = c.num_kv_heads * c.head_dim
        qb = lambda r, k: r * k // 32 * 36
        sizes = [V * D * 4, D * 4, qb(V, D)]
        for _ in range(c.num_layers):
            sizes += [D * 4, D * 4, qb(D, D), qb(KV, D), qb(KV, D), qb(D, D), qb(F, D), qb(F, D), qb(D, F)]
        return sizes


def read_btmodel(path: str) -> BtModel:
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 4 or struct.unpack_from("<I", data, 0)[0] != MAGIC:
        raise RuntimeError("Invalid .btmodel magic header")
    if len(data) < 4 + 36 + 4:
        raise RuntimeError("truncated .btmodel header")
    cfg = ModelConfig.from_buffer_copy(data[4:40])
    qt = struct.unpack_from("<I", data, 40)[0]
    off = 44
    m = BtModel(cfg, qt)
    for _ in range(3 + 9 * cfg.num_layers):
        if off + 8 > len(data):
            raise RuntimeError("truncated .btmodel tensor table")
        (sz,) = struct.unpack_from("<Q", data, off)
        off += 8
        if off + sz > len(data):
            raise RuntimeError("truncated .btmodel tensor data")
        m.tensors.append(np.frombuffer(data, dtype=np.uint8, count=sz, offset=off))
        off += sz
    return m


def write_btmodel(path: str, config: ModelConfig, tensors, quant_type: int = DT_INT8) -> None:
    with open(path, "wb") as f:
        f.write(struct.pack("<I", MAGIC))
        f.write(bytes(config))
        f.write(struct.pack("<I", quant_type))
        for t in tensors:
            a = np.ascontiguousarray(t).view(np.uint8)
            f.write(struct.pack("<Q", a.nbytes))
            f.write(a.tobytes())
