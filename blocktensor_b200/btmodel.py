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


# ---------------------------------------------------------------- .btmodel v2
# v1 stores the raw ModelConfig and nothing else (models/model_importer.cpp:53):
# no RoPE base, no KV-cache type, no tensor names or shapes.  v2 keeps v1's
# tensor order and block formats and adds a self-describing header:
#
#   u32 magic 0x324D5442 ("BTM2")   u32 version (2)   u32 header bytes (to the data)
#   ModelConfig (36 bytes)          f32 rope_theta    u32 kv_dtype (0 fp32, 1 fp16)
#   u32 quant type (DataType)       u32 tensor count
#   per tensor: u16 name length, name (utf-8), u32 dtype, u32 ndims, u64 dims[ndims],
#               u64 offset (from the file start), u64 bytes
#   tensor data, each tensor 64-byte aligned (a reader can map the file and upload
#   straight from it)
#
# dtype codes are blocktensor::DataType's (backend.hpp:11-17): FLOAT32 0, INT8 3
# (36-byte BlockQ8_0 blocks), INT4 4 (20-byte BlockQ4_0 blocks).

MAGIC_V2 = 0x324D5442
DT_FLOAT32 = 0
DT_INT4 = 4
_ALIGN = 64


def tensor_names(n_layers: int):
    names = ["embed_tokens", "output_norm", "output_head"]
    for l in range(n_layers):
        names += [f"layers.{l}.{n}" for n in LAYER_TENSORS]
    return names


@dataclass
class BtModelV2(BtModel):
    rope_theta: float = 10000.0
    kv_dtype: int = 0
    names: list = field(default_factory=list)
    dims: list = field(default_factory=list)
    dtypes: list = field(default_factory=list)


def write_btmodel_v2(path: str, config: ModelConfig, tensors, dims, rope_theta: float = 10000.0,
                     kv_dtype: int = 0, quant_type: int = DT_INT8) -> None:
    """tensors: uint8/float arrays in v1 order; dims: each tensor's logical shape (rows, cols)."""
    names = tensor_names(config.num_layers)
    if len(tensors) != len(names) or len(dims) != len(names):
        raise ValueError("write_btmodel_v2: expected 3 + 9 * num_layers tensors and shapes")
    dtypes = [DT_FLOAT32 if i < 2 or (i >= 3 and (i - 3) % 9 < 2) else quant_type for i in range(len(names))]
    arrays = [np.ascontiguousarray(t).view(np.uint8).reshape(-1) for t in tensors]
    table = bytearray()
    for n, d, dt in zip(names, dims, dtypes):
        nb = n.encode()
        table += struct.pack("<H", len(nb)) + nb + struct.pack("<II", dt, len(d)) + struct.pack(f"<{len(d)}Q", *d)
        table += b"\0" * 16  # offset and size, filled below
    fixed = 4 * 3 + 36 + 4 * 4
    header = fixed + len(table)
    off = (header + _ALIGN - 1) // _ALIGN * _ALIGN
    offsets = []
    for a in arrays:
        offsets.append(off)
        off = (off + a.nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
    # patch offsets and sizes into the table
    pos = 0
    for i, (n, d) in enumerate(zip(names, dims)):
        pos += 2 + len(n.encode()) + 8 + 8 * len(d)
        struct.pack_into("<QQ", table, pos, offsets[i], arrays[i].nbytes)
        pos += 16
    with open(path, "wb") as f:
        f.write(struct.pack("<III", MAGIC_V2, 2, header))
        f.write(bytes(config))
        f.write(struct.pack("<fIII", rope_theta, kv_dtype, quant_type, len(names)))
        f.write(bytes(table))
        for o, a in zip(offsets, arrays):
            f.seek(o)
            f.write(a.tobytes())
        f.truncate(off)


def read_btmodel_any(path: str) -> BtModel:
    """A .btmodel of either version (v1: the reference's format, RoPE base 10000)."""
    with open(path, "rb") as f:
        head = f.read(4)
    if len(head) == 4 and struct.unpack("<I", head)[0] == MAGIC:
        return read_btmodel(path)
    return read_btmodel_v2(path)


def read_btmodel_v2(path: str) -> BtModelV2:
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 12 or struct.unpack_from("<I", data, 0)[0] != MAGIC_V2:
        raise RuntimeError("Invalid .btmodel magic header")
    version, header = struct.unpack_from("<II", data, 4)
    if version != 2:
        raise RuntimeError(f"unsupported .btmodel version {version}")
    if len(data) < 12 + 36 + 16 or header > len(data):
        raise RuntimeError("truncated .btmodel header")
    cfg = ModelConfig.from_buffer_copy(data[12:48])
    theta, kv_dtype, qt, n = struct.unpack_from("<fIII", data, 48)
    if n != 3 + 9 * cfg.num_layers:
        raise RuntimeError(".btmodel v2: tensor count does not match the config")
    m = BtModelV2(cfg, qt, rope_theta=theta, kv_dtype=kv_dtype)
    pos = 64
    for _ in range(n):
        (ln,) = struct.unpack_from("<H", data, pos)
        pos += 2
        m.names.append(data[pos:pos + ln].decode())
        pos += ln
        dt, nd = struct.unpack_from("<II", data, pos)
        pos += 8
        m.dims.append(struct.unpack_from(f"<{nd}Q", data, pos))
        pos += 8 * nd
        o, sz = struct.unpack_from("<QQ", data, pos)
        pos += 16
        if o + sz > len(data):
            raise RuntimeError("truncated .btmodel tensor data")
        m.dtypes.append(dt)
        m.tensors.append(np.frombuffer(data, dtype=np.uint8, count=sz, offset=o))
    sizes = m.expected_sizes()
    for i, (t, want) in enumerate(zip(m.tensors, sizes)):
        if t.nbytes != want:
            raise RuntimeError(f".btmodel v2: tensor {m.names[i]} has {t.nbytes} bytes, expected {want}")
    return m
