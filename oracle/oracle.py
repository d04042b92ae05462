"""ctypes view of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Two libraries, both built by ``oracle/Makefile``:

* ``liboracle.so`` -- the plain-C restatement in ``bt_oracle.c`` (quantizer,
  matvec, rmsnorm/rope/softmax/silu, greedy sampler, the single-token engine
  with per-layer taps, the seeded synthetic-model generator).
* ``_ref/libbtref.so`` -- the reference's own CPU sources compiled unmodified,
  behind ``ref_shim.cpp``.  Present wherever it was built from the reference
  tree; tests that need it skip when it is missing.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module, and only to check or time the CPU reference.  The CUDA
product path never calls into it.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libbtref.so")

BLOCK = 32
BLOCK_BYTES = 36  # float scale + 32 int8 (quantization/quant_types.hpp:12-15)

# numpy view of BlockQ8_0
Q8_DTYPE = np.dtype([("scale", "<f4"), ("qs", "i1", (BLOCK,))])
assert Q8_DTYPE.itemsize == BLOCK_BYTES


class Config(C.Structure):
    """blocktensor::ModelConfig (runtime/include/blocktensor/model_config.hpp:9-19)."""

    _fields_ = [
        ("vocab_size", C.c_uint32),
        ("dim", C.c_uint32),
        ("hidden_dim", C.c_uint32),
        ("num_layers", C.c_uint32),
        ("num_heads", C.c_uint32),
        ("num_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("max_seq_len", C.c_uint32),
        ("rms_norm_eps", C.c_float),
    ]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


assert C.sizeof(Config) == 36


class _Layer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p)] + [
        (n, C.c_void_p) for n in ("q", "k", "v", "o", "gate", "up", "down")
    ]


class _Model(C.Structure):
    _fields_ = [
        ("cfg", Config),
        ("embed", C.c_void_p),
        ("out_norm", C.c_void_p),
        ("head", C.c_void_p),
        ("layers", C.POINTER(_Layer)),
        ("owns", C.c_int),
    ]


class _KV(C.Structure):
    _fields_ = [
        ("num_layers", C.c_uint32),
        ("max_seq", C.c_uint32),
        ("kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("kv_fp16", C.c_int),
        ("k", C.c_void_p),
        ("v", C.c_void_p),
    ]


STREAM_EMBED, STREAM_OUT_NORM, STREAM_HEAD = 0, 1, 2
STREAM_PROMPT = 0xF000
LAYER_TENSORS = ("attn_norm", "ffn_norm", "q", "k", "v", "o", "gate", "up", "down")


def stream_layer(l: int, j: int) -> int:
    return 16 + 16 * l + j


def _fp(a):
    return a.ctypes.data_as(C.c_void_p)


def _load_oracle():
    if not os.path.exists(ORACLE_SO):
        raise RuntimeError(f"{ORACLE_SO} missing: run `make -C oracle oracle`")
    lib = C.CDLL(ORACLE_SO)
    vp, u32, u64, f32, sz, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t, C.c_int
    sig = {
        "bto_quantize_q8_0": (i32, [vp, vp, sz]),
        "bto_dequantize_q8_0": (None, [vp, vp, sz]),
        "bto_matvec_q8_0": (None, [vp, vp, vp, u32, u32]),
        "bto_matvec_q8_0_mt": (None, [vp, vp, vp, u32, u32, i32]),
        "bto_rmsnorm": (None, [vp, vp, vp, u32, u32, f32]),
        "bto_rope": (None, [vp, vp, u32, u32, u32, u32, f32]),
        "bto_softmax": (None, [vp, vp, u32, u32]),
        "bto_silu": (None, [vp, vp, u32]),
        "bto_sample_greedy": (u32, [vp, u32]),
        "bto_gen_normal": (None, [u64, u64, u64, sz, f32, vp]),
        "bto_normal_k": (f32, [f32]),
        "bto_gen_int8": (None, [u64, u64, u64, sz, vp]),
        "bto_gen_uniform": (None, [u64, u64, u64, sz, f32, f32, vp]),
        "bto_gen_tokens": (None, [u64, u64, sz, u32, vp]),
        "bto_model_generate": (C.POINTER(_Model), [C.POINTER(Config), u64, f32, i32]),
        "bto_model_free": (None, [C.POINTER(_Model)]),
        "bto_kv_create": (C.POINTER(_KV), [u32, u32, u32, u32, i32]),
        "bto_kv_free": (None, [C.POINTER(_KV)]),
        "bto_forward_token": (i32, [C.POINTER(_Model), C.POINTER(_KV), u32, u32, f32, vp, vp, i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_ORACLE = None


def lib():
    global _ORACLE
    if _ORACLE is None:
        _ORACLE = _load_oracle()
    return _ORACLE


# ---------------------------------------------------------------- primitives

def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size // BLOCK, dtype=Q8_DTYPE)
    rc = lib().bto_quantize_q8_0(_fp(x), _fp(out), x.size)
    if rc != 0:
        raise ValueError("quantize_q8_0: num_elements must be a multiple of block size")
    return out


def dequantize_q8_0(blocks: np.ndarray) -> np.ndarray:
    out = np.zeros(blocks.size * BLOCK, dtype=np.float32)
    lib().bto_dequantize_q8_0(_fp(blocks), _fp(out), out.size)
    return out


def matvec_q8_0(blocks: np.ndarray, x: np.ndarray, M: int, N: int, nthreads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(M, dtype=np.float32)
    lib().bto_matvec_q8_0_mt(_fp(blocks), _fp(x), _fp(y), M, N, nthreads)
    return y


def rmsnorm(x, w, rows, dim, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(rows * dim, np.float32)
    lib().bto_rmsnorm(_fp(x), _fp(w), _fp(out), rows, dim, eps)
    return out


def rope(x, seq, heads, hd, pos, theta=10000.0):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().bto_rope(_fp(x), _fp(out), seq, heads, hd, pos, theta)
    return out


def softmax(x, rows, dim):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().bto_softmax(_fp(x), _fp(out), rows, dim)
    return out


def silu(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().bto_silu(_fp(x), _fp(out), x.size)
    return out


def sample_greedy(logits):
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().bto_sample_greedy(_fp(logits), logits.size))


def normal_k(sigma: float) -> float:
    return float(lib().bto_normal_k(sigma))


def gen_normal(seed, stream, n, sigma, offset=0):
    out = np.zeros(n, np.float32)
    lib().bto_gen_normal(seed, stream, offset, n, lib().bto_normal_k(sigma), _fp(out))
    return out


def gen_int8(seed, stream, n, offset=0):
    out = np.zeros(n, np.int8)
    lib().bto_gen_int8(seed, stream, offset, n, _fp(out))
    return out


def gen_uniform(seed, stream, n, lo, hi, offset=0):
    out = np.zeros(n, np.float32)
    lib().bto_gen_uniform(seed, stream, offset, n, lo, hi, _fp(out))
    return out


def gen_tokens(seed, stream, n, vocab):
    out = np.zeros(n, np.uint32)
    lib().bto_gen_tokens(seed, stream, n, vocab, _fp(out))
    return out


# ---------------------------------------------------------------- model / engine

def make_config(vocab, dim, hidden, layers, heads, kv_heads, head_dim, max_seq, eps=1e-5) -> Config:
    return Config(vocab, dim, hidden, layers, heads, kv_heads, head_dim, max_seq, eps)


@dataclass
class TensorRef:
    ptr: int
    nbytes: int
    kind: str  # "f32" or "q8"


class Model:
    """Synthetic seeded model held by the C oracle (matrices already Q8_0)."""

    def __init__(self, cfg: Config, seed: int = 0, sigma: float = 0.02, nthreads: int = 0):
        nthreads = nthreads or (os.cpu_count() or 1)
        self.cfg = cfg
        self.seed = seed
        self._p = lib().bto_model_generate(C.byref(cfg), seed, sigma, nthreads)

    def close(self):
        if getattr(self, "_p", None):
            lib().bto_model_free(self._p)
            self._p = None

    def __del__(self):
        self.close()

    def tensors(self):
        """(ptr, nbytes, kind) in .btmodel order (models/model_importer.cpp:69-85)."""
        c = self.cfg
        m = self._p.contents
        D, F, V = c.dim, c.hidden_dim, c.vocab_size
        KV = c.num_kv_heads * c.head_dim
        qb = lambda rows, cols: rows * cols // BLOCK * BLOCK_BYTES
        out = [TensorRef(m.embed, V * D * 4, "f32"), TensorRef(m.out_norm, D * 4, "f32"),
               TensorRef(m.head, qb(V, D), "q8")]
        shapes = {"q": (D, D), "k": (KV, D), "v": (KV, D), "o": (D, D),
                  "gate": (F, D), "up": (F, D), "down": (D, F)}
        for l in range(c.num_layers):
            L = m.layers[l]
            out.append(TensorRef(L.attn_norm, D * 4, "f32"))
            out.append(TensorRef(L.ffn_norm, D * 4, "f32"))
            for n in ("q", "k", "v", "o", "gate", "up", "down"):
                out.append(TensorRef(getattr(L, n), qb(*shapes[n]), "q8"))
        return out

    def tensor_array(self, t: TensorRef) -> np.ndarray:
        buf = (C.c_uint8 * t.nbytes).from_address(t.ptr)
        a = np.frombuffer(buf, dtype=np.uint8)
        return a.view(np.float32) if t.kind == "f32" else a.view(Q8_DTYPE)


class KV:
    def __init__(self, cfg: Config, max_seq: int, fp16: bool = False):
        self.cfg = cfg
        self._p = lib().bto_kv_create(cfg.num_layers, max_seq, cfg.num_kv_heads, cfg.head_dim, int(fp16))
        self.max_seq = max_seq

    def close(self):
        if getattr(self, "_p", None):
            lib().bto_kv_free(self._p)
            self._p = None

    def __del__(self):
        self.close()

    def layer(self, l):
        c = self.cfg
        n = self.max_seq * c.num_kv_heads * c.head_dim
        kv = self._p.contents
        k = np.ctypeslib.as_array((C.c_float * (c.num_layers * n)).from_address(kv.k))
        v = np.ctypeslib.as_array((C.c_float * (c.num_layers * n)).from_address(kv.v))
        return k[l * n:(l + 1) * n].copy(), v[l * n:(l + 1) * n].copy()


def forward_token(model: Model, kv: KV, token: int, pos: int, theta: float = 10000.0,
                  want_taps: bool = False, nthreads: int = 0):
    c = model.cfg
    nthreads = nthreads or (os.cpu_count() or 1)
    logits = np.zeros(c.vocab_size, np.float32)
    taps = np.zeros((c.num_layers, c.dim), np.float32) if want_taps else None
    rc = lib().bto_forward_token(model._p, kv._p, token, pos, theta, _fp(logits),
                                 _fp(taps) if taps is not None else None, nthreads)
    if rc == -2:
        raise IndexError("token or position out of range")
    return (logits, taps) if want_taps else logits


# ---------------------------------------------------------------- reference library

class RefLib:
    """The reference's own CPU code (oracle/_ref/libbtref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = C.CDLL(path)
        vp, u32, u64, f32, sz, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_float, C.c_size_t, C.c_int
        sig = {
            "btr_quantize_q8_0": (i32, [vp, vp, sz]),
            "btr_dequantize_q8_0": (i32, [vp, vp, sz]),
            "btr_matvec_q8_0": (i32, [vp, vp, vp, u32, u32]),
            "btr_quantize_q4_0": (i32, [vp, vp, sz]),
            "btr_rmsnorm": (None, [vp, vp, vp, u32, u32, f32]),
            "btr_rope": (None, [vp, vp, u32, u32, u32, u32]),
            "btr_softmax": (None, [vp, vp, u32, u32]),
            "btr_silu": (None, [vp, vp, u32]),
            "btr_sample_greedy": (u32, [vp, u32]),
            "btr_sample_top_p_top_k": (u32, [vp, u32, f32, f32, u32, u64]),
            "btr_sizeof_config": (sz, []),
            "btr_sizeof_block_q8_0": (sz, []),
            "btr_engine_create": (i32, [vp, vp, u32, u32, C.POINTER(vp)]),
            "btr_engine_import": (i32, [C.c_char_p, u32, C.POINTER(vp)]),
            "btr_engine_export": (i32, [vp, C.c_char_p]),
            "btr_engine_config": (i32, [vp, vp]),
            "btr_engine_allocated_bytes": (u64, [vp]),
            "btr_engine_forward": (i32, [vp, u32, u32, vp]),
            "btr_engine_read_kv": (i32, [vp, u32, vp, vp, u64]),
            "btr_engine_destroy": (None, [vp]),
            "btr_kv_update_probe": (i32, [u32, u32, u32, u32, u32, u32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        self.L = L

    def __getattr__(self, name):
        return getattr(self.L, name)

    # convenience wrappers -------------------------------------------------
    def quantize_q8_0(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.zeros(x.size // BLOCK, dtype=Q8_DTYPE)
        rc = self.L.btr_quantize_q8_0(_fp(x), _fp(out), x.size)
        if rc == -4:
            raise ValueError("quantize_q8_0: num_elements must be a multiple of block size")
        return out

    def matvec_q8_0(self, blocks, x, M, N):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(M, np.float32)
        assert self.L.btr_matvec_q8_0(_fp(blocks), _fp(x), _fp(y), M, N) == 0
        return y


class RefEngine:
    """The reference TransformerEngine on its CPUBackend, fed the oracle's synthetic weights."""

    def __init__(self, ref: RefLib, model: Model, kv_max_seq: int = 0):
        self.ref = ref
        self.cfg = model.cfg
        ts = model.tensors()
        arr = (C.c_uint64 * (2 * len(ts)))()
        for i, t in enumerate(ts):
            arr[2 * i] = t.ptr
            arr[2 * i + 1] = t.nbytes
        h = C.c_void_p()
        rc = ref.btr_engine_create(C.byref(model.cfg), arr, len(ts), kv_max_seq, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"btr_engine_create failed: {rc}")
        self.h = h

    @classmethod
    def from_file(cls, ref: RefLib, path: str, kv_max_seq: int = 0):
        self = cls.__new__(cls)
        self.ref = ref
        h = C.c_void_p()
        rc = ref.btr_engine_import(path.encode(), kv_max_seq, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"import_btmodel failed: {rc}")
        self.h = h
        cfg = Config()
        ref.btr_engine_config(h, C.byref(cfg))
        self.cfg = cfg
        return self

    def export(self, path: str):
        rc = self.ref.btr_engine_export(self.h, path.encode())
        if rc != 0:
            raise RuntimeError(f"export_btmodel failed: {rc}")

    def forward(self, token, pos):
        logits = np.zeros(self.cfg.vocab_size, np.float32)
        rc = self.ref.btr_engine_forward(self.h, token, pos, _fp(logits))
        if rc == -2:
            raise IndexError("out_of_range")
        if rc != 0:
            raise RuntimeError(f"forward_single_token failed: {rc}")
        return logits

    def close(self):
        if getattr(self, "h", None):
            self.ref.btr_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


def ref_available() -> bool:
    return os.path.exists(REF_SO)
