"""BlockTensor B200 backend: the int8 single-token decode path on sm_100a.

Host-side mirror of the reference's engine interface
(runtime/include/blocktensor/transformer_engine.hpp, kv_cache.hpp,
quantization/quant_types.hpp), calling the CUDA kernels through the C ABI in
include/bt_cuda.h.  Device buffers are torch CUDA tensors; weights, KV cache
and activations stay resident on the GPU.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import native
from .native import (BT_KV_FP16, BT_KV_FP32, BT_TP_HANDLE_BYTES, CudaBackendError, EngineOptions, ModelConfig,
                     TensorView, call, load)

__all__ = [
    "ModelConfig", "TransformerEngine", "KVCache", "CudaBackendError", "BT_KV_FP16", "BT_KV_FP32",
    "quantize_q8_0", "dequantize_q8_0", "matvec_q8_0", "repack_q8_0", "gemv_q8",
    "rmsnorm", "rope", "softmax", "silu", "argmax", "launch_count", "model_config",
]

Q8_BLOCK = 32
Q8_BLOCK_BYTES = 36


def model_config(vocab_size, dim, hidden_dim, num_layers, num_heads, num_kv_heads, head_dim,
                 max_seq_len, rms_norm_eps=1e-5) -> ModelConfig:
    return ModelConfig(vocab_size, dim, hidden_dim, num_layers, num_heads, num_kv_heads, head_dim,
                       max_seq_len, rms_norm_eps)


def launch_count() -> int:
    """Kernel launches issued by libbt_cuda.so in this process."""
    return int(load().bt_cuda_launch_count())


# ---------------------------------------------------------------- torch helpers

def _torch():
    import torch
    return torch


def _dev_ptr(t) -> int:
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


# ---------------------------------------------------------------- quantization (quant_types.hpp)

def quantize_q8_0(x, stream=None):
    """quantization::quantize_q8_0 (quant_types.cpp:8-34) on a CUDA fp32 tensor.

    Returns a uint8 CUDA tensor of n/32 blocks of 36 bytes (BlockQ8_0 layout).
    """
    torch = _torch()
    if x.numel() % Q8_BLOCK:
        raise ValueError("quantize_q8_0: num_elements must be a multiple of block size")
    out = torch.empty(x.numel() // Q8_BLOCK * Q8_BLOCK_BYTES, dtype=torch.uint8, device=x.device)
    call("bt_cuda_quantize_q8_0", _dev_ptr(x), _dev_ptr(out) if out.numel() else None, x.numel(), _stream(stream))
    return out


def dequantize_q8_0(blocks, n: int | None = None, stream=None):
    """quantization::dequantize_q8_0 (quant_types.cpp:36-48)."""
    torch = _torch()
    n = blocks.numel() // Q8_BLOCK_BYTES * Q8_BLOCK if n is None else n
    out = torch.empty(n, dtype=torch.float32, device=blocks.device)
    call("bt_cuda_dequantize_q8_0", _dev_ptr(blocks), _dev_ptr(out), n, _stream(stream))
    return out


def matvec_q8_0(blocks, x, M: int, N: int, stream=None):
    """quantization::matvec_q8_0 (quant_types.cpp:101-121) on 36-byte blocks."""
    torch = _torch()
    y = torch.empty(M, dtype=torch.float32, device=x.device)
    call("bt_cuda_matvec_q8_0", _dev_ptr(blocks), _dev_ptr(x), _dev_ptr(y), M, N, _stream(stream))
    return y


def repack_q8_0(blocks, M: int, K: int, stream=None):
    """36-byte blocks -> (qs [M,K] int8, scales [M,K/32] fp32) device layout."""
    torch = _torch()
    qs = torch.empty((M, K), dtype=torch.int8, device=blocks.device)
    sc = torch.empty((M, K // Q8_BLOCK), dtype=torch.float32, device=blocks.device)
    call("bt_cuda_repack_q8_0", _dev_ptr(blocks), _dev_ptr(qs), _dev_ptr(sc), M, K, _stream(stream))
    return qs, sc


def unit_bytes(M: int, K: int) -> int:
    """Bytes of an M x K matrix in the tensor-core tile layout (128 x 32 tiles of 4608 bytes)."""
    return (M + 127) // 128 * (K // Q8_BLOCK) * 4608


def pack_q8_units(blocks, M: int, K: int, stream=None):
    """36-byte blocks -> the unit layout of the tensor-core GEMV (uint8 CUDA tensor)."""
    torch = _torch()
    units = torch.empty(unit_bytes(M, K), dtype=torch.uint8, device=blocks.device)
    call("bt_cuda_pack_q8_units", _dev_ptr(blocks), _dev_ptr(units), M, K, _stream(stream))
    return units


def gemv_q8_units(units, x, M: int, K: int, stream=None, out=None):
    """y = W x on the unit layout (tensor-core GEMV of the decode engine)."""
    torch = _torch()
    y = out if out is not None else torch.empty(M, dtype=torch.float32, device=x.device)
    call("bt_cuda_gemv_q8_units", _dev_ptr(units), _dev_ptr(x), _dev_ptr(y), M, K, _stream(stream))
    return y


def gemm_q8_units(units, x, M: int, K: int, stream=None, out=None):
    """Y = X W^T for X [T, K] on the unit layout (the tensor-core GEMM of prefill / batched decode)."""
    torch = _torch()
    x2 = x.reshape(-1, K).contiguous()
    T = x2.shape[0]
    y = out if out is not None else torch.empty((T, M), dtype=torch.float32, device=x.device)
    call("bt_cuda_gemm_q8_units", _dev_ptr(units), _dev_ptr(x2), _dev_ptr(y), M, K, T, _stream(stream))
    return y


def gemv_q8(qs, scales, x, stream=None, out=None):
    """y[b] = W x[b] for x of shape [B, K] (B <= 16), W in the device layout."""
    torch = _torch()
    M, K = qs.shape
    x2 = x.reshape(-1, K)
    B = x2.shape[0]
    y = out if out is not None else torch.empty((B, M), dtype=torch.float32, device=x.device)
    call("bt_cuda_gemv_q8", _dev_ptr(qs), _dev_ptr(scales), _dev_ptr(x2), _dev_ptr(y), M, K, B, _stream(stream))
    return y


# ---------------------------------------------------------------- cpu_ref.hpp on device

def rmsnorm(x, w, rows: int, dim: int, eps: float = 1e-5, stream=None):
    torch = _torch()
    out = torch.empty(rows * dim, dtype=torch.float32, device=x.device)
    call("bt_cuda_rmsnorm", _dev_ptr(x), _dev_ptr(w), _dev_ptr(out), rows, dim, eps, _stream(stream))
    return out


def rope(x, seq: int, heads: int, head_dim: int, pos: int, theta: float = 10000.0, stream=None):
    torch = _torch()
    out = torch.empty_like(x)
    call("bt_cuda_rope", _dev_ptr(x), _dev_ptr(out), seq, heads, head_dim, pos, theta, _stream(stream))
    return out


def softmax(x, rows: int, dim: int, stream=None):
    torch = _torch()
    out = torch.empty_like(x)
    call("bt_cuda_softmax", _dev_ptr(x), _dev_ptr(out), rows, dim, _stream(stream))
    return out


def silu(x, stream=None):
    torch = _torch()
    out = torch.empty_like(x)
    call("bt_cuda_silu", _dev_ptr(x), _dev_ptr(out), x.numel(), _stream(stream))
    return out


def argmax(logits, stream=None) -> int:
    """sampling::sample_greedy (sampler.hpp:11-13): first maximum wins."""
    torch = _torch()
    out = torch.zeros(1, dtype=torch.int32, device=logits.device)
    call("bt_cuda_argmax", _dev_ptr(logits), logits.numel(), _dev_ptr(out), _stream(stream))
    return int(out.item())


# ---------------------------------------------------------------- engine (transformer_engine.hpp)

class TransformerEngine:
    """Device-resident replacement of blocktensor::TransformerEngine.

    ``TransformerEngine(config)`` allocates the weights on ``device``; fill them
    with :meth:`load` (the 3 + 9L tensors of a .btmodel, in file order) or
    :meth:`generate` (seeded synthetic weights, bit-identical to the CPU
    oracle's generator).  :meth:`forward_single_token` has the reference
    signature and returns the logits as a numpy array.
    """

    def __init__(self, config: ModelConfig, device: int = 0, rope_theta: float = 10000.0,
                 tp_rank: int = 0, tp_world: int = 1):
        self.config = config
        self.device = device
        opt = EngineOptions()
        opt.rope_theta = rope_theta
        opt.tp_rank = tp_rank
        opt.tp_world = tp_world
        self.rope_theta = rope_theta
        self.tp_rank, self.tp_world = tp_rank, tp_world
        h = C.c_void_p()
        call("bt_engine_create", device, C.byref(config), C.byref(opt), C.byref(h))
        self._h = h

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            load().bt_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @classmethod
    def from_btmodel(cls, path: str, device: int = 0) -> "TransformerEngine":
        """An engine loaded from a .btmodel file of either version (v2 carries the RoPE base;
        v1, the reference's format, uses cpu_ref::rope's 10000)."""
        from . import btmodel
        m = btmodel.read_btmodel_any(path)
        eng = cls(m.config, device=device, rope_theta=getattr(m, "rope_theta", 10000.0))
        eng.load(m.tensors)
        eng.kv_dtype_hint = BT_KV_FP16 if getattr(m, "kv_dtype", 0) == 1 else BT_KV_FP32
        return eng

    def load(self, tensors: Sequence, on_device: bool = False):
        """tensors: buffers (numpy arrays, or CUDA tensors with on_device=True) in .btmodel order."""
        n = len(tensors)
        views = (TensorView * n)()
        keep = []
        for i, t in enumerate(tensors):
            if on_device:
                views[i].data = _dev_ptr(t)
                views[i].bytes = t.numel() * t.element_size()
            else:
                a = np.ascontiguousarray(t)
                keep.append(a)
                views[i].data = a.ctypes.data
                views[i].bytes = a.nbytes
        call("bt_engine_load", self._h, views, n, int(on_device))

    def load_pointers(self, ptrs_and_sizes: Sequence[tuple[int, int]]):
        """Host (pointer, bytes) pairs in .btmodel order."""
        n = len(ptrs_and_sizes)
        views = (TensorView * n)()
        for i, (p, b) in enumerate(ptrs_and_sizes):
            views[i].data = p
            views[i].bytes = b
        call("bt_engine_load", self._h, views, n, 0)

    def generate(self, seed: int = 0, sigma: float = 0.02):
        call("bt_engine_generate", self._h, seed, sigma)

    def forward_single_token(self, token: int, pos: int, kv: "KVCache", want_logits: bool = True):
        logits = np.zeros(self.config.vocab_size, np.float32) if want_logits else None
        am = C.c_uint32()
        call("bt_engine_forward_token", self._h, kv.handle, token, pos,
             logits.ctypes.data if want_logits else None, C.byref(am))
        self.last_argmax = am.value
        return logits

    def decode(self, kv: "KVCache", prompt: Sequence[int], n_gen: int, pos0: int = 0) -> np.ndarray:
        """Prompt then greedy decode on the device; returns the token consumed at
        each position plus the final argmax (len(prompt) + n_gen + 1 ids)."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        out = np.zeros(len(p) + n_gen + 1, np.uint32)
        call("bt_engine_decode", self._h, kv.handle, p.ctypes.data, len(p), pos0, n_gen, out.ctypes.data)
        return out

    def prefill(self, kv: "KVCache", prompt: Sequence[int], pos0: int = 0):
        """bt_engine_prefill: all prompt positions but the last as batched GEMMs; the next
        step processes the last prompt token."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        call("bt_engine_prefill", self._h, kv.handle, p.ctypes.data, len(p), pos0)

    def generate_tokens(self, kv: "KVCache", prompt: Sequence[int], n_gen: int, pos0: int = 0) -> np.ndarray:
        """As decode(), with the prompt prefilled by batched GEMMs (bt_engine_prefill)."""
        self.prefill(kv, prompt, pos0)
        self.steps(kv, 1 + n_gen)
        return kv.read_tokens(pos0, len(prompt) + n_gen + 1)

    def tp_handle(self) -> bytes:
        """This rank's exchange handle (tensor parallelism; see tp.connect)."""
        buf = C.create_string_buffer(BT_TP_HANDLE_BYTES)
        call("bt_engine_tp_handle", self._h, buf)
        return buf.raw

    def tp_connect(self, handles: Sequence[bytes]):
        """Maps every rank's exchange buffer; handles in rank order."""
        if len(handles) != self.tp_world or any(len(h) != BT_TP_HANDLE_BYTES for h in handles):
            raise ValueError("tp_connect: one handle of BT_TP_HANDLE_BYTES per rank")
        buf = C.create_string_buffer(b"".join(handles), BT_TP_HANDLE_BYTES * self.tp_world)
        call("bt_engine_tp_connect", self._h, buf)

    def set_taps(self, enable: bool = True):
        call("bt_engine_set_taps", self._h, int(enable))

    def read_taps(self) -> np.ndarray:
        c = self.config
        out = np.zeros((c.num_layers, c.dim), np.float32)
        call("bt_engine_read_taps", self._h, out.ctypes.data)
        return out

    def set_trace(self, enable: bool = True):
        """Per-phase device timestamps of every later step (bt_engine_set_trace)."""
        call("bt_engine_set_trace", self._h, int(enable))

    def read_trace(self) -> np.ndarray:
        """The last step's timestamps, [5 L + 1][SMs][8] uint64 nanoseconds (0: not recorded)."""
        P = 5 * self.config.num_layers + 1
        n = P * self.num_sms * 8
        out = np.zeros(n, np.uint64)
        call("bt_engine_read_trace", self._h, out.ctypes.data, n)
        return out.reshape(P, self.num_sms, 8)

    @property
    def num_sms(self) -> int:
        import torch
        return torch.cuda.get_device_properties(self.device).multi_processor_count

    def begin(self, kv: "KVCache", prompt: Sequence[int], pos0: int = 0):
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        call("bt_engine_begin", self._h, kv.handle, p.ctypes.data, len(p), pos0)

    def steps(self, kv: "KVCache", n: int, stream=None):
        call("bt_engine_steps", self._h, kv.handle, n, stream)

    KERNEL_KINDS = ("qkv", "attention", "oproj", "gateup", "down", "head")

    def profile(self, kv: "KVCache", n_steps: int) -> dict:
        """Per-kernel-kind device milliseconds summed over n_steps eager steps."""
        ms = (C.c_float * 6)()
        call("bt_engine_profile", self._h, kv.handle, n_steps, ms)
        return {k: float(ms[i]) for i, k in enumerate(self.KERNEL_KINDS)}

    @property
    def stream_handle(self) -> int:
        return load().bt_engine_stream(self._h) or 0


class Batch:
    """Independent sequences decoded together (bt_batch_*): one token row per sequence in
    every tensor-core GEMM, attention per sequence over its own cache."""

    def __init__(self, engine: TransformerEngine, n_seq: int, max_seq: int, kv_dtype: int = BT_KV_FP32,
                 page_tokens: int = 0, n_pages: int = 0):
        """page_tokens > 0: the KV lives in a pool of n_pages pages of page_tokens positions
        (bt_batch_create_paged) that the sequences take as they grow and give back on release()."""
        self.engine = engine
        self.n_seq, self.max_seq = n_seq, max_seq
        self.page_tokens, self.n_pages = page_tokens, n_pages
        h = C.c_void_p()
        if page_tokens:
            call("bt_batch_create_paged", engine.handle, n_seq, max_seq, page_tokens, n_pages, kv_dtype, C.byref(h))
        else:
            call("bt_batch_create", engine.handle, n_seq, max_seq, kv_dtype, C.byref(h))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            load().bt_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def prefill(self, s: int, prompt: Sequence[int]):
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        call("bt_batch_prefill", self._h, s, p.ctypes.data, len(p))

    def steps(self, n: int, stream=None):
        call("bt_batch_steps", self._h, n, stream)

    def read_tokens(self, s: int, pos0: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.uint32)
        call("bt_batch_read_tokens", self._h, s, pos0, n, out.ctypes.data)
        return out

    def read_current(self) -> np.ndarray:
        """Every sequence's newest token, one copy (bt_batch_read_current)."""
        out = np.zeros(self.n_seq, np.uint32)
        call("bt_batch_read_current", self._h, out.ctypes.data)
        return out

    def read_logits(self) -> np.ndarray:
        out = np.zeros((self.n_seq, self.engine.config.vocab_size), np.float32)
        call("bt_batch_read_logits", self._h, out.ctypes.data)
        return out

    def step_bytes(self) -> int:
        b = C.c_uint64()
        call("bt_batch_step_info", self._h, C.byref(b))
        return b.value

    def release(self, s: int):
        """Ends slot s's sequence: its pages go back to the pool (paged batches only)."""
        call("bt_batch_release", self._h, s)

    def pages(self):
        """(free, total) pages of the pool."""
        f, t = C.c_uint32(), C.c_uint32()
        call("bt_batch_pages", self._h, C.byref(f), C.byref(t))
        return f.value, t.value


class KVCache:
    """Device KV cache (runtime/include/blocktensor/kv_cache.hpp) of one sequence."""

    def __init__(self, engine: TransformerEngine, max_seq: int, kv_dtype: int = BT_KV_FP32):
        self.engine = engine
        self.max_seq = max_seq
        self.kv_dtype = kv_dtype
        h = C.c_void_p()
        call("bt_kv_create", engine.handle, max_seq, kv_dtype, C.byref(h))
        self._h = h

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            load().bt_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def read_layer(self, layer: int):
        """(K, V) of one layer in the reference layout [max_seq][kv_heads][head_dim], fp32."""
        c = self.engine.config
        n = self.max_seq * c.num_kv_heads * c.head_dim
        k = np.zeros(n, np.float32)
        v = np.zeros(n, np.float32)
        call("bt_kv_read_layer", self._h, layer, k.ctypes.data, v.ctypes.data)
        return k, v

    def read_tokens(self, pos0: int, n: int) -> np.ndarray:
        """Token consumed at positions pos0 .. pos0 + n - 1 (bt_kv_read_tokens)."""
        out = np.zeros(n, np.uint32)
        call("bt_kv_read_tokens", self._h, pos0, n, out.ctypes.data)
        return out

    def state(self):
        pos, tok, am = C.c_uint32(), C.c_uint32(), C.c_uint32()
        call("bt_kv_state", self._h, C.byref(pos), C.byref(tok), C.byref(am))
        return pos.value, tok.value, am.value

    def inject_stall(self):
        """Test hook: the next step's device waits expire (bt_kv_inject_stall)."""
        call("bt_kv_inject_stall", self._h)

    def step_info(self, context: int):
        launches, nbytes = C.c_uint64(), C.c_uint64()
        call("bt_kv_step_info", self._h, context, C.byref(launches), C.byref(nbytes))
        return launches.value, nbytes.value
