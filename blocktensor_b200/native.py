"""ctypes binding of ``libbt_cuda.so`` (the C ABI declared in include/bt_cuda.h).

The library is the product: there is no CPU fallback.  If it is missing or
fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libbt_cuda.so")

BT_OK = 0
BT_ERR_UNKNOWN = -1
BT_ERR_OUT_OF_RANGE = -2
BT_ERR_RUNTIME = -3
BT_ERR_INVALID_ARGUMENT = -4
BT_ERR_CUDA = -5
BT_ERR_OUT_OF_MEMORY = -6
BT_ERR_DEVICE_TIMEOUT = -7

BT_KV_FP32 = 0
BT_KV_FP16 = 1


class CudaBackendError(RuntimeError):
    """A CUDA runtime failure inside the backend (BT_ERR_CUDA / BT_ERR_DEVICE_TIMEOUT)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class ModelConfig(C.Structure):
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

    def __repr__(self):
        return "ModelConfig(" + ", ".join(f"{f}={getattr(self, f)}" for f, _ in self._fields_) + ")"


assert C.sizeof(ModelConfig) == 36


class EngineOptions(C.Structure):
    _fields_ = [("rope_theta", C.c_float), ("tp_rank", C.c_uint32), ("tp_world", C.c_uint32),
                ("reserved", C.c_uint32 * 5)]


BT_TP_HANDLE_BYTES = 64


class TensorView(C.Structure):
    _fields_ = [("data", C.c_void_p), ("bytes", C.c_uint64)]


_vp, _u32, _u64, _i32, _f32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float

# name -> (restype, argtypes); must match include/bt_cuda.h
SIGNATURES = {
    "bt_cuda_abi_version": (_i32, []),
    "bt_cuda_last_error": (C.c_char_p, []),
    "bt_cuda_launch_count": (_u64, []),
    "bt_cuda_device_info": (_i32, [_i32, C.c_char_p, _vp, _vp, _vp]),
    "bt_cuda_alloc": (_i32, [_i32, _u64, C.POINTER(_vp)]),
    "bt_cuda_free": (_i32, [_i32, _vp]),
    "bt_cuda_copy_h2d": (_i32, [_i32, _vp, _vp, _u64]),
    "bt_cuda_copy_d2h": (_i32, [_i32, _vp, _vp, _u64]),
    "bt_cuda_synchronize": (_i32, [_i32]),
    "bt_cuda_quantize_q8_0": (_i32, [_vp, _vp, _u64, _vp]),
    "bt_cuda_dequantize_q8_0": (_i32, [_vp, _vp, _u64, _vp]),
    "bt_cuda_matvec_q8_0": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_quantize_q4_0": (_i32, [_vp, _vp, _u64, _vp]),
    "bt_cuda_dequantize_q4_0": (_i32, [_vp, _vp, _u64, _vp]),
    "bt_cuda_matvec_q4_0": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_repack_q8_0": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_gemv_q8": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "bt_cuda_gemm_q8_units": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "bt_cuda_pack_q8_units": (_i32, [_vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_gemv_q8_units": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_gemv_q8_units_noalloc": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_gemv_inject_timeout": (_i32, [_i32, _i32]),
    "bt_cuda_gemv_bench": (_i32, [_i32, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u64, _u32, _vp, C.POINTER(_f32)]),
    "bt_cuda_rmsnorm": (_i32, [_vp, _vp, _vp, _u32, _u32, _f32, _vp]),
    "bt_cuda_rope": (_i32, [_vp, _vp, _u32, _u32, _u32, _u32, _f32, _vp]),
    "bt_cuda_softmax": (_i32, [_vp, _vp, _u32, _u32, _vp]),
    "bt_cuda_silu": (_i32, [_vp, _vp, _u32, _vp]),
    "bt_cuda_argmax": (_i32, [_vp, _u32, _vp, _vp]),
    "bt_cuda_sample_top_p_top_k": (_i32, [_vp, _u32, _f32, _f32, _u32, _u64, _vp, _vp]),
    "bt_engine_create": (_i32, [_i32, C.POINTER(ModelConfig), C.POINTER(EngineOptions), C.POINTER(_vp)]),
    "bt_engine_destroy": (_i32, [_vp]),
    "bt_engine_load": (_i32, [_vp, C.POINTER(TensorView), _u32, _i32]),
    "bt_engine_generate": (_i32, [_vp, _u64, _f32]),
    "bt_kv_create": (_i32, [_vp, _u32, _i32, C.POINTER(_vp)]),
    "bt_kv_destroy": (_i32, [_vp]),
    "bt_kv_read_layer": (_i32, [_vp, _u32, _vp, _vp]),
    "bt_engine_forward_token": (_i32, [_vp, _vp, _u32, _u32, _vp, _vp]),
    "bt_engine_decode": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "bt_engine_prefill": (_i32, [_vp, _vp, _vp, _u32, _u32]),
    "bt_kv_read_tokens": (_i32, [_vp, _u32, _u32, _vp]),
    "bt_engine_set_taps": (_i32, [_vp, _i32]),
    "bt_engine_read_taps": (_i32, [_vp, _vp]),
    "bt_engine_set_trace": (_i32, [_vp, _i32]),
    "bt_engine_read_trace": (_i32, [_vp, _vp, _u64]),
    "bt_engine_tp_handle": (_i32, [_vp, _vp]),
    "bt_engine_tp_connect": (_i32, [_vp, _vp]),
    "bt_engine_begin": (_i32, [_vp, _vp, _vp, _u32, _u32]),
    "bt_engine_steps": (_i32, [_vp, _vp, _u32, _vp]),
    "bt_engine_stream": (_vp, [_vp]),
    "bt_engine_profile": (_i32, [_vp, _vp, _u32, _vp]),
    "bt_kv_state": (_i32, [_vp, _vp, _vp, _vp]),
    "bt_kv_inject_stall": (_i32, [_vp]),
    "bt_kv_step_info": (_i32, [_vp, _u32, _vp, _vp]),
    "bt_batch_create": (_i32, [_vp, _u32, _u32, _i32, C.POINTER(_vp)]),
    "bt_batch_destroy": (_i32, [_vp]),
    "bt_batch_prefill": (_i32, [_vp, _u32, _vp, _u32]),
    "bt_batch_steps": (_i32, [_vp, _u32, _vp]),
    "bt_batch_read_tokens": (_i32, [_vp, _u32, _u32, _u32, _vp]),
    "bt_batch_read_current": (_i32, [_vp, _vp]),
    "bt_batch_read_logits": (_i32, [_vp, _vp]),
    "bt_batch_step_info": (_i32, [_vp, _vp]),
    "bt_batch_create_paged": (_i32, [_vp, _u32, _u32, _u32, _u32, _i32, C.POINTER(_vp)]),
    "bt_batch_release": (_i32, [_vp, _u32]),
    "bt_batch_pages": (_i32, [_vp, _vp, _vp]),
}

_LIB = None


def load(path: str = LIB_PATH):
    """Load the shared library (raises if it is absent: there is no fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python -m blocktensor_b200.build` (nvcc, sm_100a)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def last_error() -> str:
    msg = load().bt_cuda_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str = "") -> None:
    """Map a status code to the exception type the reference throws."""
    if rc == BT_OK:
        return
    msg = last_error() or what
    if rc == BT_ERR_OUT_OF_RANGE:
        raise IndexError(msg)  # std::out_of_range
    if rc == BT_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)  # std::invalid_argument
    if rc == BT_ERR_RUNTIME:
        raise RuntimeError(msg)  # std::runtime_error
    if rc == BT_ERR_OUT_OF_MEMORY:
        raise MemoryError(msg)
    raise CudaBackendError(rc, msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
