"""GPU parity of the Q4_0 (4-bit) path against the reference's own code.

quantize_q4_0 must be bit-exact with the reference (quant_types.cpp:50-79),
dequantize exact, matvec_q4_0 within the GEMV bar (1e-5 of sum |s q x| per
row), and an INT4 .btmodel must drive the CUDA engine to the reference
engine's logits (1e-2) and greedy tokens; the reference engine runs its own
matvec_q4_0 path for it (transformer_engine.cpp:63-65, 87-91).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

Q4_DTYPE = np.dtype([("scale", "<f4"), ("qs", "u1", (16,))])


def ref_q4(ref, x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size // 32, Q4_DTYPE)
    assert ref.btr_quantize_q4_0(x.ctypes.data, out.ctypes.data, x.size) == 0
    return out


def decode_q4(blocks):
    qs = blocks["qs"]
    codes = np.stack([qs & 15, qs >> 4], axis=-1).reshape(len(blocks), 32).astype(np.int32) - 8
    return codes, blocks["scale"]


@pytest.mark.parametrize("kind", ["normal", "uniform", "edge"])
def test_quantize_q4_bit_exact(cuda, ref, kind):
    import torch
    from blocktensor_b200 import native
    rng = np.random.default_rng(4)
    if kind == "normal":
        x = (rng.standard_normal(32 * 4099) * 0.05).astype(np.float32)
    elif kind == "uniform":
        x = rng.uniform(-3, 3, 32 * 1000).astype(np.float32)
    else:
        x = np.load(os.path.join(GOLDEN, "ref_kernels.npz"))["qedge_x"]
    want = ref_q4(ref, x)
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(x.size // 32 * 20, dtype=torch.uint8, device="cuda")
    native.call("bt_cuda_quantize_q4_0", xd.data_ptr(), out.data_ptr(), x.size, None)
    got = out.cpu().numpy()
    assert np.array_equal(got, want.view(np.uint8))
    # dequantize: (code - 8) * scale exactly
    deq = torch.empty(x.size, dtype=torch.float32, device="cuda")
    native.call("bt_cuda_dequantize_q4_0", out.data_ptr(), deq.data_ptr(), x.size, None)
    codes, scale = decode_q4(want)
    expect = (codes.astype(np.float32) * scale[:, None]).astype(np.float32).reshape(-1)
    assert np.array_equal(deq.cpu().numpy().view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("M,K", [(16, 256), (4096, 4096), (1000, 11008), (7, 32)])
def test_matvec_q4_vs_reference_arithmetic(cuda, ref, M, K):
    import torch
    from blocktensor_b200 import native
    rng = np.random.default_rng(M + K)
    blocks = ref_q4(ref, (rng.standard_normal(M * K) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    codes, scale = decode_q4(blocks)
    w = codes.reshape(M, K // 32, 32).astype(np.float64) * scale.reshape(M, K // 32, 1)
    want = (w * x.reshape(1, K // 32, 32)).sum(axis=(1, 2))
    mag = np.abs(w * x.reshape(1, K // 32, 32)).sum(axis=(1, 2))
    wd = torch.from_numpy(blocks.view(np.uint8)).cuda()
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    native.call("bt_cuda_matvec_q4_0", wd.data_ptr(), xd.data_ptr(), y.data_ptr(), M, K, None)
    err = np.abs(y.cpu().numpy().astype(np.float64) - want)
    assert (err <= 1e-5 * mag + 1e-30).all(), f"worst relative error {np.max(err / (mag + 1e-30))}"


def test_int4_model_drives_engine(cuda, oracle, ref, tmp_path):
    """A Q4_0 (INT4) model: the CUDA engine repacks its 4-bit blocks and matches the
    reference engine running the same file."""
    from blocktensor_b200 import btmodel
    D, F, L, H, V = 128, 256, 2, 4, 256
    cfg = cuda.model_config(V, D, F, L, H, H, D // H, 64)
    rng = np.random.default_rng(9)
    tensors = [(rng.standard_normal(V * D) * 0.02).astype(np.float32), np.ones(D, np.float32),
               ref_q4(ref, rng.standard_normal(V * D) * 0.05)]
    for _ in range(L):
        tensors += [np.ones(D, np.float32), np.ones(D, np.float32)]
        for r, k in ((D, D), (D, D), (D, D), (D, D), (F, D), (F, D), (D, F)):
            tensors.append(ref_q4(ref, rng.standard_normal(r * k) * 0.05))
    path = str(tmp_path / "q4.btmodel")
    btmodel.write_btmodel(path, cfg, [np.asarray(t).view(np.uint8) for t in tensors], quant_type=btmodel.DT_INT4)
    r = oracle.RefEngine.from_file(ref, path, kv_max_seq=64)
    eng = cuda.TransformerEngine.from_btmodel(path)
    kv = cuda.KVCache(eng, 64)
    tok = 5
    for p in range(20):
        a = eng.forward_single_token(tok, p, kv)
        b = r.forward(tok, p)
        err = np.abs(a.astype(np.float64) - b) / (1.0 + np.abs(b))
        assert err.max() <= 1e-2, f"pos {p}: {err.max()}"
        assert int(np.argmax(a)) == int(np.argmax(b))
        tok = int(np.argmax(b))
    kv.close()
    eng.close()
    r.close()
