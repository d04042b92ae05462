"""GPU parity of the standalone kernels against the oracle and the reference goldens.

Bars: quantize / dequantize / repack bit-exact; matvec and GEMV within fp32
reordering tolerance (|gpu - ref| <= 1e-4 * (1 + |ref|) relative to the row's
magnitude); rmsnorm / rope / softmax / silu at the reference's own 1e-4 form
(tests/test_stage3_kernels.cpp:45-47); argmax exact with first-max-wins ties.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    return torch


@pytest.fixture(scope="module")
def gk():
    return np.load(os.path.join(GOLDEN, "ref_kernels.npz"))


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def approx_ref(gpu, ref, tol):
    """The reference tests' comparison: |a - b| <= tol * (1 + |a|)."""
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(gpu - ref) > tol * (1.0 + np.abs(ref))
    assert not bad.any(), f"{bad.sum()} mismatches, worst {np.abs(gpu - ref).max()}"


@pytest.mark.parametrize("name", ["qn", "qu", "qedge", "mv_raw"])
def test_quantize_bit_exact_golden(cuda, torch_mod, gk, name):
    x = gk[f"{name}_x"] if name != "mv_raw" else gk["mv_raw"]
    want = gk[f"{name}_blocks"] if name != "mv_raw" else gk["mv_blocks"]
    got = cuda.quantize_q8_0(dev(torch_mod, x)).cpu().numpy()
    assert np.array_equal(got, want)
    if name != "mv_raw":
        deq = cuda.dequantize_q8_0(dev(torch_mod, want)).cpu().numpy()
        assert np.array_equal(deq.view(np.uint32), gk[f"{name}_deq"].view(np.uint32))


@pytest.mark.parametrize("n_blocks,scale", [(1, 1.0), (7, 0.02), (4099, 0.02), (65537, 5.0)])
def test_quantize_bit_exact_oracle(cuda, oracle, torch_mod, n_blocks, scale):
    rng = np.random.default_rng(n_blocks)
    x = (rng.standard_normal(32 * n_blocks) * scale).astype(np.float32)
    got = cuda.quantize_q8_0(dev(torch_mod, x)).cpu().numpy()
    assert np.array_equal(got, oracle.quantize_q8_0(x).view(np.uint8))


def test_quantize_errors(cuda, torch_mod):
    with pytest.raises(ValueError):
        cuda.quantize_q8_0(torch_mod.zeros(33, device="cuda"))
    # empty input is a no-op
    assert cuda.quantize_q8_0(torch_mod.zeros(0, device="cuda")).numel() == 0


def test_repack(cuda, oracle, torch_mod):
    rng = np.random.default_rng(3)
    M, K = 45, 32 * 7
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.1).astype(np.float32))
    qs, sc = cuda.repack_q8_0(dev(torch_mod, b.view(np.uint8)), M, K)
    assert np.array_equal(qs.cpu().numpy().reshape(M, K // 32, 32), b["qs"].reshape(M, K // 32, 32))
    assert np.array_equal(sc.cpu().numpy().ravel(), b["scale"])


def test_matvec_golden(cuda, torch_mod, gk):
    """test_stage4_quant.cpp:47-94 (M=16, N=256) at the test's own 1e-2 form, and at 1e-5."""
    y = cuda.matvec_q8_0(dev(torch_mod, gk["mv_blocks"]), dev(torch_mod, gk["mv_x"]), 16, 256).cpu().numpy()
    approx_ref(y, gk["mv_y"], 1e-2)
    approx_ref(y, gk["mv_y"], 1e-5)


@pytest.mark.parametrize("M,K", [(16, 256), (288, 288), (864, 288), (4096, 4096), (1000, 11008), (7, 32)])
def test_matvec_aos_vs_oracle(cuda, oracle, torch_mod, M, K):
    rng = np.random.default_rng(M + K)
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    want = oracle.matvec_q8_0(b, x, M, K, nthreads=8)
    got = cuda.matvec_q8_0(dev(torch_mod, b.view(np.uint8)), dev(torch_mod, x), M, K).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-5 * (1 + float(np.abs(want).max())))


def gemv_case(oracle, M, K, B, seed):
    """The GEMV microbenchmark distribution: int8 uniform [-127,127], scales U(0.001,0.02), x N(0,1)."""
    q = oracle.gen_int8(seed, 0xA000, M * K).reshape(M, K)
    s = oracle.gen_uniform(seed, 0xA001, M * K // 32, 0.001, 0.02).reshape(M, K // 32)
    x = oracle.gen_normal(seed, 0xA002, B * K, 1.0).reshape(B, K)
    blocks = np.zeros(M * K // 32, oracle.Q8_DTYPE)
    blocks["qs"] = q.reshape(-1, 32)
    blocks["scale"] = s.ravel()
    want = np.stack([oracle.matvec_q8_0(blocks, x[b], M, K, nthreads=8) for b in range(B)])
    return q, s, x, want


@pytest.mark.parametrize("B", [1, 2, 3, 4, 8, 16])
@pytest.mark.parametrize("M,K", [(4096, 4096), (300, 11008), (33, 288)])
def test_gemv_q8_vs_oracle(cuda, oracle, torch_mod, M, K, B):
    q, s, x, want = gemv_case(oracle, M, K, B, seed=M + B)
    got = cuda.gemv_q8(dev(torch_mod, q), dev(torch_mod, s), dev(torch_mod, x)).cpu().numpy()
    # error budget of a K-term fp32 sum in a different order
    np.testing.assert_allclose(got, want, rtol=2e-4, atol=2e-5 * np.sqrt(K) * 0.02 * 127)


def test_rmsnorm_rope_softmax_silu_golden(cuda, torch_mod, gk):
    t = torch_mod
    approx_ref(cuda.rmsnorm(dev(t, gk["rms_x"]), dev(t, gk["rms_w"]), 4, 512, 1e-5).cpu().numpy(), gk["rms_y"], 1e-4)
    for pos in (0, 7, 300):
        got = cuda.rope(dev(t, gk["rope_x"]), 2, 4, 64, pos).cpu().numpy()
        approx_ref(got, gk[f"rope_y_pos{pos}"], 1e-4)
    approx_ref(cuda.softmax(dev(t, gk["softmax_x"]), 4, 256).cpu().numpy(), gk["softmax_y"], 1e-4)
    approx_ref(cuda.silu(dev(t, gk["silu_x"])).cpu().numpy(), gk["silu_y"], 1e-4)


def test_argmax(cuda, torch_mod, gk):
    t = torch_mod
    assert cuda.argmax(dev(t, gk["greedy_logits"])) == int(gk["greedy_id"]) == 3
    x = np.full(100003, -5.0, np.float32)
    x[[17, 5000, 99999]] = 2.0
    assert cuda.argmax(dev(t, x)) == 17          # first maximum wins (std::max_element)
    x = np.full(32000, -np.inf, np.float32)
    assert cuda.argmax(dev(t, x)) == 0
    rng = np.random.default_rng(9)
    y = rng.standard_normal(128256).astype(np.float32)
    assert cuda.argmax(dev(t, y)) == int(np.argmax(y))


def test_launch_counter_moves(cuda, torch_mod):
    before = cuda.launch_count()
    cuda.silu(torch_mod.ones(64, device="cuda"))
    torch_mod.cuda.synchronize()
    assert cuda.launch_count() == before + 1


@pytest.mark.parametrize("M,K", [(4096, 4096), (22016, 4096), (4096, 11008), (32000, 4096), (33, 288),
                                 (864, 288), (100, 64), (1000, 2816), (5, 32)])
def test_gemv_units_vs_oracle(cuda, oracle, torch_mod, M, K):
    """Tensor-core unit-layout GEMV (the engine's) against the reference matvec arithmetic."""
    rng = np.random.default_rng(M * 7 + K)
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    want = oracle.matvec_q8_0(b, x, M, K, nthreads=8)
    units = cuda.pack_q8_units(dev(torch_mod, b.view(np.uint8)), M, K)
    got = cuda.gemv_q8_units(units, dev(torch_mod, x), M, K).cpu().numpy()
    # |sum_b s_b sum_i q_i x_i| bound: the error budget is relative to sum |s q x|
    mag = np.abs(b["scale"].reshape(M, K // 32, 1) * b["qs"].reshape(M, K // 32, 32).astype(np.float64)
                 * np.abs(x.reshape(1, K // 32, 32))).sum(axis=(1, 2))
    err = np.abs(got.astype(np.float64) - want)
    assert (err <= 1e-5 * mag + 1e-30).all(), f"worst relative error {np.max(err / (mag + 1e-30))}"


def outlier_case(oracle, M, K, seed):
    """x N(0,1) with one block scaled by 1e4 and another by 1e3; the weights of those two
    blocks are zero in the even rows, so the even rows' true sums are made of the
    ordinary blocks only and an error proportional to the outliers would show there."""
    rng = np.random.default_rng(seed)
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    x = rng.standard_normal(K).astype(np.float32)
    nb = K // 32
    big, mid = nb // 3, (2 * nb) // 3
    x[32 * big:32 * big + 32] *= 1e4
    x[32 * mid:32 * mid + 32] *= 1e3
    qs = b["qs"].reshape(M, nb, 32)
    qs[0::2, big] = 0
    qs[0::2, mid] = 0
    want = oracle.matvec_q8_0(b, x, M, K, nthreads=8)
    mag = np.abs(b["scale"].reshape(M, nb, 1) * qs.astype(np.float64) * np.abs(x.reshape(1, nb, 32))).sum(axis=(1, 2))
    return b, x, want, mag


@pytest.mark.parametrize("M,K", [(4096, 4096), (1000, 11008)])
def test_gemv_units_outlier_blocks(cuda, oracle, torch_mod, M, K):
    """Outlier activations: every block keeps 22 bits relative to its own max, so rows that
    do not touch the outlier blocks stay within the GEMV bar of their own magnitude."""
    b, x, want, mag = outlier_case(oracle, M, K, seed=M + K)
    units = cuda.pack_q8_units(dev(torch_mod, b.view(np.uint8)), M, K)
    got = cuda.gemv_q8_units(units, dev(torch_mod, x), M, K).cpu().numpy()
    err = np.abs(got.astype(np.float64) - want)
    assert (err <= 1e-5 * mag + 1e-30).all(), f"worst relative error {np.max(err / (mag + 1e-30))}"


def test_gemv_units_timeout_is_reported(cuda, torch_mod):
    """A device wait that gave up (injected on the host) turns into BT_ERR_DEVICE_TIMEOUT
    on the next call, and the call after it is valid again."""
    from blocktensor_b200 import native
    M, K = 256, 256
    rng = np.random.default_rng(1)
    w = dev(torch_mod, (rng.standard_normal(M * K) * 0.02).astype(np.float32))
    units = cuda.pack_q8_units(cuda.quantize_q8_0(w), M, K)
    x = dev(torch_mod, rng.standard_normal(K).astype(np.float32))
    good = cuda.gemv_q8_units(units, x, M, K).cpu().numpy()
    native.call("bt_cuda_gemv_inject_timeout", torch_mod.cuda.current_device(), 0)
    with pytest.raises(native.CudaBackendError) as ei:
        cuda.gemv_q8_units(units, x, M, K)
    assert ei.value.code == native.BT_ERR_DEVICE_TIMEOUT
    assert np.array_equal(cuda.gemv_q8_units(units, x, M, K).cpu().numpy(), good)


def test_gemv_units_deterministic_and_repeatable(cuda, oracle, torch_mod):
    M, K = 4096, 4096
    rng = np.random.default_rng(5)
    b = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    units = cuda.pack_q8_units(dev(torch_mod, b.view(np.uint8)), M, K)
    x = dev(torch_mod, rng.standard_normal(K).astype(np.float32))
    a = cuda.gemv_q8_units(units, x, M, K).cpu().numpy()
    for _ in range(3):
        assert np.array_equal(cuda.gemv_q8_units(units, x, M, K).cpu().numpy(), a)
    # zero vector -> exact zeros; scaling x by 2 doubles y exactly (power-of-two invariance)
    z = cuda.gemv_q8_units(units, torch_mod.zeros(K, device="cuda"), M, K).cpu().numpy()
    assert (z == 0).all()
    a2 = cuda.gemv_q8_units(units, x * 2, M, K).cpu().numpy()
    assert np.array_equal(a2, a * 2)
