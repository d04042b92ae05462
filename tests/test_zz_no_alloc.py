"""GPU: bt_cuda_gemv_q8_units_noalloc, the GEMV entry point for callers that
cannot allocate device memory (an engine with its own up-front memory pool, a
runtime whose allocator must see every byte, a decode loop that must not hit
cudaMalloc's implicit synchronisation).  It keeps its scratch in a fixed device
array inside the library instead of a workspace cudaMalloc'd on first use.

Called through the C ABI and compared, on two calls in a row (the second call
reuses the array the first one left behind), with bt_cuda_gemv_q8_units on the
same inputs and with the oracle's matvec, within the GEMV bar of
test_gpu_kernels.py.  The file name sorts last so that a run stopping at the
first failure has run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(t):
    return t.data_ptr()


def _mag(blocks, x, M, K):
    """sum_b |s_b| sum_i |q_i x_i| per row: the scale the GEMV's error is measured against."""
    nb = K // 32
    return np.abs(blocks["scale"].reshape(M, nb, 1) * blocks["qs"].reshape(M, nb, 32).astype(np.float64)
                  * np.abs(x.reshape(1, nb, 32))).sum(axis=(1, 2))


def _run_pair(cuda, units, x, M, K):
    import torch
    from blocktensor_b200 import native
    want = torch.empty(M, dtype=torch.float32, device="cuda")
    got = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    native.call("bt_cuda_gemv_q8_units", _ptr(units), _ptr(x), _ptr(want), M, K, None)
    native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(got), M, K, None)
    torch.cuda.synchronize()
    return want.cpu().numpy(), got.cpu().numpy()


@pytest.mark.parametrize("M,K", [(4096, 4096), (22016, 4096), (1000, 2816), (33, 288)])
def test_noalloc_matches_allocating_entry_point_and_oracle(cuda, oracle, M, K):
    import torch

    rng = np.random.default_rng(M + 3 * K)
    blocks = oracle.quantize_q8_0((rng.standard_normal(M * K) * 0.02).astype(np.float32))
    units = cuda.pack_q8_units(torch.from_numpy(blocks.view(np.uint8)).cuda(), M, K)
    for _ in range(2):  # two calls in a row, different inputs
        x = rng.standard_normal(K).astype(np.float32)
        want_h, got_h = _run_pair(cuda, units, torch.from_numpy(x).cuda(), M, K)
        assert np.isfinite(got_h).all()
        # the same kernel on the same inputs: the two entry points agree exactly
        np.testing.assert_array_equal(got_h, want_h)
        # and both are within the GEMV bar of the oracle: 1e-5 of sum |s q x| per row
        ref = oracle.matvec_q8_0(blocks, x, M, K, nthreads=8)
        err = np.abs(got_h.astype(np.float64) - ref)
        mag = _mag(blocks, x, M, K)
        assert (err <= 1e-5 * mag + 1e-30).all(), f"worst relative error {np.max(err / (mag + 1e-30))}"


def test_noalloc_outlier_blocks(cuda, oracle):
    """One block of x 1e4 and one 1e3 times the rest; the even rows do not touch them."""
    import torch
    from test_gpu_kernels import outlier_case

    M, K = 4096, 4096
    blocks, x, ref, mag = outlier_case(oracle, M, K, seed=77)
    units = cuda.pack_q8_units(torch.from_numpy(blocks.view(np.uint8)).cuda(), M, K)
    for _ in range(2):
        want_h, got_h = _run_pair(cuda, units, torch.from_numpy(x).cuda(), M, K)
        np.testing.assert_array_equal(got_h, want_h)
        err = np.abs(got_h.astype(np.float64) - ref)
        assert (err <= 1e-5 * mag + 1e-30).all(), f"worst relative error {np.max(err / (mag + 1e-30))}"


def test_noalloc_takes_no_device_memory(cuda):
    """After the first call (which loads the kernels and looks up the array's device
    address), calls of every size leave the device's free memory unchanged: the
    scratch is the library's fixed array, not an allocation."""
    import torch
    from blocktensor_b200 import native

    sizes = [(33, 288), (4096, 4096), (1 << 20, 32)]
    bufs = []
    for M, K in sizes:
        units = torch.zeros(cuda.unit_bytes(M, K), dtype=torch.uint8, device="cuda")
        x = torch.ones(K, dtype=torch.float32, device="cuda")
        y = torch.empty(M, dtype=torch.float32, device="cuda")
        bufs.append((units, x, y, M, K))
    units, x, y, M, K = bufs[0]
    native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(y), M, K, None)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for units, x, y, M, K in bufs * 2:
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(y), M, K, None)
        torch.cuda.synchronize()
        assert (y == 0).all()  # zero weights: every row is exactly zero
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_oversize(cuda):
    import torch
    from blocktensor_b200 import native

    buf = torch.zeros(64, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(buf), _ptr(buf), _ptr(buf), (1 << 20) + 1, 32, None)
    with pytest.raises(ValueError):
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(buf), _ptr(buf), _ptr(buf), 16, 48384 + 32, None)


def test_noalloc_timeout_is_reported(cuda):
    """A device wait that gave up (injected on the host) is reported as
    BT_ERR_DEVICE_TIMEOUT by the next call, and the call after it is valid again."""
    import torch
    from blocktensor_b200 import native

    M, K = 256, 256
    rng = np.random.default_rng(2)
    w = torch.from_numpy((rng.standard_normal(M * K) * 0.02).astype(np.float32)).cuda()
    units = cuda.pack_q8_units(cuda.quantize_q8_0(w), M, K)
    x = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(y), M, K, None)
    good = y.cpu().numpy()
    native.call("bt_cuda_gemv_inject_timeout", torch.cuda.current_device(), 1)
    with pytest.raises(native.CudaBackendError) as ei:
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(y), M, K, None)
    assert ei.value.code == native.BT_ERR_DEVICE_TIMEOUT
    native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(y), M, K, None)
    assert np.array_equal(y.cpu().numpy(), good)
