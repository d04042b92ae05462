"""GPU: bt_cuda_gemv_q8_units_noalloc, the GEMV entry point for callers that
cannot allocate device memory (an engine with its own up-front memory pool, a
runtime whose allocator must see every byte, a decode loop that must not hit
cudaMalloc's implicit synchronisation).  It keeps its scratch in a fixed device
array inside the library instead of a workspace cudaMalloc'd on first use.

Called through the C ABI and compared with bt_cuda_gemv_q8_units on the same
inputs, on two calls in a row (the second call reuses the array the first one
left behind), within the GEMV tolerance of test_gpu_kernels.py.  The file name
sorts last so that a run stopping at the first failure has run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(t):
    return t.data_ptr()


@pytest.mark.parametrize("M,K", [(4096, 4096), (22016, 4096), (1000, 2816), (33, 288)])
def test_noalloc_matches_allocating_entry_point(cuda, M, K):
    import torch
    from blocktensor_b200 import native

    rng = np.random.default_rng(M + 3 * K)
    w = torch.from_numpy((rng.standard_normal(M * K) * 0.02).astype(np.float32)).cuda()
    blocks = cuda.quantize_q8_0(w)
    units = cuda.pack_q8_units(blocks, M, K)
    xs = [torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda() for _ in range(2)]
    for x in xs:  # two calls in a row, different inputs
        want = torch.empty(M, dtype=torch.float32, device="cuda")
        got = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
        native.call("bt_cuda_gemv_q8_units", _ptr(units), _ptr(x), _ptr(want), M, K, None)
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(units), _ptr(x), _ptr(got), M, K, None)
        torch.cuda.synchronize()
        want_h, got_h = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(got_h).all()
        # the GEMV bar of test_gpu_kernels.py: within 1e-5 of sum |s q x| per row
        mag = float(np.abs(want_h).max()) + 1.0
        np.testing.assert_allclose(got_h, want_h, rtol=1e-5, atol=1e-5 * mag)


def test_noalloc_rejects_oversize(cuda):
    import torch
    from blocktensor_b200 import native

    buf = torch.zeros(64, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(buf), _ptr(buf), _ptr(buf), (1 << 20) + 1, 32, None)
    with pytest.raises(ValueError):
        native.call("bt_cuda_gemv_q8_units_noalloc", _ptr(buf), _ptr(buf), _ptr(buf), 16, 48 * 1024 + 32, None)
