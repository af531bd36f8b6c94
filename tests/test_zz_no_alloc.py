"""dcg_mul_mat_noalloc -- the matmul entry point that allocates nothing.

It exists for callers that cannot allocate device memory where they run the matmul (a ggml
custom-op callback inside the compute thread pool, a plugin host that forbids allocation after
start-up).  Through the C ABI, two calls in a row (different inputs, so stale contents of the
shared fixed buffer would show) must agree with dcg_mul_mat, which takes caller scratch, within
the tolerance the other matmul tests use.  Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = 1e-5


# m = 20 runs three 8-row chunks; m = 60 at k = 14336 is the largest Q8_K activation that fits
@pytest.mark.parametrize("wt,n,k,m", [(12, 4096, 14336, 1), (8, 1024, 4096, 8), (14, 512, 2560, 3),
                                      (12, 768, 4096, 20), (12, 256, 14336, 60)])
def test_noalloc_matches_mul_mat_twice(wt, n, k, m):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200 import _lib, ops
    L = _lib.load()
    torch.manual_seed(n + k + m)
    w = ops.QuantWeight.from_float(torch.randn(n, k, device="cuda") * 0.02, wt)
    stream = torch.cuda.current_stream().cuda_stream
    from oracle import oracle as O
    wd = torch.from_numpy(O.dequantize(w.to_ggml().cpu().numpy(), wt, k)).double().cuda()
    for call in range(2):
        x = torch.randn(m, k, device="cuda") * (1 + call)
        y_ref = ops.mul_mat(w, x)
        y = torch.full((m, n), float("nan"), device="cuda")
        rc = L.dcg_mul_mat_noalloc(wt, w.packed.data_ptr(), n, k, x.data_ptr(), m, y.data_ptr(),
                                   stream)
        assert rc == 0, L.dcg_last_error()
        torch.cuda.synchronize()
        bound = x.abs().double() @ wd.abs().T + 1e-30   # sum_k |x_k w_k| (unquantized x, upper-ish)
        err = (y.double() - y_ref.double()).abs()
        assert torch.isfinite(y).all()
        assert bool((err <= RTOL * bound).all()), float((err / bound).max())


def test_noalloc_limit_is_exact():
    """m = 60 fits the fixed buffer at k = 14336 for a Q4_K weight (Q8_K activation); m = 61 does not."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200 import _lib
    L = _lib.load()
    k, n = 14336, 256
    assert L.dcg_act_size(15, 60, k) <= 1 << 20 < L.dcg_act_size(15, 61, k)
    w = torch.zeros(L.dcg_packed_weight_size(12, n, k), dtype=torch.uint8, device="cuda")
    x = torch.zeros(61, k, device="cuda")
    y = torch.zeros(61, n, device="cuda")
    assert L.dcg_mul_mat_noalloc(12, w.data_ptr(), n, k, x.data_ptr(), 60, y.data_ptr(), None) == 0
    rc = L.dcg_mul_mat_noalloc(12, w.data_ptr(), n, k, x.data_ptr(), 61, y.data_ptr(), None)
    assert rc == -1 and b"no-allocation buffer" in L.dcg_last_error()
    torch.cuda.synchronize()


def test_noalloc_rejects_oversize():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from densecore_b200 import _lib
    L = _lib.load()
    x = torch.zeros(256, 8192, device="cuda")
    y = torch.zeros(256, 256, device="cuda")
    w = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    rc = L.dcg_mul_mat_noalloc(12, w.data_ptr(), 256, 8192, x.data_ptr(), 256, y.data_ptr(), None)
    assert rc == -1 and b"no-allocation buffer" in L.dcg_last_error()
    code = ctypes.c_int(-1)
    assert L.dcg_device_error(ctypes.byref(code), 0) == 0 and code.value == 0
