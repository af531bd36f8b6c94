"""CPU-side checks of the C ABI: the library loads without a GPU, exports every function
include/dcgpu.h declares, and its pure-host helpers agree with the ggml geometry."""
import ctypes

import pytest

from densecore_b200 import _lib, ggml_types as T
from oracle import oracle as O


def test_library_exports_every_header_symbol():
    L = _lib.load()
    declared = _lib.header_symbols()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/dcgpu.h but not exported"
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signature table out of sync with header"


@pytest.mark.parametrize("t,k", [(T.Q8_0, 4096), (T.Q4_K, 14336), (T.Q6_K, 2560), (T.Q8_K, 4096),
                                 (T.F16, 128), (T.F32, 7)])
def test_row_size_matches_ggml(t, k):
    assert _lib.load().dcg_row_size(t, k) == T.row_size(t, k)
    if t in O.BLOCK:
        assert T.row_size(t, k) == O.row_size(t, k)


def test_host_errors_without_gpu():
    L = _lib.load()
    # argument checks run before any CUDA call
    assert L.dcg_quantize_row_q8_0(None, None, 1, 32, None) == -1
    assert L.dcg_mul_mat(99, None, 1, 256, None, 1, None, None, 0, None) == -1
    assert b"unsupported" in L.dcg_last_error()
    assert L.dcg_packed_weight_size(T.Q4_K, 10, 512) == 10 * 2 * 144 + (256 - (2880 % 256)) % 256
    h = ctypes.c_void_p()
    assert L.dcg_ctx_create(0, ctypes.byref(h)) != 0 or h.value  # no device here: error code
