"""CPU checks of the C ABI library: it loads, exports every symbol the
header declares, and fails cleanly (no crash, an error message) without a
GPU."""
import ctypes

import pytest


def test_library_exports_every_declared_symbol(b200):
    L = b200.lib()
    names = b200.exported_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n


def test_backend_init_without_gpu_fails_cleanly(b200):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = b200.lib().sam3b200_backend_init(0)
    assert not h
    assert b200.last_error()


def test_null_handles_are_rejected(b200):
    L = b200.lib()
    assert L.sam3b200_backend_synchronize(None) == b200.STATUS_FAILED
    assert L.sam3b200_tensor_set(None, None, None, 0, 0) == b200.STATUS_FAILED
    assert L.sam3b200_mul_mat(None, None, None, 0, 0, None, None, 0) == b200.STATUS_FAILED
    assert not L.sam3b200_weight_upload(None, 8, None, 32, 1)


def test_mul_mat_refuses_an_unaligned_bias(b200):
    """The tensor-core epilogue reads the bias four floats at a time: a bias view that is not 16-byte
    aligned is refused on the host instead of faulting on the device."""
    L = b200.lib()
    for fn in (L.sam3b200_mul_mat, L.sam3b200_mul_mat_noalloc):
        assert fn(None, None, None, 0, 0, (1 << 20) + 4, None, 0) == b200.STATUS_FAILED
        assert "16-byte aligned" in b200.last_error()
