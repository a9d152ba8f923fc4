"""Failure detection on the GPU without a GPU fault: every mbarrier wait of the
tensor-core pipelines is bounded; when a phase never completes the kernel gives
up, records a code in the backend's error word and returns, and
sam3b200_backend_synchronize reports FAILED (the reference's callers treat a
non-success ggml_status as a failed compute, sam3.cpp:1019-1030).  Here a wait
on a barrier that nothing arrives on runs out after 2 ms."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_synchronize_fails(b200, backend, oracle):
    backend.synchronize()
    backend.debug_wait_timeout(2_000_000)
    with pytest.raises(b200.B200Error, match="timed out"):
        backend.synchronize()
    # the error is reported once, and the context stays usable: a MUL_MAT afterwards is exact
    backend.synchronize()
    rng = np.random.default_rng(4)
    M, K, N = 128, 256, 128
    wq = oracle.quantize_weights(8, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    w = backend.weight(8, wq, K, N)
    y = backend.alloc(M * N * 4)
    backend.mul_mat(w, backend.upload(x), M, y)
    backend.synchronize()
    assert np.array_equal(y.get((M, N), np.float32), oracle.mul_mat(8, wq, K, N, x))
    w.free()


def test_wait_limit_is_bounded(b200, backend):
    with pytest.raises(b200.B200Error, match="limit"):
        backend.debug_wait_timeout(5_000_000_000)
