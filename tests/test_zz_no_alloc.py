"""sam3b200_mul_mat_noalloc -- the MUL_MAT variant for callers that cannot
allocate device memory while computing (a framework that plans every device
byte in advance, or a latency-bound loop that cannot take cudaMalloc's
synchronisation).  It must give the same result as sam3b200_mul_mat, call
after call, although every call reuses the same fixed scratch array.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _weight_and_inputs(oracle, M, K, N, seed):
    rng = np.random.default_rng(seed)
    wq = oracle.quantize_weights(8, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    xs = [rng.normal(0, 1, size=(M, K)).astype(np.float32) for _ in range(2)]
    bias = rng.normal(0, 0.02, size=(N,)).astype(np.float32)
    return wq, xs, bias


@pytest.mark.parametrize("M,K,N", [(300, 1024, 512), (5184, 1024, 1024), (40, 256, 96)])
def test_noalloc_matches_mul_mat_two_calls_in_a_row(oracle, backend, M, K, N):
    wq, xs, bias = _weight_and_inputs(oracle, M, K, N, seed=M + K + N)
    w = backend.weight(8, wq, K, N)
    bd = backend.upload(bias)
    y_ref, y_na = backend.alloc(M * N * 4), backend.alloc(M * N * 4)
    for x in xs:  # two calls in a row: the second must not see the first's scratch
        xd = backend.upload(x)
        backend.mul_mat(w, xd, M, y_ref, bias=bd)
        backend.mul_mat_noalloc(w, xd, M, y_na, bias=bd)
        backend.synchronize()
        ref = y_ref.get((M, N), np.float32)
        got = y_na.get((M, N), np.float32)
        assert rel_err(got, ref) <= TOL
    w.free()


def test_noalloc_rejects_shapes_beyond_its_scratch(oracle, b200, backend):
    K, N, M = 4736, 32, 12000  # 12000 x 4736 codes alone are ~57 MB > 48 MiB
    wq = oracle.quantize_weights(8, np.zeros((N, K), np.float32))
    w = backend.weight(8, wq, K, N)
    x, y = backend.alloc(M * K * 4), backend.alloc(M * N * 4)
    with pytest.raises(b200.B200Error, match="scratch"):
        backend.mul_mat_noalloc(w, x, M, y)
    w.free()
