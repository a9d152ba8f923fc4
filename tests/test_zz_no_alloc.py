"""sam3b200_mul_mat_noalloc -- the MUL_MAT variant for callers that cannot
allocate device memory while computing (a framework that plans every device
byte in advance, or a latency-bound loop that cannot take cudaMalloc's
synchronisation).  It must give the same result as sam3b200_mul_mat, call
after call, although every call reuses the same fixed scratch array.

Both entry points quantise the same activations and run the same exact
kernels, so their outputs are compared bit for bit.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _weight(oracle, K, N, seed, qtype=8):
    rng = np.random.default_rng(seed)
    wq = oracle.quantize_weights(qtype, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    bias = rng.normal(0, 0.02, size=(N,)).astype(np.float32)
    return wq, bias


@pytest.mark.parametrize("qtype", [8, 2])  # Q8_0, Q4_0
@pytest.mark.parametrize("Ms,K,N", [((300, 300), 1024, 512), ((5184, 5184), 1024, 1024), ((40, 40), 256, 96),
                                    ((5184, 200), 4736, 256), ((700, 33), 512, 128)])
def test_noalloc_matches_mul_mat_two_calls_in_a_row(oracle, backend, qtype, Ms, K, N):
    """Two calls in a row (the second with the same or a smaller M, so scratch
    left over from the first call would show), each bit-identical to
    sam3b200_mul_mat on the same inputs."""
    wq, bias = _weight(oracle, K, N, seed=sum(Ms) + K + N + qtype, qtype=qtype)
    w = backend.weight(qtype, wq, K, N)
    bd = backend.upload(bias)
    rng = np.random.default_rng(K + N)
    for M in Ms:
        x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
        xd = backend.upload(x)
        y_ref, y_na = backend.alloc(M * N * 4), backend.alloc(M * N * 4)
        backend.mul_mat(w, xd, M, y_ref, bias=bd)
        backend.mul_mat_noalloc(w, xd, M, y_na, bias=bd)
        backend.synchronize()
        assert np.array_equal(y_na.get((M, N), np.float32), y_ref.get((M, N), np.float32))
    w.free()


def test_noalloc_rejects_shapes_beyond_its_scratch(oracle, b200, backend):
    # 10200 x 4736: 48.3 MB of codes + 3.1 MB of scale records > 48 MiB; 9800 x 4736 fits
    K, N = 4736, 32
    wq = oracle.quantize_weights(8, np.zeros((N, K), np.float32))
    w = backend.weight(8, wq, K, N)
    M = 10200
    x, y = backend.upload(np.zeros((M, K), np.float32)), backend.alloc(M * N * 4)
    with pytest.raises(b200.B200Error, match="scratch"):
        backend.mul_mat_noalloc(w, x, M, y)
    backend.mul_mat_noalloc(w, x, 9800, y)  # within the array: accepted
    backend.synchronize()
    w.free()


def test_noalloc_refuses_dense_weights(b200, backend):
    """F16 weights have no quantised path: the entry point refuses them with an error."""
    K, N, M = 64, 32, 8
    w = backend.weight(b200.TYPE_F16, np.zeros((N, K), np.float16).view(np.uint8), K, N)
    x, y = backend.alloc(M * K * 4), backend.alloc(M * N * 4)
    with pytest.raises(b200.B200Error, match="not supported"):
        backend.mul_mat_noalloc(w, x, M, y)
    w.free()
