"""One ViT block through the B200 ggml backend object, the way sam3.cpp drives a ggml backend:
the graph built node for node as sam3_vit_block_forward builds it (sam3.cpp:3714-3805), weights
placed with ggml_backend_alloc_ctx_tensors + ggml_backend_tensor_set, the graph allocated with
ggml_gallocr and run with ggml_backend_graph_compute.  The result matches the CPU oracle's block
(the same graph restated in C) at the north-star bound, max |d| / max |ref| <= 1e-2."""
import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _run(ggml_caller, hp, tensors, idx, x):
    E, heads, mlp, window = hp["embed"], hp["heads"], hp["mlp"], hp["window"]
    G = hp["img"] // hp["patch"]
    glob = idx in hp["global_idx"]
    pre = f"vit.blocks.{idx}."
    hpv = (ctypes.c_int32 * 6)(E, heads, G, 0 if glob else window, hp["wtype"], mlp)
    keep = []

    def ptr(name):
        a = np.ascontiguousarray(tensors[pre + name][1])
        keep.append(a)
        return a.ctypes.data_as(ctypes.c_void_p)

    weights = (ctypes.c_void_p * 4)(*[ptr(n + ".weight") for n in ("attn.qkv", "attn.proj", "mlp.lin1", "mlp.lin2")])
    vecs = (ctypes.c_void_p * 8)(*[ptr(n) for n in ("attn.qkv.bias", "attn.proj.bias", "mlp.lin1.bias",
                                                    "mlp.lin2.bias", "norm1.weight", "norm1.bias", "norm2.weight",
                                                    "norm2.bias")])
    freqs = ptr("attn.freqs_cis")
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    n = ctypes.c_int32()
    fn = ggml_caller.vit_block_graph_run
    fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    st = fn(0, ctypes.addressof(hpv), ctypes.addressof(weights), ctypes.addressof(vecs), freqs,
            x.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p), ctypes.addressof(n))
    assert st == 0, f"ggml_backend_graph_compute returned {st}"
    return out, n.value


@pytest.mark.parametrize("idx", [0, 1])  # block 0 windowed, block 1 global
def test_vit_block_graph_through_the_backend(model, oracle, ggml_caller, idx):
    hp = model.SAM3_VIT_TEST
    tensors = model.random_vit_weights(hp, seed=1)
    ov = oracle.OracleVit(hp, tensors)
    x = np.random.default_rng(40 + idx).standard_normal((ov.G ** 2, hp["embed"]), dtype=np.float32)
    got, nodes = _run(ggml_caller, hp, tensors, idx, x)
    assert nodes == (67 if idx in hp["global_idx"] else 69)
    err = rel_err(got, ov.block(idx, x))
    assert err <= 1e-2, err


@pytest.mark.parametrize("idx", [0, 7])
def test_full_size_vit_block_graph_through_the_backend(model, oracle, ggml_caller, idx):
    """SAM3 ViT-32 geometry (72 x 72 tokens, E = 1024, 16 heads, MLP 4736, Q8_0): a windowed and a
    global block."""
    hp = dict(model.SAM3_VIT, depth=8, global_idx=(7,))
    tensors = model.random_vit_weights(hp, seed=2)
    ov = oracle.OracleVit(hp, tensors)
    x = np.random.default_rng(50 + idx).standard_normal((ov.G ** 2, hp["embed"]), dtype=np.float32)
    got, _ = _run(ggml_caller, hp, tensors, idx, x)
    err = rel_err(got, ov.block(idx, x))
    assert err <= 1e-2, err
