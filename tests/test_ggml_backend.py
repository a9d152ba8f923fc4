"""The B200 ggml backend object (sam3.cpp_b200/ggml/ggml-b200.cpp) from a ggml caller, on the host:
the ViT block graph built node for node as sam3_vit_block_forward builds it (sam3.cpp:3714-3805)
is accepted node by node by the device's supports_op -- at the reduced test size and at the
SAM3 ViT-32 size, windowed and global, Q8_0 and Q4_0 weights."""
import ctypes

import pytest

Q4_0, Q8_0 = 2, 8


@pytest.mark.parametrize("hp", [(256, 4, 48, 24, Q8_0, 1024), (256, 4, 48, 0, Q8_0, 1024),
                                (1024, 16, 72, 24, Q8_0, 4736), (1024, 16, 72, 0, Q4_0, 4736)])
def test_every_node_of_the_vit_block_graph_is_supported(ggml_caller, hp):
    h = (ctypes.c_int32 * 6)(*hp)
    n, ok = ctypes.c_int32(), ctypes.c_int32()
    first = ctypes.create_string_buffer(64)
    assert ggml_caller.vit_block_graph_check(h, ctypes.byref(n), ctypes.byref(ok), first, 64) == 0
    # LN (3 nodes) x 2, the qkv path, RoPE on q and k, attention, proj, window part / unpart, MLP
    assert n.value == (69 if hp[3] else 67)
    assert ok.value == n.value, first.value
