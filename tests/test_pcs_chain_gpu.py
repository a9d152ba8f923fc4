"""The text-prompt (PCS) detector chained on the device as sam3_segment_pcs wires it
(sam3.cpp:12800-12860): ViT with both necks -> text encoder -> fusion encoder -> DETR decoder ->
segmentation head, every hand-off a device pointer through the *_run_device entries (no host round
trip).  Each stage is checked against its CPU oracle on the device intermediates it consumed, so the
test pins the hand-offs (pointers, offsets, layouts) rather than compounding chaotic random-weight
error across stages."""
import ctypes

import numpy as np
import pytest

from conftest import rel_err
from test_ddec_gpu import make_ddec_tensors
from test_fenc_gpu import make_fenc_tensors
from test_loader_gpu import text_tensors
from test_seghead_gpu import make_seg_tensors

pytestmark = pytest.mark.gpu

D = 256


def out_ptr(fn, h, *idx, with_ne=False):
    """Device pointer returned by one of the runners' *_output entries."""
    p = ctypes.c_void_p()
    args = list(idx) + [ctypes.byref(p)]
    if with_ne:
        args.append((ctypes.c_int64 * 4)())
    assert fn(h, *args) == 0
    return p.value


def host(b200, backend, ptr, shape):
    out = np.empty(shape, np.float32)
    assert b200.lib().sam3b200_tensor_get(backend.h, ptr, out.ctypes.data, 0, out.nbytes) == 0
    return out


def test_pcs_chain_on_device(oracle, b200, backend, model):
    import ddec_oracle
    import fenc_oracle
    import seghead_oracle
    lib = b200.lib()
    hp = model.SAM3_VIT_TEST
    G = hp["img"] // hp["patch"]  # 48
    N, L, NQ = G * G, 16, 50
    vit = backend.vit(hp)
    txt = backend.text_encoder(dict(width=256, heads=4, layers=2, ctx_len=L, vocab=1000, out_dim=D))
    fe = backend.fusion_encoder(dict(d_model=D, heads=8, layers=6, ffn_dim=2048, max_tokens=N, max_prompt=L))
    ddhp = dict(d_model=D, heads=8, layers=2, ffn_dim=2048, num_queries=NQ, feat=G)
    dd = backend.detr_decoder(dict(ddhp, max_prompt=L))
    sh = backend.seg_head(dict(d_model=D, heads=8, feat=G, max_queries=NQ, max_prompt=L))
    try:
        vit.load({**model.random_vit_weights(hp, seed=1), **model.random_det_neck_weights(hp, seed=2)})
        txt.load(text_tensors(oracle))
        fe_gpu, fe_ref = make_fenc_tensors(oracle, 2, 3)
        fe.load(fe_gpu)
        dd_gpu, dd_ref = make_ddec_tensors(oracle, ddhp, 2, 4)
        dd.load(dd_gpu)
        sh_gpu, sh_ref = make_seg_tensors(oracle, 2, 5)
        sh.load(sh_gpu)

        rng = np.random.default_rng(11)
        vit.encode(rng.integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8))
        ids = np.array([406, 320, 929, 7], np.int32)
        txt.encode(ids)
        pe = rng.normal(0, 1, size=(N, D)).astype(np.float32)
        bias = np.where(np.arange(L) < len(ids), 0.0, -1.0e9).astype(np.float32)
        valid = np.where(np.arange(L) < len(ids), L / len(ids), 0.0).astype(np.float32)
        pe_d, bias_d, valid_d = backend.upload(pe), backend.upload(bias), backend.upload(valid)

        neck = [out_ptr(lib.sam3b200_vit_output_det, vit.h, i, with_ne=True) for i in range(3)]
        text_p = ctypes.c_void_p()
        assert lib.sam3b200_text_output(txt.h, ctypes.byref(text_p), (ctypes.c_int64 * 2)()) == 0
        text_d = text_p.value

        assert lib.sam3b200_fenc_run_device(fe.h, neck[2], text_d, pe_d.ptr, bias_d.ptr, N, L) == 0
        cond = out_ptr(lib.sam3b200_fenc_output, fe.h)
        assert lib.sam3b200_ddec_run_device(dd.h, cond, pe_d.ptr, text_d, bias_d.ptr, valid_d.ptr, L) == 0
        q_p, b_p, s_p, p_p = (ctypes.c_void_p() for _ in range(4))
        assert lib.sam3b200_ddec_outputs(dd.h, ctypes.byref(q_p), ctypes.byref(b_p), ctypes.byref(s_p),
                                         ctypes.byref(p_p)) == 0
        # the object queries follow the presence row
        assert lib.sam3b200_seg_run_device(sh.h, cond, neck[0], neck[1], q_p.value + D * 4, NQ, text_d, bias_d.ptr,
                                           L) == 0
        backend.synchronize()
        masks = host(b200, backend, out_ptr(lib.sam3b200_seg_output, sh.h), (NQ, 16 * N))

        # each stage against its oracle on the device intermediates it consumed
        neck_h = [host(b200, backend, neck[i], (s * s, D)) for i, s in enumerate((4 * G, 2 * G, G))]
        text_h = host(b200, backend, text_d, (L, D))
        cond_h = host(b200, backend, cond, (N, D))
        want = fenc_oracle.run(fe_ref, 6, 8, neck_h[2], text_h, pe, bias)
        spread = rel_err(fenc_oracle.run(fe_ref, 6, 8, neck_h[2], text_h, pe, bias, np.float32), want)
        assert rel_err(cond_h, want) <= max(1e-2, 2 * spread)
        q_h = host(b200, backend, q_p.value, (NQ + 1, D))
        boxes_h = host(b200, backend, b_p.value, (NQ, 4))
        ref = ddec_oracle.run(ddhp, dd_ref, cond_h, pe, text_h, bias, valid)
        other = ddec_oracle.run(ddhp, dd_ref, cond_h, pe, text_h, bias, valid, np.float32)
        for key, got in (("queries", q_h), ("boxes", boxes_h)):
            assert rel_err(got, ref[key]) <= max(1e-2, 2 * rel_err(other[key], ref[key])), key
        want = seghead_oracle.run(sh_ref, G, cond_h, neck_h[0], neck_h[1], q_h[1:], text_h, bias)
        assert rel_err(masks, want) <= 1e-2
    finally:
        for r in (vit, txt, fe, dd, sh):
            r.free()
