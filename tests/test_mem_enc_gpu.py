"""Tracker memory encoder (sam3.cpp:11510-11615) through the C ABI against the CPU oracle
(oracle/mem_enc_oracle.py), for Q8_0 files (F32 convolution kernels, Q8_0 fuser MLP) and F16 files
(F16 everywhere the weight-type rule allows it, sam3.cpp:1762-1786)."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

D, MD, FD = 256, 64, 1024
DS = (1, 4, 16, 64, 256)


def make_mem_enc_tensors(oracle, ftype=8, seed=0):
    """ftype 8: Q8_0 file (convolution kernels F32, d0 % 32 != 0); ftype 1: F16 file."""
    rng = np.random.default_rng(seed)
    gpu, ref = {}, {}
    ct = 1 if ftype == 1 else 0

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name], ref[name] = (0, arr, arr.shape[::-1]), arr

    def conv(name, oc, ic, k, std):
        w = rng.normal(0, std, size=(oc, ic, k, k)).astype(np.float32)
        if ct == 1:
            w16 = w.astype(np.float16)
            gpu[name], ref[name] = (1, w16, (k, k, ic, oc)), (1, w16.astype(np.float32))
        else:
            gpu[name], ref[name] = (0, w, (k, k, ic, oc)), (0, w)

    def lin(name, K, N):
        w = rng.normal(0, 1.0 / np.sqrt(K), size=(N, K)).astype(np.float32)
        if ftype == 1:
            w16 = w.astype(np.float16)
            gpu[name], ref[name] = (1, w16, (K, N)), (1, w16, K, N)
        else:
            q = oracle.quantize_weights(ftype, w)
            gpu[name], ref[name] = (ftype, q, (K, N)), (ftype, q, K, N)

    for s, (ci, ni) in enumerate(((0, 1), (3, 4), (6, 7), (9, 10))):
        conv(f"mem_enc.ds.{ci}.weight", DS[s + 1], DS[s], 3, 1.0 / np.sqrt(9 * DS[s]))
        f32(f"mem_enc.ds.{ci}.bias", rng.normal(0, 0.1, size=DS[s + 1]))
        f32(f"mem_enc.ds.{ni}.weight", 1 + rng.normal(0, 0.1, size=DS[s + 1]))
        f32(f"mem_enc.ds.{ni}.bias", rng.normal(0, 0.1, size=DS[s + 1]))
    conv("mem_enc.ds.12.weight", D, D, 1, 1.0 / 16)
    f32("mem_enc.ds.12.bias", rng.normal(0, 0.1, size=D))
    conv("mem_enc.pix_feat_proj.weight", D, D, 1, 1.0 / 16)
    f32("mem_enc.pix_feat_proj.bias", rng.normal(0, 0.1, size=D))
    for i in range(2):
        p = f"mem_enc.fuser.{i}."
        conv(p + "dwconv.weight", D, 1, 7, 1.0 / 7)
        f32(p + "dwconv.bias", rng.normal(0, 0.1, size=D))
        f32(p + "norm.weight", 1 + rng.normal(0, 0.1, size=D))
        f32(p + "norm.bias", rng.normal(0, 0.1, size=D))
        lin(p + "pwconv1.weight", D, FD)
        f32(p + "pwconv1.bias", rng.normal(0, 0.1, size=FD))
        lin(p + "pwconv2.weight", FD, D)
        f32(p + "pwconv2.bias", rng.normal(0, 0.1, size=D))
        f32(p + "gamma", rng.normal(0, 0.5, size=D))
    conv("mem_enc.out_proj.weight", MD, D, 1, 1.0 / 16)
    f32("mem_enc.out_proj.bias", rng.normal(0, 0.1, size=MD))
    f32("no_obj_embed_spatial", rng.normal(0, 0.5, size=MD))
    f32("mem_enc.tpos_enc", rng.normal(0, 0.1, size=(7, MD)))
    return gpu, ref


@pytest.mark.parametrize("feat,img,ftype,obj_score", [
    (64, 1024, 8, 1.5),    # SAM2 Hiera-B+ at 1024 (config 5), Q8_0 file, object visible
    (64, 1024, 1, -2.0),   # F16 file, occluded: + no_obj_embed_spatial
    (72, 1008, 8, -0.5),   # SAM3 tracker at 1008 (16H = 1152 != img)
])
def test_mem_enc_matches_oracle(oracle, backend, feat, img, ftype, obj_score):
    import mem_enc_oracle
    gpu, ref = make_mem_enc_tensors(oracle, ftype, seed=feat + ftype)
    hp = dict(feat=feat, img=img, d_model=D, mem_dim=MD, fuser_layers=2, fuser_dim=FD, sigmoid_scale=20.0,
              sigmoid_bias=-10.0, max_mask=(4 * feat) ** 2)
    rng = np.random.default_rng(feat)
    logits = rng.normal(0, 4, size=(4 * feat, 4 * feat)).astype(np.float32)
    pix = rng.normal(0, 1, size=(feat * feat, D)).astype(np.float32)
    me = backend.mem_encoder(hp)
    try:
        me.load(gpu)
        got = me.run(logits, pix, obj_score)
    finally:
        me.free()
    want = mem_enc_oracle.encode(hp, ref, logits, pix, obj_score)
    assert got.shape == want.shape and np.isfinite(got).all()
    assert rel_err(got, want) <= 1e-2, rel_err(got, want)


def test_mem_enc_rejects(b200, backend):
    hp = dict(feat=8, img=128, d_model=D, mem_dim=MD, fuser_layers=2, fuser_dim=FD, sigmoid_scale=20.0,
              sigmoid_bias=-10.0, max_mask=32 * 32)
    me = backend.mem_encoder(hp)
    try:
        with pytest.raises(b200.B200Error):
            me.run(np.zeros((32, 32), np.float32), np.zeros((64, D), np.float32))  # weights missing
        with pytest.raises(b200.B200Error):
            me.run(np.zeros((64, 64), np.float32), np.zeros((64, D), np.float32))  # mask beyond capacity
    finally:
        me.free()
    with pytest.raises(b200.B200Error):
        backend.mem_encoder(dict(hp, d_model=128))
