"""GPU parity of the SAM3 visual encoder (sam3_encode_image, sam3.cpp:6028)
against the CPU oracle, through the C ABI, stage by stage and end to end.

Tolerance (north-star bound for fp32 tensors): max|got - ref| / max|ref|
<= 1e-2.  Preprocessing is integer-exact and checked bit for bit.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(params=["dq16", "exact"])
def arith(request, b200, backend):
    """The encoder's linear-layer arithmetic (sam3b200_set_arith): DQ16 (the
    default: Q8_0 codes dequantised to fp16, fp16 tensor cores) and EXACT
    (int8 block dots, block-ordered fp32 fold); both at the same bound."""
    prev = backend.set_arith(b200.ARITH_DQ16 if request.param == "dq16" else b200.ARITH_EXACT)
    yield request.param
    backend.set_arith(prev)


@pytest.fixture(scope="module")
def small(model, oracle, backend):
    hp = model.SAM3_VIT_TEST
    tensors = model.random_vit_weights(hp, seed=1)
    vit = backend.vit(hp)
    vit.load(tensors)
    ov = oracle.OracleVit(hp, tensors)
    yield hp, tensors, vit, ov
    vit.free()


@pytest.mark.parametrize("w,h", [(672, 672), (500, 380), (1200, 1198)])
def test_preprocess_bit_exact(model, oracle, backend, small, w, h):
    hp, _, _, ov = small
    rgb = np.random.default_rng(w + h).integers(0, 256, size=(h, w, 3), dtype=np.uint8)
    src = backend.upload(rgb)
    out = backend.alloc(3 * hp["img"] ** 2 * 4)
    backend.preprocess(src, w, h, hp["img"], out)
    backend.synchronize()
    got = out.get((3, hp["img"], hp["img"]), np.float32)
    assert np.array_equal(got, ov.preprocess(rgb))


@pytest.mark.parametrize("w,h,img", [(1024, 1024, 1024), (640, 480, 1024), (300, 900, 512)])
def test_preprocess_sam2_bit_exact(oracle, backend, small, w, h, img):
    """sam2_preprocess_image (sam3.cpp:3522-3548): ImageNet normalisation, same resize."""
    _, _, _, ov = small
    rgb = np.random.default_rng(7 * w + h).integers(0, 256, size=(h, w, 3), dtype=np.uint8)
    src = backend.upload(rgb)
    out = backend.alloc(3 * img * img * 4)
    backend.preprocess_sam2(src, w, h, img, out)
    backend.synchronize()
    got = out.get((3, img, img), np.float32)
    assert np.array_equal(got, ov.preprocess_sam2(rgb, img))


def test_prefix(backend, small):
    hp, _, vit, ov = small
    img = ov.preprocess(np.random.default_rng(3).integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8))
    ref = ov.prefix(img)
    dimg, dx = backend.upload(img), backend.alloc(ref.nbytes)
    vit.run_prefix(dimg, dx)
    backend.synchronize()
    assert rel_err(dx.get(ref.shape, np.float32), ref) <= TOL


@pytest.fixture(scope="module")
def small_q4(model, oracle, backend):
    """The test geometry with Q4_0 linear weights: every MUL_MAT epilogue
    (RoPE'd Q/K/V^T, GELU + Q8_0 re-quantisation, residual) on nibble codes."""
    hp = dict(model.SAM3_VIT_TEST, wtype=model.Q4_0)
    tensors = model.random_vit_weights(hp, seed=3)
    vit = backend.vit(hp)
    vit.load(tensors)
    yield hp, tensors, vit, oracle.OracleVit(hp, tensors)
    vit.free()


@pytest.mark.parametrize("idx", [0, 1])
def test_block_q4_0(backend, small_q4, idx, arith):
    hp, _, vit, ov = small_q4
    x = np.random.default_rng(20 + idx).standard_normal((ov.G ** 2, hp["embed"]), dtype=np.float32)
    ref = ov.block(idx, x)
    dx = backend.upload(x)
    vit.run_block(idx, dx)
    backend.synchronize()
    err = rel_err(dx.get(ref.shape, np.float32), ref)
    assert err <= TOL, err


@pytest.mark.parametrize("idx", [0, 1])  # block 0 windowed, block 1 global
def test_block(backend, small, idx, arith):
    hp, _, vit, ov = small
    x = np.random.default_rng(idx).standard_normal((ov.G ** 2, hp["embed"]), dtype=np.float32)
    ref = ov.block(idx, x)
    dx = backend.upload(x)
    vit.run_block(idx, dx)
    backend.synchronize()
    err = rel_err(dx.get(ref.shape, np.float32), ref)
    assert err <= TOL, err


def test_neck(backend, small):
    hp, _, vit, ov = small
    x = np.random.default_rng(9).standard_normal((ov.G ** 2, hp["embed"]), dtype=np.float32)
    refs = ov.neck(x)
    vit.run_neck(backend.upload(x))
    for i, ref in enumerate(refs):
        err = rel_err(vit.output_host(i), ref)
        assert err <= TOL, (i, err)


def test_encode_end_to_end(small, arith):
    hp, _, vit, ov = small
    rgb = np.random.default_rng(5).integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8)
    x_ref, outs_ref = ov.encode(rgb)
    outs = vit.encode(rgb)
    assert rel_err(vit.output_host(-1).reshape(x_ref.shape), x_ref) <= TOL
    for i in range(4):
        err = rel_err(outs[i], outs_ref[i])
        assert err <= TOL, (i, err)


def test_encode_twice_is_deterministic(small):
    hp, _, vit, _ = small
    rgb = np.random.default_rng(6).integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8)
    a = vit.encode(rgb)
    b = vit.encode(rgb)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


@pytest.fixture(scope="module")
def full8(model, oracle, backend):
    """SAM3 ViT-32 geometry (1008^2, embed 1024, 16 heads, mlp 4736) with 8
    blocks, block 7 global -- the two block kinds at full size."""
    hp = dict(model.SAM3_VIT, depth=8, global_idx=(7,))
    tensors = model.random_vit_weights(hp, seed=2)
    vit = backend.vit(hp)
    vit.load(tensors)
    yield hp, vit, oracle.OracleVit(hp, tensors)
    vit.free()


@pytest.mark.parametrize("idx", [0, 7])
def test_full_size_block(backend, full8, idx, arith):
    hp, vit, ov = full8
    x = np.random.default_rng(idx).standard_normal((ov.G ** 2, hp["embed"]), dtype=np.float32)
    ref = ov.block(idx, x)
    dx = backend.upload(x)
    vit.run_block(idx, dx)
    backend.synchronize()
    err = rel_err(dx.get(ref.shape, np.float32), ref)
    assert err <= TOL, err


@pytest.fixture(scope="module")
def full32(model, oracle, backend):
    """Config 3 exactly as benchmarked: SAM3 ViT-32 (32 blocks, E = 1024, 16
    heads, MLP 4736, global blocks 7/15/23/31, Q8_0 weights) + tracker neck."""
    hp = model.SAM3_VIT
    tensors = model.random_vit_weights(hp, seed=11)
    vit = backend.vit(hp)
    vit.load(tensors)
    rgb = np.random.default_rng(12).integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8)
    yield hp, vit, oracle.OracleVit(hp, tensors), rgb
    vit.free()


def test_full_size_every_stage_on_the_gpu_trajectory(backend, full32, arith):
    """sam3_encode_image (sam3.cpp:6028-6216) at config 3, stage by stage along
    the GPU's own trajectory, at the fixed 1e-2 bound: the prefix on the
    preprocessed image, then each of the 32 blocks on the residual stream the
    GPU produced before it, then the neck on the GPU's final stream -- each
    against the oracle stage on the same input (the per-stage comparison of
    the reference's own test, tests/test_metal_block_stage_compare.cpp:380-440).
    The stepwise GPU path is the encode path: its outputs equal encode()'s bit
    for bit."""
    hp, vit, ov, rgb = full32
    img = ov.preprocess(rgb)
    dimg = backend.upload(img)
    x_ref = ov.prefix(img)
    dx = backend.alloc(x_ref.nbytes)
    vit.run_prefix(dimg, dx)
    backend.synchronize()
    x = dx.get(x_ref.shape, np.float32)
    errs = {"prefix": rel_err(x, x_ref)}
    for i in range(hp["depth"]):
        want = ov.block(i, x)
        vit.run_block(i, dx)
        backend.synchronize()
        x = dx.get(x_ref.shape, np.float32)
        errs[f"block{i}"] = rel_err(x, want)
    vit.run_neck(dx)
    refs = ov.neck(x)
    for i in range(4):
        errs[f"neck{i}"] = rel_err(vit.output_host(i), refs[i])
    print("stage errors:", ", ".join(f"{k} {v:.2e}" for k, v in errs.items()))
    assert max(errs.values()) <= TOL, errs
    outs = vit.encode(rgb)
    assert np.array_equal(vit.output_host(-1).reshape(x.shape), x)
    for i in range(4):
        assert np.array_equal(outs[i], vit.output_host(i))


def test_full_size_free_running_divergence(full32):
    """The free-running encode against the oracle's, next to the oracle against
    itself.  Thirty-two re-quantised blocks amplify any rounding-level change:
    the oracle with its attention in float64 instead of float32 -- an equally
    valid evaluation -- already lands ~1.4e-2 (max |d| / max |ref|) from its
    float32 self at the final stream and the neck, so no implementation that is
    not bit-identical to one particular evaluation can hold 1e-2 here.  The GPU
    must stay within 1.5x of that self-divergence."""
    hp, vit, ov, rgb = full32
    outs = vit.encode(rgb)
    x = vit.output_host(-1)
    x32, n32 = ov.encode(rgb)
    x64, n64 = ov.encode(rgb, attn_f64=True)
    gpu = [rel_err(x.reshape(x32.shape), x32)] + [rel_err(outs[i], n32[i]) for i in range(4)]
    own = [rel_err(x64, x32)] + [rel_err(n64[i], n32[i]) for i in range(4)]
    print("free-running, GPU vs oracle:", ", ".join(f"{e:.3e}" for e in gpu))
    print("free-running, oracle f64 vs f32:", ", ".join(f"{e:.3e}" for e in own))
    for g, o in zip(gpu, own):
        assert g <= 1.5 * o, (gpu, own)


def test_missing_weights_fail_loudly(b200, backend, model):
    hp = model.SAM3_VIT_TEST
    vit = backend.vit(hp)
    with pytest.raises(b200.B200Error):
        vit.encode(np.zeros((hp["img"], hp["img"], 3), np.uint8))
    with pytest.raises(b200.B200Error):
        vit.set_tensor("vit.blocks.0.attn.qkv.weight", 1, np.zeros(4, np.float32), (2, 2))
    vit.free()


def test_detector_neck(model, oracle, backend, small):
    """A full SAM3 model's second neck ("neck.det.*") on the same ViT output: its four levels match the
    oracle neck with those weights, and the tracker neck's levels are unchanged by its presence."""
    hp, tensors, vit_trk, _ = small
    det = model.random_det_neck_weights(hp, seed=9)
    vit = backend.vit(hp)
    try:
        vit.load({**tensors, **det})
        rgb = np.random.default_rng(8).integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8)
        trk = vit.encode(rgb)
        for a, b in zip(trk, vit_trk.encode(rgb)):
            assert np.array_equal(a, b)
        x = vit.output_host(-1)
        od = oracle.OracleVit(hp, {**tensors, **det}, neck_prefix="neck.det.")
        want = od.neck(x.reshape(-1, hp["embed"]))
        for i in range(4):
            got = vit.output_det_host(i)
            assert rel_err(got.reshape(want[i].shape), want[i]) <= TOL, i
    finally:
        vit.free()


def test_batch_encode_matches_single_encodes(b200, backend, small):
    """sam3b200_encode_images: n images through the blocks as one token batch (image-major rows, every
    launch over all of them) give each image exactly its single-image encode -- bit for bit, since no
    per-row arithmetic depends on the other rows -- also after a larger batch grew the buffers."""
    hp, _, vit, _ = small
    prev = backend.set_arith(b200.ARITH_DQ16)
    try:
        rng = np.random.default_rng(31)
        rgbs = [rng.integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8) for _ in range(3)]
        singles = [vit.encode(r) for r in rgbs]
        for group in (rgbs, rgbs[1:]):
            got = vit.encode_batch(group)
            for g, want in zip(got, singles[len(rgbs) - len(group):]):
                for a, b in zip(g, want):
                    assert np.array_equal(a, b)
    finally:
        backend.set_arith(prev)


def test_batch_encode_full_size(b200, backend, full8):
    """Two 1008^2 images as one batch through windowed and global (N = 5184) ViT-32 blocks at full size:
    both images' ViT outputs equal their single encodes bit for bit."""
    hp, vit, _ = full8
    prev = backend.set_arith(b200.ARITH_DQ16)
    try:
        rng = np.random.default_rng(32)
        rgbs = [rng.integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8) for _ in range(2)]
        singles = []
        for r in rgbs:
            outs = vit.encode(r)
            singles.append((vit.output_host(-1).copy(), outs))
        outs = vit.encode_batch(rgbs)
        x_all = vit.output_host(-1)  # the first image's rows; the second image's follow in device memory
        assert np.array_equal(x_all, singles[0][0])
        for i in range(2):
            for a, b in zip(outs[i], singles[i][1]):
                assert np.array_equal(a, b)
    finally:
        backend.set_arith(prev)
