"""SAM prompt encoder + mask decoder (PVS, sam3.cpp:10164-11115) through the C ABI against the CPU
oracle (oracle/sam_dec_oracle.py): decoder outputs within 1e-2, final binary masks at IoU >= 0.99."""
import numpy as np
import pytest

from conftest import rel_err
from sam_dec_model import dec_hparams, make_tensors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dec_oracle():
    import sam_dec_oracle as d
    return d


@pytest.fixture(scope="module")
def dec16(oracle, backend):
    hp = dec_hparams(16)
    gpu, ref = make_tensors(oracle, seed=5)
    dec = backend.sam_decoder(hp)
    dec.load(gpu)
    yield hp, dec, ref
    dec.free()


PROMPTS = [  # (coords in a 300 x 200 image, labels): one positive point; box + negative point; two points
    ([[120.0, 80.0]], [1]),
    ([[40.0, 30.0], [250.0, 170.0], [60.0, 150.0]], [2, 3, 0]),
    ([[10.0, 190.0], [299.0, 0.5]], [1, 0]),
]


@pytest.mark.parametrize("case", range(len(PROMPTS)))
def test_decoder_matches_oracle(backend, dec_oracle, dec16, case):
    hp, dec, ref = dec16
    H = hp["feat_size"]
    rng = np.random.default_rng(40 + case)
    img = rng.normal(0, 1, size=(H, H, 256)).astype(np.float32)
    s0 = rng.normal(0, 1, size=(4 * H, 4 * H, 256)).astype(np.float32)
    s1 = rng.normal(0, 1, size=(2 * H, 2 * H, 256)).astype(np.float32)
    coords, labels = PROMPTS[case]
    di, d0, d1 = backend.upload(img), backend.upload(s0), backend.upload(s1)
    dec.run(di.ptr, d0.ptr, d1.ptr, coords, labels, 300, 200, 4 * H * 4)
    masks, iou, obj, tok = dec.outputs()
    want = dec_oracle.decode(hp, ref, img, s0, s1, coords, labels, 300, 200, 4 * H * 4)
    assert rel_err(masks, want[0]) <= 1e-2
    assert np.abs(iou - want[1]).max() <= 1e-2
    assert abs(obj - want[2]) <= 1e-2 * max(1.0, abs(want[2]))
    assert rel_err(tok, want[3]) <= 1e-2
    for m in range(4):
        got = dec.mask(m, 300, 200)
        ref_mask = dec_oracle.resize_threshold(want[0][m], 300, 200)
        assert 0.02 < (ref_mask > 0).mean() < 0.98  # a non-trivial mask
        assert dec_oracle.mask_iou(got, ref_mask) >= 0.99, (m, dec_oracle.mask_iou(got, ref_mask))


def test_decoder_rejects_bad_prompts(b200, backend, dec16):
    hp, dec, _ = dec16
    buf = backend.alloc(16)
    with pytest.raises(b200.B200Error):
        dec.run(buf.ptr, buf.ptr, buf.ptr, [[1.0, 1.0]], [5], 10, 10, 64)  # label out of range
    with pytest.raises(b200.B200Error):
        dec.run(buf.ptr, buf.ptr, buf.ptr, [[1.0, 1.0]] * 16, [1] * 16, 10, 10, 64)  # beyond max_points


def test_config1_image_to_mask(oracle, dec_oracle, backend):
    """Config 1 end to end (SAM2.1 Hiera-tiny, Q8_0, one positive point): uint8 image -> SAM2 preprocessing
    -> Hiera trunk + FPN -> prompt encoder + mask decoder -> masks at the original size.

    Three checks.  (a) The decoder at this geometry, fed the oracle's own FPN features: every final mask at
    IoU >= 0.99 against the oracle.  (c) The decoder fed the GPU's own FPN features (the chain's actual
    hand-off), against the oracle decoder on those same features: every final mask at IoU >= 0.99, or
    disagreeing only on pixels whose reference logit is within 1e-2 of the logit range, or twice the
    oracle's own float64-vs-float32 logit difference, of zero; with
    the Hiera encode held to 1e-2 stage by stage on its own trajectory (test_hiera_gpu), every stage of
    the chain meets the fixed bounds.  (b) The whole chain free-running against the oracle chain: twelve random-init
    quantised Hiera blocks amplify rounding-level differences (see test_hiera_gpu), so two valid oracle
    evaluations (attention in float64 and float32) agree only to IoU 0.98-0.99 on these masks; the GPU
    must agree with the oracle to within twice that disagreement, 1 - 2 (1 - self IoU), and never
    better than asked: min(0.99, that)."""
    import hiera_oracle
    from hiera_model import hiera_tiny, make_tensors as hiera_tensors
    hp, dhp = hiera_tiny(1024), dec_hparams(64)
    hg, hr = hiera_tensors(oracle, hiera_oracle, hp, seed=31)
    dg, dr = make_tensors(oracle, seed=32)
    W, Hh = 900, 700
    rgb = np.random.default_rng(33).integers(0, 256, size=(Hh, W, 3), dtype=np.uint8)
    point, label = [[410.0, 300.0]], [1]
    chw_ref = oracle.preprocess_sam2(rgb, 1024)
    _, fpn = hiera_oracle.encode(hp, hr, chw_ref)
    _, fpn32 = hiera_oracle.encode(hp, hr, chw_ref, np.float32)
    masks, iou_ref, _, _ = dec_oracle.decode(dhp, dr, fpn[2], fpn[0], fpn[1], point, label, W, Hh, 1024)
    masks32 = dec_oracle.decode(dhp, dr, fpn32[2], fpn32[0], fpn32[1], point, label, W, Hh, 1024)[0]
    enc, dec = backend.hiera(hp), backend.sam_decoder(dhp)
    try:
        enc.load(hg)
        dec.load(dg)
        # (a) decoder on the oracle's features
        f2, f0, f1 = (backend.upload(np.ascontiguousarray(f)) for f in (fpn[2], fpn[0], fpn[1]))
        dec.run(f2.ptr, f0.ptr, f1.ptr, point, label, W, Hh, 1024)
        for m in range(4):
            ref = dec_oracle.resize_threshold(masks[m], W, Hh)
            assert dec_oracle.mask_iou(dec.mask(m, W, Hh), ref) >= 0.99, ("decoder", m)
        # (b) the whole chain on the GPU
        src = backend.upload(rgb)
        chw = backend.alloc(3 * 1024 * 1024 * 4)
        backend.preprocess_sam2(src, W, Hh, 1024, chw)
        enc.encode_device(chw)
        dec.run(enc.output_ptr(2), enc.output_ptr(0), enc.output_ptr(1), point, label, W, Hh, 1024)
        got = [dec.mask(m, W, Hh) for m in range(4)]
        _, iou, _, _ = dec.outputs()
        # (c) the oracle decoder on the GPU's own FPN features
        gf = [enc.output_host(lvl) for lvl in range(3)]
        gf = [np.ascontiguousarray(f.reshape(fpn[lvl].shape)) for lvl, f in enumerate(gf)]
        masks_g = dec_oracle.decode(dhp, dr, gf[2], gf[0], gf[1], point, label, W, Hh, 1024)[0]
        masks_g32 = dec_oracle.decode(dhp, dr, gf[2], gf[0], gf[1], point, label, W, Hh, 1024,
                                      attn_dtype=np.float32)[0]
        for m in range(4):
            lg = dec_oracle.resize_logits(masks_g[m], W, Hh)
            ref_g = np.where(lg > 0, 255, 0).astype(np.uint8)
            iou_g = dec_oracle.mask_iou(got[m], ref_g)
            # where IoU < 0.99 every disagreeing pixel must be one whose reference logit is ambiguous:
            # within 1e-2 of the logit range, or within twice the oracle's own float64-vs-float32
            # logit difference, of the threshold.  The random-init decoder leaves wide plateaus of
            # near-zero logits here, where the oracle's two evaluations already disagree on ~1.1% of
            # the pixels of masks 0 and 3
            noise = float(np.abs(dec_oracle.resize_logits(masks_g32[m], W, Hh) - lg).max())
            dis = (got[m] > 0) != (ref_g > 0)
            ambiguous = np.abs(lg) <= max(1e-2 * np.abs(lg).max(), 2 * noise)
            assert iou_g >= 0.99 or bool(np.all(ambiguous[dis])), ("decoder on the GPU's features", m, iou_g,
                                                                  int(dis.sum()), int((dis & ~ambiguous).sum()))
    finally:
        enc.free()
        dec.free()
    assert np.abs(iou - iou_ref).max() <= 2e-2
    for m in range(4):
        ref = dec_oracle.resize_threshold(masks[m], W, Hh)
        self_iou = dec_oracle.mask_iou(dec_oracle.resize_threshold(masks32[m], W, Hh), ref)
        bound = min(0.99, 1 - 2 * (1 - self_iou))
        assert dec_oracle.mask_iou(got[m], ref) >= bound, (m, dec_oracle.mask_iou(got[m], ref), bound)
