"""SAM prompt encoder + mask decoder (PVS) through the C ABI against the CPU
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
