"""The native weight-file reader (sam3b200_file_*) on CPU: header, hyper-parameter words and tensor
directory of files in sam3.cpp's format (sam3.cpp:3095-3198, 3204-3330), written by the package's
writer; malformed files are rejected with an error, not read past their end."""
import struct

import numpy as np
import pytest


@pytest.fixture(scope="module")
def wf():
    from conftest import _load_pkg_module
    return _load_pkg_module("weight_file")


def write_vit_file(tmp_path, model, wf, extra=None, seed=1):
    hp = model.SAM3_VIT_TEST
    tensors = dict(model.random_vit_weights(hp, seed=seed))
    if extra:
        tensors.update(extra)
    path = tmp_path / "vit.ggml"
    wf.write(str(path), wf.SAM3_MAGIC, wf.SAM3_VERSION, 8, wf.sam3_hparam_words(hp), tensors)
    return path, hp, tensors


def test_sam3_directory_and_hparams(tmp_path, b200, model, wf):
    extra = {"geom.points_direct_project.weight": (0, np.arange(2 * 256, dtype=np.float32), (2, 256))}
    path, hp, tensors = write_vit_file(tmp_path, model, wf, extra)
    f = b200.WeightFile(str(path))
    try:
        info = f.info()
        assert info == dict(magic=wf.SAM3_MAGIC, version=3, ftype=8, n_tensors=len(tensors))
        assert f.hparams() == wf.sam3_hparam_words(hp)
        raw = path.read_bytes()
        for rec, (name, (qtype, arr, ne)) in zip(f.tensors(), tensors.items()):
            assert rec["name"] == name and rec["type"] == qtype
            assert rec["ne"] == tuple(list(ne) + [1] * (4 - len(ne)))
            assert rec["offset"] % 32 == 0 and rec["bytes"] == np.ascontiguousarray(arr).nbytes
            assert raw[rec["offset"]:rec["offset"] + rec["bytes"]] == np.ascontiguousarray(arr).tobytes()
        v = f.vit_hparams()
        assert (v.img, v.patch, v.embed, v.depth, v.heads, v.mlp, v.window) == \
            (hp["img"], hp["patch"], hp["embed"], hp["depth"], hp["heads"], hp["mlp"], hp["window"])
        assert list(v.global_idx)[:v.n_global] == list(hp["global_idx"])
        assert (v.pos_grid, v.neck_dim, v.wtype) == (hp["pos_grid"], hp["neck_dim"], hp["wtype"])
        assert f.text_hparams() == dict(width=1024, heads=16, layers=24, ctx_len=32, vocab=49408, out_dim=256)
    finally:
        f.close()


def test_sam2_hparams(tmp_path, b200, wf):
    words = [1024, 1, 96, 1, 4, 1, 2, 7, 2, 3, 5, 7, 9, 0, 0, 0, 0, 0, 3, 8, 4, 14, 7, 7, 7, 1, 256, 2, 2, 3, 0, 0,
             256, 2, 3, 3, 64, 4, 7, 16, 2000, -1000] + [1] * 15
    assert len(words) == 57
    path = tmp_path / "sam2.ggml"
    wf.write(str(path), wf.SAM2_MAGIC, wf.SAM2_VERSION, 8, words,
             {"no_mem_embed": (0, np.zeros(256, np.float32), (256, 1, 1))})
    f = b200.WeightFile(str(path))
    try:
        assert f.hparams() == words
        h = f.hiera_hparams()
        assert (h.img, h.embed, h.heads, list(h.stages), h.q_pool, list(h.window_spec)) == \
            (1024, 96, 1, [1, 2, 7, 2], 3, [8, 4, 14, 7])
        assert (h.n_global, list(h.global_idx)[:3], h.bkg_h, h.bkg_w, h.scalp, h.neck_dim) == \
            (3, [5, 7, 9], 7, 7, 1, 256)
        assert (h.fpn_top_down_n, list(h.fpn_top_down_levels)[:2]) == (2, [2, 3])
        assert f.tensors()[0]["ne"] == (256, 1, 1, 1)
        with pytest.raises(b200.B200Error):
            f.vit_hparams()  # not a SAM3 file
    finally:
        f.close()


def _corrupt(tmp_path, data: bytes, name: str):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def test_malformed_files_are_rejected(tmp_path, b200, model, wf):
    path, _, _ = write_vit_file(tmp_path, model, wf)
    raw = path.read_bytes()
    bad = {
        "magic": struct.pack("<I", 0x12345678) + raw[4:],
        "version": raw[:4] + struct.pack("<i", 2) + raw[8:],
        "truncated": raw[:len(raw) - 100],
        "short": raw[:10],
    }
    for name, data in bad.items():
        with pytest.raises(b200.B200Error):
            b200.WeightFile(_corrupt(tmp_path, data, name))
    # an unsupported ggml type in the first record
    hp_words = wf.sam3_hparam_words(model.SAM3_VIT_TEST)
    p = tmp_path / "type.ggml"
    wf.write(str(p), wf.SAM3_MAGIC, wf.SAM3_VERSION, 8, hp_words, {"vit.ln_pre.weight": (9, np.zeros(64, np.uint8), (32,))})
    with pytest.raises(b200.B200Error):
        b200.WeightFile(str(p))
    # an EdgeTAM (backbone 2) SAM2 file
    p = tmp_path / "edgetam.ggml"
    wf.write(str(p), wf.SAM2_MAGIC, wf.SAM2_VERSION, 8, [1024, 2] + [0] * 55, {})
    with pytest.raises(b200.B200Error):
        b200.WeightFile(str(p))
    with pytest.raises(b200.B200Error):
        b200.WeightFile(str(tmp_path / "missing.ggml"))
