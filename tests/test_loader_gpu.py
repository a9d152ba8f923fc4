"""Loading a sam3.cpp weight file through the native streaming loader (sam3b200_file_load: pinned
double buffer, reader thread, routing by tensor name) gives the same encoder and text encoder as
setting every tensor through the C ABI: outputs bit-identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TEXT_SMALL = dict(text_width=256, text_heads=4, text_layers=2, text_ctx_len=16, text_vocab_size=1000,
                  text_out_dim=256, visual_only=0)


def text_tensors(oracle, seed=3):
    rng = np.random.default_rng(seed)
    E, L, V, F = 256, 16, 1000, 1024
    t = {}

    def f32(name, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        t[name] = (0, arr, arr.shape[::-1])

    def lin(name, K, N):
        t[name] = (8, oracle.quantize_weights(8, rng.normal(0, 0.05, size=(N, K)).astype(np.float32)), (K, N))

    f32("text.token_embed.weight", rng.normal(0, 0.02, size=(V, E)))
    f32("text.pos_embed", rng.normal(0, 0.01, size=(L, E)))
    for i in range(2):
        p = f"text.blocks.{i}."
        lin(p + "attn.in_proj.weight", E, 3 * E)
        f32(p + "attn.in_proj.bias", rng.normal(0, 0.02, size=3 * E))
        lin(p + "attn.out_proj.weight", E, E)
        f32(p + "attn.out_proj.bias", rng.normal(0, 0.02, size=E))
        for n in ("ln_1", "ln_2"):
            f32(p + n + ".weight", 1 + rng.normal(0, 0.1, size=E))
            f32(p + n + ".bias", rng.normal(0, 0.1, size=E))
        lin(p + "mlp.fc1.weight", E, F)
        f32(p + "mlp.fc1.bias", rng.normal(0, 0.02, size=F))
        lin(p + "mlp.fc2.weight", F, E)
        f32(p + "mlp.fc2.bias", rng.normal(0, 0.02, size=E))
    f32("text.ln_final.weight", np.ones(E))
    f32("text.ln_final.bias", np.zeros(E))
    lin("text.resizer.weight", E, 256)
    f32("text.resizer.bias", rng.normal(0, 0.02, size=256))
    return t


def test_file_load_matches_set_tensor(tmp_path, oracle, b200, backend, model):
    from conftest import _load_pkg_module
    wf = _load_pkg_module("weight_file")
    hp = model.SAM3_VIT_TEST
    vit_t = model.random_vit_weights(hp, seed=1)
    txt_t = text_tensors(oracle)
    extra = {"geom.boxes_direct_project.weight": (0, np.zeros((256, 4), np.float32), (4, 256)),
             "sam_dec.iou_token.weight": (0, np.zeros(256, np.float32), (256, 1))}  # no decoder passed: skipped
    path = tmp_path / "sam3_small.ggml"
    wf.write(str(path), wf.SAM3_MAGIC, wf.SAM3_VERSION, 8, wf.sam3_hparam_words(hp, **TEXT_SMALL),
             {**vit_t, **txt_t, **extra})
    f = b200.WeightFile(str(path))
    vit_a = backend.vit(f.vit_hparams().to_dict())
    txt_a = backend.text_encoder(dict(f.text_hparams()))
    vit_b = backend.vit(hp)
    txt_b = backend.text_encoder(dict(width=256, heads=4, layers=2, ctx_len=16, vocab=1000, out_dim=256))
    try:
        loaded, skipped = f.load(backend, vit=vit_a, text=txt_a)
        assert (loaded, skipped) == (len(vit_t) + len(txt_t), len(extra))
        assert sorted(f.skipped()) == sorted(extra)
        vit_b.load(vit_t)
        txt_b.load(txt_t)
        rgb = np.random.default_rng(7).integers(0, 256, (hp["img"], hp["img"], 3), dtype=np.uint8)
        for x, y in zip(vit_a.encode(rgb), vit_b.encode(rgb)):
            assert np.array_equal(x, y)
        ids = np.array([49, 7, 311, 2], np.int32)
        assert np.array_equal(txt_a.encode(ids), txt_b.encode(ids))
    finally:
        for r in (vit_a, vit_b, txt_a, txt_b):
            r.free()
        f.close()


def test_file_load_stops_at_a_rejected_tensor(tmp_path, b200, backend, model):
    from conftest import _load_pkg_module
    wf = _load_pkg_module("weight_file")
    hp = model.SAM3_VIT_TEST
    t = dict(model.random_vit_weights(hp, seed=2))
    t["vit.ln_pre.weight"] = (0, np.ones(hp["embed"] + 1, np.float32), (hp["embed"] + 1,))  # wrong size
    path = tmp_path / "bad.ggml"
    wf.write(str(path), wf.SAM3_MAGIC, wf.SAM3_VERSION, 8, wf.sam3_hparam_words(hp), t)
    f = b200.WeightFile(str(path))
    vit = backend.vit(hp)
    try:
        with pytest.raises(b200.B200Error):
            f.load(backend, vit=vit)
    finally:
        vit.free()
        f.close()
