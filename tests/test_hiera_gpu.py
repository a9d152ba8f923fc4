"""SAM2 Hiera image encoder (sam3.cpp:4194-4583; config 1 = Hiera-tiny) through the
C ABI against the CPU oracle (oracle/hiera_oracle.py)."""
import numpy as np
import pytest

from conftest import rel_err
from hiera_model import hiera_base_plus, hiera_tiny, make_tensors

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def hiera_oracle():
    import hiera_oracle as h
    return h


@pytest.fixture(scope="module")
def tiny256(oracle, hiera_oracle, backend):
    hp = hiera_tiny(256)
    gpu, ref = make_tensors(oracle, hiera_oracle, hp, seed=3)
    model = backend.hiera(hp)
    model.load(gpu)
    yield hp, model, ref
    model.free()


def test_block_metadata_matches_oracle(hiera_oracle, tiny256):
    hp, model, _ = tiny256
    blocks, _ = hiera_oracle.metadata(hp)
    for i, m in enumerate(blocks):
        assert model.block_info(i) == (m["dim_in"], m["dim_out"], m["heads"], m["ws"], int(m["q_stride"]))


@pytest.mark.parametrize("i", range(12))
def test_block_matches_oracle(backend, hiera_oracle, tiny256, i):
    """Every Hiera-tiny block at a 256x256 input: windowed (8, 4, padded 14, padded 7), global,
    Q-stride with dimension projection, and the padded Q-stride block whose output is cropped."""
    hp, model, ref = tiny256
    blocks, _ = hiera_oracle.metadata(hp)
    m = blocks[i]
    S = 64
    for b in blocks[:i]:
        if b["q_stride"]:
            S //= 2
    x = np.random.default_rng(100 + i).normal(0, 1, size=(S, S, m["dim_in"])).astype(np.float32)
    So = S // 2 if m["q_stride"] else S
    dx = backend.upload(x)
    out = backend.alloc(So * So * m["dim_out"] * 4)
    model.run_block(i, dx, S, S, out)
    backend.synchronize()
    got = out.get((So, So, m["dim_out"]), np.float32)
    p = f"hiera.blocks.{i}."
    want = hiera_oracle.block(m, {k[len(p):]: v for k, v in ref.items() if k.startswith(p)}, x)
    assert rel_err(got, want) <= 1e-2, (i, rel_err(got, want))


def test_prefix_matches_oracle(backend, hiera_oracle, tiny256):
    hp, model, ref = tiny256
    img = np.random.default_rng(7).normal(0, 1, size=(3, 256, 256)).astype(np.float32)
    x = backend.alloc(64 * 64 * 96 * 4)
    model.run_prefix(backend.upload(img), x)
    backend.synchronize()
    pe = hiera_oracle.pos_embed(ref["hiera.pos_embed"], ref["hiera.pos_embed_window"], 64)
    want = hiera_oracle.prefix(img, ref["hiera.patch_embed.weight"], ref["hiera.patch_embed.bias"], pe)
    assert rel_err(x.get((64, 64, 96), np.float32), want) <= 1e-2


@pytest.mark.parametrize("img", [256, 1024])
def test_encode_matches_oracle(oracle, hiera_oracle, backend, img):
    """Free-running trunk + FPN neck from a preprocessed image: the four stage outputs and the three
    FPN levels against the oracle's own encode, next to the oracle against itself.

    Twelve chained blocks of activation quantisation amplify rounding-level differences (a code
    that flips costs a full quantisation step downstream): two equally valid oracle evaluations
    (attention in float64 and in float32) already differ by up to ~1.7e-2 at 1024x1024, and the
    divergence saturates quickly with the size of the perturbation -- the oracle's own encode with
    the attention operands rounded to fp16 (q, k, v, probabilities: the tensor-core kernel's
    operand precision, each a relative 2^-11 perturbation) moves stage 2 at 256x256 by 1.24e-2
    against 0.63e-2 for float32.  So the free-running GPU encode is held to 1e-2, twice the float32
    self-divergence or 1.25 times the fp16-operand one, whichever is largest; parity at the fixed
    1e-2 bound is checked block by block and stage by stage on the GPU's own trajectory
    (test_encode_every_stage_on_the_gpu_trajectory)."""
    hp = hiera_tiny(img)
    gpu, ref = make_tensors(oracle, hiera_oracle, hp, seed=11)
    model = backend.hiera(hp)
    try:
        model.load(gpu)
        chw = np.random.default_rng(img).normal(0, 1, size=(3, img, img)).astype(np.float32)
        model.encode_device(backend.upload(chw))
        stages, fpn = hiera_oracle.encode(hp, ref, chw)
        stages32, fpn32 = hiera_oracle.encode(hp, ref, chw, np.float32)
        stages16, fpn16 = hiera_oracle.encode(hp, ref, chw, np.float16)
        for s in range(4):
            bound = max(1e-2, 2 * rel_err(stages32[s], stages[s]), 1.25 * rel_err(stages16[s], stages[s]))
            err = rel_err(model.output_host(4 + s), stages[s])
            assert err <= bound, ("stage", s, err, bound)
        for lvl in range(3):
            bound = max(1e-2, 2 * rel_err(fpn32[lvl], fpn[lvl]), 1.25 * rel_err(fpn16[lvl], fpn[lvl]))
            err = rel_err(model.output_host(lvl), fpn[lvl])
            assert err <= bound, ("fpn", lvl, err, bound)
    finally:
        model.free()


@pytest.mark.parametrize("img", [256, 1024])
def test_encode_every_stage_on_the_gpu_trajectory(oracle, hiera_oracle, backend, img):
    """sam2_encode_image_hiera (sam3.cpp:5861-6022) stage by stage along the GPU's own trajectory at the
    fixed 1e-2 bound: the prefix on the image, each of the 12 blocks on the output the GPU produced
    before it, and the FPN neck on the GPU's four stage outputs -- each against the oracle stage on the
    same input.  The stepwise path is the encode path: its stage outputs equal encode_device's bit for
    bit."""
    hp = hiera_tiny(img)
    gpu, ref = make_tensors(oracle, hiera_oracle, hp, seed=11)
    model = backend.hiera(hp)
    try:
        model.load(gpu)
        chw = np.random.default_rng(img).normal(0, 1, size=(3, img, img)).astype(np.float32)
        blocks, ends = hiera_oracle.metadata(hp)
        S = (img - 1) // 4 + 1
        dx = backend.alloc(S * S * blocks[0]["dim_in"] * 4)
        model.run_prefix(backend.upload(chw), dx)
        backend.synchronize()
        x = dx.get((S, S, blocks[0]["dim_in"]), np.float32)
        pe = hiera_oracle.pos_embed(ref["hiera.pos_embed"], ref["hiera.pos_embed_window"], S)
        errs = {"prefix": rel_err(x, hiera_oracle.prefix(chw, ref["hiera.patch_embed.weight"],
                                                          ref["hiera.patch_embed.bias"], pe))}
        stages = []
        for i, m in enumerate(blocks):
            p = f"hiera.blocks.{i}."
            want = hiera_oracle.block(m, {k[len(p):]: v for k, v in ref.items() if k.startswith(p)}, x)
            So = S // 2 if m["q_stride"] else S
            out = backend.alloc(So * So * m["dim_out"] * 4)
            model.run_block(i, backend.upload(x), S, S, out)
            backend.synchronize()
            x = out.get((So, So, m["dim_out"]), np.float32)
            errs[f"block{i}"] = rel_err(x, want)
            S = So
            if i in ends:
                stages.append(x)
        model.encode_device(backend.upload(chw))
        for s in range(4):
            assert np.array_equal(model.output_host(4 + s).reshape(stages[s].shape), stages[s]), s
        convs = [(ref[f"fpn.convs.{j}.weight"], ref[f"fpn.convs.{j}.bias"]) for j in range(4)]
        want_fpn = hiera_oracle.fpn(stages, convs, hp["fpn_top_down_levels"], hp["scalp"])
        for lvl in range(len(want_fpn)):
            errs[f"fpn{lvl}"] = rel_err(model.output_host(lvl).reshape(want_fpn[lvl].shape), want_fpn[lvl])
        print("stage errors:", ", ".join(f"{k} {v:.2e}" for k, v in errs.items()))
        assert max(errs.values()) <= 1e-2, errs
    finally:
        model.free()


def test_hiera_rejects_unknown_tensor_and_missing(b200, backend):
    model = backend.hiera(hiera_tiny(256))
    try:
        with pytest.raises(b200.B200Error):
            model.set_tensor("hiera.blocks.99.norm1.weight", 0, np.zeros(96, np.float32), (96,))
        with pytest.raises(b200.B200Error):
            model.load({})  # nothing set: missing tensors reported
    finally:
        model.free()


@pytest.mark.parametrize("i", [4, 5, 10])
def test_block_matches_oracle_1024(oracle, hiera_oracle, backend, i):
    """Stage-2 geometry of a 1024x1024 input: block 4 (14-token windows padded 64 -> 70), block 5
    (global, 4096 tokens: 32 key tiles of the tcgen05 flash kernel) and block 10 (Q-stride, padded
    windows, cropped output)."""
    hp = hiera_tiny(1024)
    gpu, ref = make_tensors(oracle, hiera_oracle, hp, seed=21)
    model = backend.hiera(hp)
    try:
        model.load(gpu)
        blocks, _ = hiera_oracle.metadata(hp)
        m = blocks[i]
        S, So = 64, (32 if m["q_stride"] else 64)
        x = np.random.default_rng(200 + i).normal(0, 1, size=(S, S, m["dim_in"])).astype(np.float32)
        out = backend.alloc(So * So * m["dim_out"] * 4)
        model.run_block(i, backend.upload(x), S, S, out)
        backend.synchronize()
        p = f"hiera.blocks.{i}."
        want = hiera_oracle.block(m, {k[len(p):]: v for k, v in ref.items() if k.startswith(p)}, x)
        err = rel_err(out.get((So, So, m["dim_out"]), np.float32), want)
        assert err <= 1e-2, (i, err)
    finally:
        model.free()


@pytest.fixture(scope="module", params=["mixed", "f16"])
def base_plus256(request, oracle, hiera_oracle, backend):
    """Hiera-base+ (config 5's backbone: embed 112, stages 2/3/16/3, global blocks 12/16/20, 14x14
    background embedding) at a 256x256 input; "mixed": Q8_0 weights except the ones whose row length
    112 is no multiple of 32 (F16, as ggml's quantiser leaves them); "f16": an F16 file."""
    hp = hiera_base_plus(256)
    gpu, ref = make_tensors(oracle, hiera_oracle, hp, seed=9, wtype=request.param)
    model = backend.hiera(hp)
    model.load(gpu)
    yield hp, model, ref
    model.free()


@pytest.mark.parametrize("i", [0, 1, 2, 4, 5, 12, 21, 22])
def test_base_plus_block_matches_oracle(backend, hiera_oracle, base_plus256, i):
    """Hiera-B+ blocks: stage 1 (dims 112, F16 linear weights in both files), the stage transitions with
    their dimension projection (112 -> 224, 448 -> 896), a global block (12), the last stage."""
    hp, model, ref = base_plus256
    blocks, _ = hiera_oracle.metadata(hp)
    m = blocks[i]
    assert model.block_info(i) == (m["dim_in"], m["dim_out"], m["heads"], m["ws"], int(m["q_stride"]))
    S = 64
    for b in blocks[:i]:
        if b["q_stride"]:
            S //= 2
    x = np.random.default_rng(200 + i).normal(0, 1, size=(S, S, m["dim_in"])).astype(np.float32)
    So = S // 2 if m["q_stride"] else S
    out = backend.alloc(So * So * m["dim_out"] * 4)
    model.run_block(i, backend.upload(x), S, S, out)
    backend.synchronize()
    got = out.get((So, So, m["dim_out"]), np.float32)
    p = f"hiera.blocks.{i}."
    want = hiera_oracle.block(m, {k[len(p):]: v for k, v in ref.items() if k.startswith(p)}, x)
    assert rel_err(got, want) <= 1e-2, (i, rel_err(got, want))


def test_base_plus_encode_every_stage_on_the_gpu_trajectory(backend, hiera_oracle, base_plus256):
    """The whole Hiera-B+ trunk + FPN at 256x256 stage by stage along the GPU's trajectory (each block
    against the oracle block on the GPU's own input) at the fixed 1e-2 bound."""
    hp, model, ref = base_plus256
    blocks, ends = hiera_oracle.metadata(hp)
    img = np.random.default_rng(8).normal(0, 1, size=(3, 256, 256)).astype(np.float32)
    x = backend.alloc(64 * 64 * hp["embed"] * 4)
    model.run_prefix(backend.upload(img), x)
    backend.synchronize()
    S, errs = 64, {}
    cur = x.get((S, S, hp["embed"]), np.float32)
    for i, m in enumerate(blocks):
        So = S // 2 if m["q_stride"] else S
        out = backend.alloc(So * So * m["dim_out"] * 4)
        model.run_block(i, backend.upload(cur), S, S, out)
        backend.synchronize()
        got = out.get((So, So, m["dim_out"]), np.float32)
        p = f"hiera.blocks.{i}."
        errs[i] = rel_err(got, hiera_oracle.block(m, {k[len(p):]: v for k, v in ref.items() if k.startswith(p)}, cur))
        cur, S = got, So
    print("Hiera-B+ block errors:", ", ".join(f"{k}: {v:.2e}" for k, v in errs.items()))
    assert max(errs.values()) <= 1e-2, errs
