"""Seeded random-init SAM2 Hiera-tiny weights (config 1: N(0, 0.02) weights,
linear weights quantised to Q8_0 with the reference rule) in the two forms the
tests need: GPU upload tuples and the oracle's arrays."""
import numpy as np

Q8_0, F32T = 8, 0

HIERA_TINY = dict(embed=96, heads=1, stages=[1, 2, 7, 2], q_pool=3, window_spec=[8, 4, 14, 7],
                  global_idx=[5, 7, 9], bkg_h=7, bkg_w=7, neck_dim=256, fpn_top_down_levels=[2, 3], scalp=1)


HIERA_BASE_PLUS = dict(embed=112, heads=2, stages=[2, 3, 16, 3], q_pool=3, window_spec=[8, 4, 14, 7],
                       global_idx=[12, 16, 20], bkg_h=14, bkg_w=14, neck_dim=256, fpn_top_down_levels=[2, 3], scalp=1)
F16T = 1


def hiera_tiny(img: int) -> dict:
    return dict(HIERA_TINY, img=img)


def hiera_base_plus(img: int) -> dict:
    return dict(HIERA_BASE_PLUS, img=img)


def make_tensors(oracle, hiera_oracle, hp: dict, seed: int = 0, wtype: str = "q8"):
    """-> (gpu: name -> (type, array, ne), ref: name -> array | (qtype, blocks, K, N)).
    wtype: "q8" -- every linear weight Q8_0; "mixed" -- Q8_0 where the row length is a multiple of 32,
    F16 otherwise (what ggml's quantiser leaves in a Q8_0 Hiera-B+ file); "f16" -- every one F16."""
    rng = np.random.default_rng(seed)
    blocks, ends = hiera_oracle.metadata(hp)
    gpu, ref = {}, {}

    def f32(name, arr, ne):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name] = (F32T, arr, ne)
        ref[name] = arr

    def lin(name, K, N):
        w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
        if wtype == "f16" or (wtype == "mixed" and K % 32 != 0):
            w16 = w.astype(np.float16)
            gpu[name] = (F16T, w16, (K, N))
            ref[name] = (F16T, w16, K, N)
            return
        q = oracle.quantize_weights(Q8_0, w)
        gpu[name] = (Q8_0, q, (K, N))
        ref[name] = (Q8_0, q, K, N)

    E, ws0 = hp["embed"], hp["window_spec"][0]
    f32("hiera.patch_embed.weight", rng.normal(0, 0.02, size=(E, 3, 7, 7)), (7, 7, 3, E))
    f32("hiera.patch_embed.bias", rng.normal(0, 0.02, size=E), (E,))
    f32("hiera.pos_embed", rng.normal(0, 0.02, size=(E, hp["bkg_h"], hp["bkg_w"])), (hp["bkg_w"], hp["bkg_h"], E))
    f32("hiera.pos_embed_window", rng.normal(0, 0.02, size=(E, ws0, ws0)), (ws0, ws0, E))
    for i, m in enumerate(blocks):
        p, di, do = f"hiera.blocks.{i}.", m["dim_in"], m["dim_out"]
        f32(p + "norm1.weight", 1 + rng.normal(0, 0.1, size=di), (di,))
        f32(p + "norm1.bias", rng.normal(0, 0.1, size=di), (di,))
        f32(p + "norm2.weight", 1 + rng.normal(0, 0.1, size=do), (do,))
        f32(p + "norm2.bias", rng.normal(0, 0.1, size=do), (do,))
        lin(p + "attn.qkv.weight", di, 3 * do)
        f32(p + "attn.qkv.bias", rng.normal(0, 0.02, size=3 * do), (3 * do,))
        lin(p + "attn.proj.weight", do, do)
        f32(p + "attn.proj.bias", rng.normal(0, 0.02, size=do), (do,))
        lin(p + "mlp.fc1.weight", do, 4 * do)
        f32(p + "mlp.fc1.bias", rng.normal(0, 0.02, size=4 * do), (4 * do,))
        lin(p + "mlp.fc2.weight", 4 * do, do)
        f32(p + "mlp.fc2.bias", rng.normal(0, 0.02, size=do), (do,))
        if di != do:
            lin(p + "proj.weight", di, do)
            f32(p + "proj.bias", rng.normal(0, 0.02, size=do), (do,))
    D = hp["neck_dim"]
    stage_dims = [blocks[e]["dim_out"] for e in ends]
    for j in range(4):
        C = stage_dims[3 - j]
        f32(f"fpn.convs.{j}.weight", rng.normal(0, 0.02, size=(D, C)), (1, 1, C, D))
        f32(f"fpn.convs.{j}.bias", rng.normal(0, 0.02, size=D), (D,))
    return gpu, ref
