"""Seeded random-init SAM mask-decoder and prompt-encoder weights (N(0, 0.02) linear weights
quantised to Q8_0; LayerNorm weights near 1; embeddings and the Fourier matrix N(0, 1)), in the
GPU-upload form and the oracle's form."""
import numpy as np

Q8_0, F32T = 8, 0


def dec_hparams(H: int) -> dict:
    return dict(feat_size=H, embed=256, depth=2, heads=8, mlp_dim=2048, n_multimask=3, pred_obj_scores=1,
                max_points=16)


def make_tensors(oracle, seed: int = 0):
    rng = np.random.default_rng(seed)
    D = 256
    gpu, ref = {}, {}

    def f32(name, arr, ne):
        arr = np.ascontiguousarray(arr, np.float32)
        gpu[name] = (F32T, arr, ne)
        ref[name] = arr

    def lin(name, K, N, sd=0.02):
        w = rng.normal(0, sd, size=(N, K)).astype(np.float32)
        q = oracle.quantize_weights(Q8_0, w)
        gpu[name] = (Q8_0, q, (K, N))
        ref[name] = (Q8_0, q, K, N)

    def attn(pfx, idim):
        for n in ("q", "k", "v"):
            lin(f"{pfx}.{n}_proj.weight", D, idim, 0.06)
            f32(f"{pfx}.{n}_proj.bias", rng.normal(0, 0.02, size=idim), (idim,))
        lin(f"{pfx}.out_proj.weight", idim, D, 0.06)
        f32(f"{pfx}.out_proj.bias", rng.normal(0, 0.02, size=D), (D,))

    def norm(pfx, n=D):
        f32(pfx + ".weight", 1 + rng.normal(0, 0.1, size=n), (n,))
        f32(pfx + ".bias", rng.normal(0, 0.1, size=n), (n,))

    f32("sam_pe.pe_gaussian", rng.normal(0, 1, size=(2, 128)), (128, 2))
    for i in range(4):
        f32(f"sam_pe.point_embeddings.{i}.weight", rng.normal(0, 1, size=D), (D, 1))
    f32("sam_pe.not_a_point_embed.weight", rng.normal(0, 1, size=D), (D, 1))
    f32("sam_pe.no_mask_embed.weight", rng.normal(0, 1, size=D), (D, 1))
    f32("no_mem_embed", rng.normal(0, 0.02, size=D), (D, 1, 1))
    f32("sam_dec.iou_token.weight", rng.normal(0, 1, size=D), (D, 1))
    f32("sam_dec.mask_tokens.weight", rng.normal(0, 1, size=(4, D)), (D, 4))
    f32("sam_dec.obj_score_token.weight", rng.normal(0, 1, size=D), (D, 1))
    for i in range(2):
        p = f"sam_dec.twoway.{i}"
        attn(p + ".sa", D)
        attn(p + ".cross_attn_token_to_image", 128)
        attn(p + ".cross_attn_image_to_token", 128)
        for j in range(1, 5):
            norm(f"{p}.norm{j}")
        lin(p + ".mlp.lin1.weight", D, 2048)
        f32(p + ".mlp.lin1.bias", rng.normal(0, 0.02, size=2048), (2048,))
        lin(p + ".mlp.lin2.weight", 2048, D)
        f32(p + ".mlp.lin2.bias", rng.normal(0, 0.02, size=D), (D,))
    attn("sam_dec.final_attn", 128)
    norm("sam_dec.final_norm")
    f32("sam_dec.upscale.0.weight", rng.normal(0, 0.05, size=(D, 64, 2, 2)), (2, 2, 64, D))
    f32("sam_dec.upscale.0.bias", rng.normal(0, 0.02, size=64), (64,))
    norm("sam_dec.upscale.1", 64)
    f32("sam_dec.upscale.3.weight", rng.normal(0, 0.1, size=(64, 32, 2, 2)), (2, 2, 32, 64))
    f32("sam_dec.upscale.3.bias", rng.normal(0, 0.02, size=32), (32,))
    f32("sam_dec.conv_s0.weight", rng.normal(0, 0.05, size=(32, D)), (1, 1, D, 32))
    f32("sam_dec.conv_s0.bias", rng.normal(0, 0.02, size=32), (32,))
    f32("sam_dec.conv_s1.weight", rng.normal(0, 0.05, size=(64, D)), (1, 1, D, 64))
    f32("sam_dec.conv_s1.bias", rng.normal(0, 0.02, size=64), (64,))
    for m in range(4):
        for j in range(3):
            lin(f"sam_dec.hyper.{m}.layers.{j}.weight", D, 32 if j == 2 else D, 0.06)
            f32(f"sam_dec.hyper.{m}.layers.{j}.bias", rng.normal(0, 0.02, size=32 if j == 2 else D), (32 if j == 2 else D,))
    for head, nout in (("iou_prediction_head", 4), ("pred_obj_score_head", 1)):
        for j in range(3):
            n = nout if j == 2 else D
            lin(f"sam_dec.{head}.layers.{j}.weight", D, n, 0.06)
            f32(f"sam_dec.{head}.layers.{j}.bias", rng.normal(0, 0.02, size=n), (n,))
    return gpu, ref
