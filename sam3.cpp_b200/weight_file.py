"""Writing weight files in the format sam3.cpp reads (sam3_load_model /
sam3_load_tensors, sam3.cpp:3095-3198, 3204-3330): used to hand seeded
random-init models to the native loader (sam3b200_file_open / _load) the way a
converted checkpoint would be.

Layout: uint32 magic ("sam3" 0x73616D33 version 3, "sam2" 0x73616D32 version 1),
int32 version, ftype, tensor count; the int32 hyper-parameter words in the
order of sam3_load_hparams / sam2_load_hparams; then per tensor int32 n_dims,
name length, ggml type, ne[0..n_dims) (ne0 first), the name, zero padding to
a 32-byte file offset, and the data (ggml blocks for quantised types).
"""
from __future__ import annotations

import struct

import numpy as np

SAM3_MAGIC, SAM3_VERSION = 0x73616D33, 3
SAM2_MAGIC, SAM2_VERSION = 0x73616D32, 1

# sam3_load_hparams word order after the global block indices (sam3.cpp:1495-1524)
SAM3_TAIL_FIELDS = ("text_width", "text_heads", "text_layers", "text_ctx_len", "text_vocab_size", "text_out_dim",
                    "neck_dim", "fenc_layers", "fenc_heads", "fenc_ffn_dim", "ddec_layers", "ddec_heads",
                    "ddec_ffn_dim", "ddec_num_queries", "geom_layers", "n_presence_tokens", "n_geom_queries",
                    "sam_embed_dim", "sam_dec_depth", "sam_n_multimask", "sam_iou_head_depth", "mem_out_dim",
                    "mem_attn_layers", "num_maskmem", "max_obj_ptrs", "n_amb_experts", "visual_only")
SAM3_TAIL_DEFAULTS = dict(text_width=1024, text_heads=16, text_layers=24, text_ctx_len=32, text_vocab_size=49408,
                          text_out_dim=256, neck_dim=256, fenc_layers=6, fenc_heads=8, fenc_ffn_dim=2048,
                          ddec_layers=6, ddec_heads=8, ddec_ffn_dim=2048, ddec_num_queries=200, geom_layers=3,
                          n_presence_tokens=1, n_geom_queries=4, sam_embed_dim=256, sam_dec_depth=2,
                          sam_n_multimask=3, sam_iou_head_depth=3, mem_out_dim=64, mem_attn_layers=4,
                          num_maskmem=7, max_obj_ptrs=16, n_amb_experts=2, visual_only=1)


def sam3_hparam_words(vit_hp: dict, **tail) -> list[int]:
    """The SAM3 hyper-parameter words for a visual encoder configuration (the model.SAM3_VIT keys) plus
    the remaining fields (defaults: the released SAM3, visual-only)."""
    ratio = int(round(vit_hp["mlp"] * 1000 / vit_hp["embed"]))
    g = list(vit_hp["global_idx"])
    words = [vit_hp["img"], vit_hp["patch"], vit_hp["embed"], vit_hp["depth"], vit_hp["heads"], ratio,
             vit_hp["window"], len(g)] + g[:4]
    vals = dict(SAM3_TAIL_DEFAULTS, neck_dim=vit_hp["neck_dim"], **tail)
    return words + [int(vals[k]) for k in SAM3_TAIL_FIELDS]


def _write_tensor(fout, name: str, qtype: int, arr: np.ndarray, ne) -> None:
    nb = name.encode()
    ne = [int(x) for x in ne]
    while len(ne) > 1 and ne[-1] == 1:  # ggml n_dims of the registered shape
        ne.pop()
    fout.write(struct.pack("<iii", len(ne), len(nb), qtype))
    fout.write(struct.pack(f"<{len(ne)}i", *ne))
    fout.write(nb)
    fout.write(b"\0" * ((32 - fout.tell() % 32) % 32))
    fout.write(np.ascontiguousarray(arr).tobytes())


def write(path: str, magic: int, version: int, ftype: int, hparam_words: list[int], tensors: dict) -> None:
    """tensors: name -> (ggml type, array, ne), the arrays already in the type's storage
    (f32, f16, or uint8 ggml blocks)."""
    with open(path, "wb") as fout:
        fout.write(struct.pack("<Iiii", magic, version, ftype, len(tensors)))
        fout.write(struct.pack(f"<{len(hparam_words)}i", *hparam_words))
        for name, (qtype, arr, ne) in tensors.items():
            _write_tensor(fout, name, qtype, arr, ne)
