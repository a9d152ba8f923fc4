"""The video tracker's frame loop on the GPU (sam3b200_tracker: sam3_tracker_add_instance +
sam3_propagate_frame, sam3.cpp:12017-12262) over a 9-frame stream with one box prompt on frame 0 --
config 5's structure (SAM2 tracker: 7 memory slots, 16 object pointers, multimask_output_in_sam, the
fixed_no_obj_ptr blend) at a reduced geometry (Hiera-tiny at 512: 32 x 32 tokens) so that the
numpy oracles finish in seconds.

Every frame is checked stage by stage on the GPU's own trajectory against the CPU oracles, each fed
the GPU's inputs of that stage: the memory prompt (bit-exact features, positional rows within 1e-5),
the memory attention (1e-2), the decoder (predicted IoUs within 1e-2, the kept mask at IoU >= 0.99 at the
original size), the memory encoder (1e-2) and the object pointer (1e-4).  The decoder's mask logits are
reported, not bounded, here: its token MLPs re-quantise seven token rows to Q8_0, and a code that flips
on a rounding-level input difference moves one mask's logits by ~1-2% of their maximum (typically the
four masks agree within 2e-3; single masks reach 2.4e-2 on some frames), while the kept mask's binary
IoU stays >= 0.99.  The decoder's logits are held to 1e-2 on their own in test_sam_dec_gpu.

Then the whole loop free-running against the oracle loop fed the same encoder features.  The loop
amplifies rounding-level differences: the Q8_0 re-quantisation of every linear layer's input flips
codes, and the kept mask is an argmax over predicted IoUs.  Two equally valid oracle evaluations --
the memory attention in float64 and in float32 -- already fall to IoU 0.90-0.98 against each other on
some frames of such a stream, while i.i.d. noise of 5e-3 on the conditioned features keeps IoU above
0.99.  So the free-running GPU loop is held to the oracle's own spread: its mean mask disagreement
(1 - IoU) over the stream at most 1.5x the float32 oracle's, or 0.01."""
import numpy as np
import pytest

from conftest import rel_err
from hiera_model import hiera_tiny, make_tensors as hiera_tensors
from sam_dec_model import dec_hparams, make_tensors as dec_tensors
from test_mem_attn_gpu import LAYERS, make_mem_tensors
from test_mem_enc_gpu import make_mem_enc_tensors

pytestmark = pytest.mark.gpu

D, MD, IMG, NMEM, NPTR = 256, 64, 512, 7, 16
W, HH = 600, 450
BOX, BOX_LABELS = [[110.0, 90.0], [420.0, 360.0]], [2, 3]


def tracker_tensors(seed):
    rng = np.random.default_rng(seed)
    t = {}
    for j in range(3):
        t[f"obj_ptr_proj.layers.{j}.weight"] = rng.normal(0, 1 / 16, size=(D, D)).astype(np.float32)
        t[f"obj_ptr_proj.layers.{j}.bias"] = rng.normal(0, 0.1, size=D).astype(np.float32)
    t["no_obj_ptr"] = rng.normal(0, 1, size=D).astype(np.float32)
    t["obj_ptr_tpos_proj.weight"] = rng.normal(0, 1 / 16, size=(MD, D)).astype(np.float32)
    t["obj_ptr_tpos_proj.bias"] = rng.normal(0, 0.1, size=MD).astype(np.float32)
    t["mem_enc.tpos_enc"] = rng.normal(0, 0.1, size=(NMEM, MD)).astype(np.float32)
    return {k: (0, v, v.shape[::-1]) for k, v in t.items()}, t


def synth_logits(mask_u8, S):
    """sam3_tracker_add_instance's +-6 logits on the S x S grid from a binary mask (sam3.cpp:12043-12054)."""
    h, w = mask_u8.shape
    sy = (np.arange(S) * h) // S
    sx = (np.arange(S) * w) // S
    return np.where(mask_u8[sy][:, sx] > 127, 6.0, -6.0).astype(np.float32)


@pytest.fixture(scope="module")
def stream(oracle, backend):
    import hiera_oracle
    hp_h = hiera_tiny(IMG)
    H = IMG // 16
    hg, _ = hiera_tensors(oracle, hiera_oracle, hp_h, seed=71)
    hp_d = dec_hparams(H)
    dg, dr = dec_tensors(oracle, seed=72)
    ag, ar = make_mem_tensors(oracle, seed=73)
    eg, er = make_mem_enc_tensors(oracle, 8, seed=74)
    tg, tr_ref = tracker_tensors(75)
    hp_a = dict(d_model=D, mem_dim=MD, layers=LAYERS, ffn_dim=2048, max_tokens=H * H,
                max_mem_tokens=NMEM * H * H + NPTR * (D // MD))
    hp_e = dict(feat=H, img=IMG, d_model=D, mem_dim=MD, fuser_layers=2, fuser_dim=1024, sigmoid_scale=20.0,
                sigmoid_bias=-10.0, max_mask=(4 * H) ** 2)
    hp_t = dict(feat=H, img=IMG, d_model=D, mem_dim=MD, num_maskmem=NMEM, max_obj_ptrs=NPTR, multimask_in_sam=1,
                multimask_token_for_obj_ptr=1, fixed_no_obj_ptr=1, max_instances=4, max_keep_alive=100)
    enc, dec = backend.hiera(hp_h), backend.sam_decoder(hp_d)
    attn, menc = backend.mem_attention(hp_a), backend.mem_encoder(hp_e)
    enc.load(hg)
    dec.load(dg)
    attn.load(ag)
    menc.load(eg)
    tr = backend.tracker(hp_t, enc, dec, attn, menc)
    tr.load(tg)
    frames = [np.random.default_rng(80 + f).integers(0, 256, size=(HH, W, 3), dtype=np.uint8) for f in range(9)]
    yield dict(H=H, hp_d=hp_d, hp_e=hp_e, dr=dr, ar=ar, er=er, tr_ref=tr_ref, enc=enc, dec=dec, attn=attn,
               tr=tr, frames=frames)
    for x in (tr, enc, dec, attn, menc):
        x.free()


def test_stream_every_stage_on_the_gpu_trajectory_and_free_running(oracle, backend, stream):
    import mem_attn_oracle
    import mem_enc_oracle
    import mem_prompt_oracle as mpo
    import sam_dec_oracle as dco
    s = stream
    H, tr, dec, attn = s["H"], s["tr"], s["dec"], s["attn"]
    N, S = H * H, 4 * H
    t = s["tr_ref"]
    mlp_w = [t[f"obj_ptr_proj.layers.{j}.weight"] for j in range(3)]
    mlp_b = [t[f"obj_ptr_proj.layers.{j}.bias"] for j in range(3)]
    tables = {"tpos_enc": t["mem_enc.tpos_enc"], "tpos_proj_w": t["obj_ptr_tpos_proj.weight"],
              "tpos_proj_b": t["obj_ptr_tpos_proj.bias"]}
    pe64 = mpo.sinusoidal_pe_2d(H, H, MD).reshape(N, MD)
    src_pos = mpo.sinusoidal_pe_2d(H, H, D).reshape(N, D)
    rq = mem_attn_oracle.axial_cis(D, H, H)
    chw = backend.alloc(3 * IMG * IMG * 4)
    shadow = mpo.MemBank(NMEM, NPTR)    # the free-running oracle loop's own bank (attention in float64)
    shadow32 = mpo.MemBank(NMEM, NPTR)  # the same loop with the attention in float32
    ious_free, ious_self, errs, dec_errs = [], [], {}, {}

    def ptr_of(tok, obj):
        return mpo.extract_obj_ptr(tok, obj, mlp_w, mlp_b, t["no_obj_ptr"], blend=True)

    def oracle_propagate(bank_slots, bank_ptrs, cur, curr):
        sel = mpo.select_memory_frames(len(bank_slots), NMEM)
        prompt, ppos, n_ptr = mpo.build_mem_prompt(D, MD, NMEM, NPTR, [bank_slots[k][2] for k in sel],
                                                   [pe64] * len(sel), [bank_slots[k][1] for k in sel],
                                                   [p[1] for p in bank_ptrs], [p[0] for p in bank_ptrs], cur,
                                                   **tables)
        return prompt, ppos, n_ptr, np.concatenate([rq] * len(sel))

    for f, rgb in enumerate(s["frames"]):
        backend.preprocess_sam2(backend.upload(rgb), W, HH, IMG, chw)
        tr.encode(chw)
        f2, f0, f1 = (np.ascontiguousarray(s["enc"].output_host(lvl)) for lvl in (2, 0, 1))
        curr = f2.reshape(N, D)
        if f == 0:
            iid = tr.add_instance(BOX, BOX_LABELS, W, HH)
            inst = tr.instance(iid)
            want = dco.decode(s["hp_d"], s["dr"], f2, f0, f1, BOX, BOX_LABELS, W, HH, IMG)
            errs["f0 mask"] = rel_err(inst["mask"], want[0][0])
            assert rel_err(inst["token"], want[3]) <= 1e-2
            assert abs(inst["obj"] - want[2]) <= 1e-2 * max(1.0, abs(want[2]))
            got_mask = tr.mask(iid, W, HH)
            assert dco.mask_iou(got_mask, dco.resize_threshold(want[0][0], W, HH)) >= 0.99
            slots, ptrs = tr.bank(iid)
            assert [(sl[0], sl[1]) for sl in slots] == [(0, True)] and [p[0] for p in ptrs] == [0]
            mem = mem_enc_oracle.encode(s["hp_e"], s["er"], synth_logits(got_mask, S), curr, inst["obj"])
            errs["f0 memory"] = rel_err(slots[0][2], mem)
            assert rel_err(ptrs[0][1], ptr_of(inst["token"], inst["obj"])) <= 1e-4
            # the oracle loop's frame 0 on the same encoder features
            o_mask = dco.resize_threshold(want[0][0], W, HH)
            for bank in (shadow, shadow32):
                bank.add_slot(mem_enc_oracle.encode(s["hp_e"], s["er"], synth_logits(o_mask, S), curr, want[2]), 0,
                              True)
                bank.add_ptr(ptr_of(want[3], want[2]), 0)
            ious_free.append(dco.mask_iou(got_mask, o_mask))
            ious_self.append(1.0)
            continue
        slots, ptrs = tr.bank(iid)
        cur = tr.frame_index
        tr.propagate()
        inst = tr.instance(iid)
        # (1) every stage on the GPU's own inputs
        prompt, ppos, n_ptr, rk = oracle_propagate(slots, ptrs, cur, curr)
        gp, gpp = tr.prompt(prompt.shape[0])
        assert np.array_equal(gp, prompt), f
        np.testing.assert_allclose(gpp, ppos, rtol=1e-5, atol=1e-5)
        cond = attn.output_host(N)
        want_cond = mem_attn_oracle.run(s["ar"], LAYERS, curr, src_pos, gp, gpp, rq, rk, n_ptr)
        errs[f"f{f} attention"] = rel_err(cond, want_cond)
        masks, iou, obj, _ = dec.outputs()
        wm, wiou, wobj, wtoks = dco.decode(s["hp_d"], s["dr"], cond, f0, f1, [], [], W, HH, IMG, tracking=True,
                                           all_tokens=True)
        dec_errs[f] = [rel_err(masks[m], wm[m]) for m in range(4)]
        assert np.abs(iou - wiou).max() <= 1e-2 and abs(obj - wobj) <= 1e-2 * max(1.0, abs(wobj))
        best = 1 + int(np.argmax(iou[1:]))
        if abs(np.sort(wiou[1:])[-1] - np.sort(wiou[1:])[-2]) > 2e-2:  # no near-tie: the same mask is kept
            assert best == 1 + int(np.argmax(wiou[1:]))
        assert np.array_equal(inst["mask"], masks[best]) and inst["iou"] == pytest.approx(iou[best])
        assert rel_err(inst["token"], wtoks[best]) <= 1e-2
        got_mask = tr.mask(iid, W, HH)
        assert dco.mask_iou(got_mask, dco.resize_threshold(wm[best], W, HH)) >= 0.99, f
        new_slots, new_ptrs = tr.bank(iid)
        assert new_slots[-1][0] == cur and not new_slots[-1][1] and len(new_slots) == min(len(slots) + 1, NMEM)
        assert new_slots[0][1]  # the conditioning frame is never evicted
        mem = mem_enc_oracle.encode(s["hp_e"], s["er"], inst["mask"], curr, inst["obj"])
        errs[f"f{f} memory"] = rel_err(new_slots[-1][2], mem)
        assert rel_err(new_ptrs[-1][1], ptr_of(inst["token"], inst["obj"])) <= 1e-4
        # (2) the oracle loops on their own banks
        kept = []
        for bank, dt in ((shadow, np.float64), (shadow32, np.float32)):
            prompt, ppos, n_ptr, rk = oracle_propagate(bank.slots, bank.ptrs, cur, curr)
            ocond = mem_attn_oracle.run(s["ar"], LAYERS, curr, src_pos, prompt, ppos, rq, rk, n_ptr, dt)
            om, oiou, oobj, otoks = dco.decode(s["hp_d"], s["dr"], ocond, f0, f1, [], [], W, HH, IMG,
                                               tracking=True, all_tokens=True)
            ob = 1 + int(np.argmax(oiou[1:]))
            bank.add_slot(mem_enc_oracle.encode(s["hp_e"], s["er"], om[ob], curr, oobj), cur, False)
            bank.add_ptr(ptr_of(otoks[ob], oobj), cur)
            kept.append(dco.resize_threshold(om[ob], W, HH))
        ious_free.append(dco.mask_iou(got_mask, kept[0]))
        ious_self.append(dco.mask_iou(kept[1], kept[0]))
    print("stage errors:", ", ".join(f"{k} {v:.2e}" for k, v in errs.items()))
    print("decoder mask-logit errors per frame:", {f: [f"{e:.1e}" for e in v] for f, v in dec_errs.items()})
    assert max(errs.values()) <= 1e-2, errs
    print("free-running mask IoU per frame, GPU vs oracle:", ", ".join(f"{v:.4f}" for v in ious_free))
    print("free-running mask IoU per frame, oracle f32 vs f64 attention:", ", ".join(f"{v:.4f}" for v in ious_self))
    assert len(tr.bank(iid)[0]) == NMEM and tr.frame_index == 8
    gpu_dis = float(np.mean(1.0 - np.asarray(ious_free)))
    own_dis = float(np.mean(1.0 - np.asarray(ious_self)))
    assert gpu_dis <= max(1.5 * own_dis, 0.01), (ious_free, ious_self)
