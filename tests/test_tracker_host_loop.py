"""The tracker's host-side state driving the memory attention over a short stream, on the CPU: the
native memory bank (sam3b200_mem_bank_*) supplies each frame's prompt, positional codes, pointer-token
count and RoPE tables in exactly the layout the memory attention takes (sam3b200_mem_attn_run and its
oracle share it), pointers come from sam3b200_extract_obj_ptr, and the attention output feeds the next
slot.  The memory attention and the memory encoder are the CPU oracle here (their B200 kernels are
checked against the same oracle in test_mem_attn_gpu.py / test_mem_enc_gpu.py); the bank's prompt is
checked against the restated sam3_build_prompt_and_pos at every frame."""
import numpy as np

import mem_attn_oracle
import mem_prompt_oracle as mpo
from test_mem_attn_gpu import D, LAYERS, MD, make_mem_tensors

HP = {"d_model": D, "mem_dim": MD, "num_maskmem": 7, "max_obj_ptrs": 16}


def test_stream_of_frames_through_the_host_bank(oracle, b200):
    rng = np.random.default_rng(21)
    H, n_frames = 6, 9
    N = H * H
    _, ref = make_mem_tensors(oracle, seed=3)
    tables = {"tpos_enc": rng.normal(0, 0.1, size=(7, MD)).astype(np.float32),
              "tpos_proj_w": rng.normal(0, 0.05, size=(MD, D)).astype(np.float32),
              "tpos_proj_b": rng.normal(0, 0.1, size=MD).astype(np.float32)}
    mlp_w = [rng.normal(0, 1 / 16, size=(D, D)).astype(np.float32) for _ in range(3)]
    mlp_b = [rng.normal(0, 0.1, size=D).astype(np.float32) for _ in range(3)]
    no_ptr = rng.normal(0, 1, size=D).astype(np.float32)
    to_mem = rng.normal(0, 1 / 16, size=(D, MD)).astype(np.float32)  # stand-in for the memory encoder
    src_pos = b200.sinusoidal_pe_2d(H, H, D).reshape(N, D)
    bank = b200.MemBank(HP, H)
    shadow = mpo.MemBank(7, 16)
    pe64 = mpo.sinusoidal_pe_2d(H, H, MD).reshape(N, MD)
    for f in range(n_frames):
        curr = rng.normal(0, 1, size=(N, D)).astype(np.float32)
        if f == 0:
            cond = curr  # the prompted frame is decoded without memory
        else:
            prompt, ppos, n_ptr = bank.prompt(f, **tables)
            rq, rk = bank.rope()
            sel = mpo.select_memory_frames(len(shadow.slots), 7)
            want = mpo.build_mem_prompt(D, MD, 7, 16, [shadow.slots[s][2] for s in sel], [pe64] * len(sel),
                                        [shadow.slots[s][1] for s in sel], [p[1] for p in shadow.ptrs],
                                        [p[0] for p in shadow.ptrs], f, **tables)
            assert np.array_equal(prompt, want[0]) and n_ptr == want[2]
            np.testing.assert_allclose(ppos, want[1], rtol=1e-5, atol=1e-5)
            assert rk.shape[0] == prompt.shape[0] - n_ptr == len(sel) * N
            cond = mem_attn_oracle.run(ref, LAYERS, curr, src_pos, prompt, ppos, rq, rk, n_ptr)
            assert cond.shape == (N, D) and np.isfinite(cond).all()
        score = 1.0 if f % 4 != 3 else -1.0  # the object leaves the frame now and then
        ptr = b200.extract_obj_ptr(cond[0], score, mlp_w, mlp_b, no_ptr)
        if score <= 0:
            assert np.array_equal(ptr, no_ptr)
        mem = (cond @ to_mem).astype(np.float32)
        bank.add_slot(mem, f, f == 0)
        shadow.add_slot(mem, f, f == 0)
        bank.add_ptr(ptr, f)
        shadow.add_ptr(ptr, f)
    slots, ptr_frames = bank.state()
    assert slots[0] == (0, True) and len(slots) == 7 and slots[-1] == (n_frames - 1, False)
    assert ptr_frames == list(range(n_frames))
    bank.free()
