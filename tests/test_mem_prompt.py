"""Host-side memory of the tracker (sam3b200_select_memory_frames, sam3b200_build_mem_prompt,
sam3b200_extract_obj_ptr, sam3b200_sinusoidal_pe_2d, sam3b200_mem_bank_*) against the CPU
restatement of sam3_select_memory_frames, sam3_build_prompt_and_pos, sam3_extract_obj_ptr_cpu,
sam3_sinusoidal_pe_2d and the bank eviction rules (oracle/mem_prompt_oracle.py).  No GPU: the reference runs this on the
CPU between the decoder and the memory-attention graphs, and so does this library."""
import numpy as np
import pytest

import mem_prompt_oracle as mpo

HP = {"d_model": 256, "mem_dim": 64, "num_maskmem": 7, "max_obj_ptrs": 16}  # SAM2 / SAM3 trackers


@pytest.mark.parametrize("max_slots", range(0, 10))
def test_select_memory_frames_matches_the_restatement(b200, max_slots):
    for bank in range(0, 41):
        got = b200.select_memory_frames(bank, max_slots)
        assert got == mpo.select_memory_frames(bank, max_slots), (bank, max_slots)
        if bank:
            assert got == sorted(set(got))
            if bank > max_slots:
                assert got[0] == 0 and got[-1] == bank - 1  # the first and the newest slot always take part
                assert len(got) <= max(max_slots, 2)


def test_select_memory_frames_known_cases(b200):
    """Hand-derived from the reference rule: 7 slots of a 20-slot bank: step 18 / 6 = 3 ->
    1 + 3, 1 + 6, ... clamped to 18."""
    assert b200.select_memory_frames(5, 7) == [0, 1, 2, 3, 4]
    assert b200.select_memory_frames(20, 7) == [0, 4, 7, 10, 13, 16, 19]
    assert b200.select_memory_frames(9, 7) == [0, 2, 3, 4, 5, 6, 8]  # step 7 / 6: 1 + 1.16.. -> 2, ..., 1 + 5.83 -> 6


def _case(rng, n_slots, slot_tokens, n_ptrs, cond=(0,), with_tables=True):
    MD, D = HP["mem_dim"], HP["d_model"]
    feats = [rng.normal(0, 1, size=(slot_tokens, MD)).astype(np.float32) for _ in range(n_slots)]
    pes = [rng.normal(0, 1, size=(slot_tokens, MD)).astype(np.float32) for _ in range(n_slots)]
    is_cond = [1 if s in cond else 0 for s in range(n_slots)]
    ptrs = [rng.normal(0, 1, size=D).astype(np.float32) for _ in range(n_ptrs)]
    frames = list(rng.integers(0, 30, size=n_ptrs))
    tables = {}
    if with_tables:
        tables = {"tpos_enc": rng.normal(0, 0.1, size=(HP["num_maskmem"], MD)).astype(np.float32),
                  "tpos_proj_w": rng.normal(0, 0.05, size=(MD, D)).astype(np.float32),
                  "tpos_proj_b": rng.normal(0, 0.1, size=MD).astype(np.float32)}
    return feats, pes, is_cond, ptrs, frames, tables


def _check(b200, case, cur_frame):
    feats, pes, is_cond, ptrs, frames, tables = case
    got_p, got_pos, got_n = b200.build_mem_prompt(HP, feats, pes, is_cond, ptrs, frames, cur_frame, **tables)
    ref_p, ref_pos, ref_n = mpo.build_mem_prompt(HP["d_model"], HP["mem_dim"], HP["num_maskmem"],
                                                 HP["max_obj_ptrs"], feats, pes, is_cond, ptrs, frames, cur_frame,
                                                 **tables)
    assert got_n == ref_n and got_p.shape == ref_p.shape
    m_spatial = got_p.shape[0] - got_n
    assert np.array_equal(got_p, ref_p)                           # copies
    assert np.array_equal(got_pos[:m_spatial], ref_pos[:m_spatial])  # one f32 add per element
    # pointer codes: libm sin/cos/pow and an f32 dot against numpy's float32 / float64 -- 1e-5
    np.testing.assert_allclose(got_pos[m_spatial:], ref_pos[m_spatial:], rtol=1e-5, atol=1e-5)
    return got_p, got_pos, got_n


def test_config5_prompt(b200):
    """7 memory frames of 64 x 64 tokens (frame 0 conditioning) + 20 pointers, 16 of them used:
    28,736 prompt tokens, the memory attention's M at config 5."""
    rng = np.random.default_rng(5)
    case = _case(rng, 7, 64 * 64, 20)
    case[4][:3] = [10, 9, 11]  # distance 0 -> 1, and 1 on either side
    p, pos, n = _check(b200, case, cur_frame=10)
    assert p.shape == (7 * 4096 + 16 * 4, 64) and n == 64
    assert np.array_equal(pos[:4096], case[1][0] + case[5]["tpos_enc"][6])  # conditioning slot: t = 0
    assert np.array_equal(pos[4096:8192], case[1][1] + case[5]["tpos_enc"][6 - 6])  # t = 7 - 1 = 6 -> row 0
    # the four tokens of a pointer share its positional code and carry its 256 values in order
    assert np.array_equal(pos[-64:-60], np.repeat(pos[-64][None], 4, 0))
    assert np.array_equal(p[7 * 4096:7 * 4096 + 4].reshape(-1), case[3][0])


def test_slots_beyond_the_temporal_table_get_no_temporal_code(b200):
    """With 8 slots the oldest non-conditioning one has t = 8 >= num_maskmem: spatial code only."""
    rng = np.random.default_rng(6)
    case = _case(rng, 8, 16, 3, cond=())
    _, pos, _ = _check(b200, case, cur_frame=4)
    assert np.array_equal(pos[:16], case[1][0])


@pytest.mark.parametrize("n_slots,n_ptrs,tables", [(0, 5, True), (3, 0, True), (2, 2, False), (0, 0, True)])
def test_edge_shapes(b200, n_slots, n_ptrs, tables):
    rng = np.random.default_rng(n_slots * 10 + n_ptrs)
    _check(b200, _case(rng, n_slots, 32, n_ptrs, with_tables=tables), cur_frame=7)


def test_rejects_bad_arguments(b200):
    L = b200.lib()
    assert L.sam3b200_build_mem_prompt(None, 0, 0, None, None, None, 0, None, None, 0, None, None, None, None,
                                       None, 0, None) == -1
    assert "hyper-parameters" in b200.last_error()
    assert L.sam3b200_select_memory_frames(20, 7, None, 0) == -1
    hp = b200.MemPromptHparams(256, 64, 7, 16)
    import ctypes
    n = ctypes.c_int32()
    buf = np.empty((4, 64), np.float32)
    ptr = np.zeros(256, np.float32)
    arr = (ctypes.c_void_p * 1)(ptr.ctypes.data)
    frames = np.zeros(1, np.int32)
    # one pointer = 4 tokens, room for 3
    assert L.sam3b200_build_mem_prompt(ctypes.byref(hp), 0, 0, None, None, None, 1, arr, frames.ctypes.data, 0,
                                       None, None, None, buf.ctypes.data, buf.ctypes.data, 3, ctypes.byref(n)) == -1
    assert "room for 3" in b200.last_error()


@pytest.mark.parametrize("score,blend", [(2.5, False), (-0.3, False), (0.0, False), (1.0, True), (-1.0, True)])
def test_extract_obj_ptr(b200, score, blend):
    """sam3_extract_obj_ptr_cpu: MLP pointer for a present object, no_obj_ptr (SAM3) or the blend (SAM2)."""
    rng = np.random.default_rng(int(abs(score) * 10) + blend)
    D = 256
    tok = rng.normal(0, 1, size=D).astype(np.float32)
    w = [rng.normal(0, 1 / 16, size=(D, D)).astype(np.float32) for _ in range(3)]
    b = [rng.normal(0, 0.1, size=D).astype(np.float32) for _ in range(3)]
    nop = rng.normal(0, 1, size=D).astype(np.float32)
    got = b200.extract_obj_ptr(tok, score, w, b, nop, blend)
    ref = mpo.extract_obj_ptr(tok, score, w, b, nop, blend)
    if score <= 0:
        assert np.array_equal(got, nop)  # the absent-object pointer, exactly
    else:
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)
        assert not np.array_equal(got, nop)


@pytest.mark.parametrize("H,W,d", [(72, 72, 64), (64, 64, 256), (5, 7, 16)])
def test_sinusoidal_pe_2d(b200, H, W, d):
    got = b200.sinusoidal_pe_2d(H, W, d)
    ref = mpo.sinusoidal_pe_2d(H, W, d)
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6)  # libm vs numpy float32 sin / cos / pow
    assert np.array_equal(got[0, :, : d // 2], np.repeat(got[0, :1, : d // 2], W, 0))  # y half constant along x


def _stream(b200, cond_frames, n_frames, H=8):
    """Feed a bank and its restatement the slots and pointers of n_frames frames; compare after each."""
    rng = np.random.default_rng(len(cond_frames) * 100 + n_frames)
    bank = b200.MemBank(HP, H)
    ref = mpo.MemBank(HP["num_maskmem"], HP["max_obj_ptrs"])
    tables = {"tpos_enc": rng.normal(0, 0.1, size=(7, 64)).astype(np.float32),
              "tpos_proj_w": rng.normal(0, 0.05, size=(64, 256)).astype(np.float32),
              "tpos_proj_b": rng.normal(0, 0.1, size=64).astype(np.float32)}
    pe = mpo.sinusoidal_pe_2d(H, H, 64).reshape(-1, 64)
    for f in range(n_frames):
        if f:  # the prompt frame f attends to: what the bank held after frame f - 1
            got = bank.prompt(f, **tables)
            sel = mpo.select_memory_frames(len(ref.slots), HP["num_maskmem"])
            want = mpo.build_mem_prompt(256, 64, 7, 16, [ref.slots[s][2] for s in sel], [pe] * len(sel),
                                        [ref.slots[s][1] for s in sel], [p[1] for p in ref.ptrs],
                                        [p[0] for p in ref.ptrs], f, **tables)
            assert got[2] == want[2] and got[0].shape == want[0].shape
            assert np.array_equal(got[0], want[0])
            np.testing.assert_allclose(got[1], want[1], rtol=1e-5, atol=1e-5)
        feats = rng.normal(0, 1, size=(H * H, 64)).astype(np.float32)
        ptr = rng.normal(0, 1, size=256).astype(np.float32)
        bank.add_slot(feats, f, f in cond_frames)
        ref.add_slot(feats, f, f in cond_frames)
        bank.add_ptr(ptr, f)
        ref.add_ptr(ptr, f)
        slots, ptrs = bank.state()
        assert slots == [(s[0], s[1]) for s in ref.slots]
        assert ptrs == [p[0] for p in ref.ptrs]
    return bank


def test_mem_bank_video_stream(b200):
    """16 frames, box prompt on frame 0 (conditioning) and a correction on frame 9: at most 7 slots,
    conditioning slots kept, the oldest other slot dropped first; 16 newest pointers."""
    bank = _stream(b200, {0, 9}, 20)
    slots, ptrs = bank.state()
    assert len(slots) == 7 and (0, True) in slots and (9, True) in slots and slots[-1] == (19, False)
    assert ptrs == list(range(4, 20))
    bank.free()


def test_mem_bank_all_conditioning(b200):
    """Every frame prompted: no non-conditioning slot to drop, so slot 1 goes (frame 0 stays)."""
    bank = _stream(b200, set(range(12)), 12)
    slots, _ = bank.state()
    assert [s[0] for s in slots] == [0] + list(range(6, 12))
    bank.free()


@pytest.mark.parametrize("dim,ex,ey", [(256, 64, 64), (256, 72, 72), (64, 24, 24), (64, 72, 72)])
def test_axial_cis_matches_the_tables_the_gpu_tests_use(b200, dim, ex, ey):
    """sam3_compute_axial_cis: the tracker's (d 256) and the ViT's (d 64) RoPE tables, against the oracle table
    the memory-attention parity tests feed the GPU."""
    import mem_attn_oracle
    # libm powf vs numpy's float32 power can differ by an ulp in a frequency, which the position (up to 71)
    # multiplies: a few 1e-6 in the angle
    np.testing.assert_allclose(b200.axial_cis(dim, ex, ey), mem_attn_oracle.axial_cis(dim, ex, ey), rtol=0, atol=1e-5)


def test_mem_bank_rope(b200):
    """rope_q = the H x H table; rope_k = that table once per selected slot; none for an empty bank."""
    import mem_attn_oracle
    H = 8
    bank = b200.MemBank(HP, H)
    rq, rk = bank.rope()
    assert rk is None
    np.testing.assert_allclose(rq, mem_attn_oracle.axial_cis(256, H, H), rtol=0, atol=1e-5)
    for f in range(10):
        bank.add_slot(np.zeros((H * H, 64), np.float32), f, f == 0)
    rq, rk = bank.rope()
    assert rk.shape == (7 * H * H, 128, 2)
    assert np.array_equal(rk, np.concatenate([rq] * 7))
    bank.free()
