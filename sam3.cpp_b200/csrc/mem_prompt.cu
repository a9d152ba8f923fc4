// mem_prompt.cu -- host-side preparation of the memory attention's inputs for
// one propagated frame, as sam3_propagate_single does it before it builds its
// graph (sam3.cpp:11175-11233): which memory-bank slots take part
// (sam3_select_memory_frames, :9427-9451), their temporal positions (a
// conditioning frame 0, the others n_sel - s), the pointer distances
// (max(1, |frame - pointer frame|), at most max_obj_ptrs pointers), and the
// prompt / prompt_pos token rows with the object-pointer tokens
// (sam3_build_prompt_and_pos, :9126-9217, with the 1-D sine code of
// sam3_get_1d_sine_pe, :3641-3651).  The reference runs this on the CPU
// between two graphs; it stays host code here and feeds
// sam3b200_mem_attn_run's prompt, prompt_pos and n_obj_ptr_tokens.
#include "../../include/sam3_b200.h"
#include "backend_impl.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

namespace {

// sam3_get_1d_sine_pe: out[i] = sin(pos / T^(2 floor(i/2) / (dim/2))), out[dim/2 + i] = cos(...)
void sine_pe_1d(float *out, float pos, int dim) {
    const int half = dim / 2;
    for (int i = 0; i < half; ++i) {
        const int paired = i & ~1;
        const float dim_t = powf(10000.0f, static_cast<float>(paired) / static_cast<float>(half));
        const float val = pos / dim_t;
        out[i] = sinf(val);
        out[half + i] = cosf(val);
    }
}

}  // namespace

// The positional row of an object pointer's tokens: the 1-D sine code of max(1, |frame distance|) / 15
// (d_model wide) through obj_ptr_tpos_proj (weight ggml [D, MD]: w[j * D + i]; bias [MD]; NULL = zeros).
void b200::obj_ptr_pos_row(int D, int MD, int rel, const float *w, const float *b, float *out) {
    std::vector<float> sine(static_cast<size_t>(D));
    sine_pe_1d(sine.data(), static_cast<float>(rel) / 15.0f, D);
    for (int j = 0; j < MD; ++j) {
        float sum = b ? b[j] : 0.0f;
        for (int i = 0; i < D; ++i) sum += (w ? w[i + static_cast<int64_t>(j) * D] : 0.0f) * sine[i];
        out[j] = sum;
    }
}

using b200::set_error;

extern "C" int sam3b200_select_memory_frames(int bank_size, int max_slots, int32_t *out, int cap) {
    if (bank_size < 0 || max_slots < 0 || (cap > 0 && !out)) {
        set_error("select_memory_frames: bad arguments");
        return -1;
    }
    std::vector<int32_t> sel;
    if (bank_size <= max_slots) {
        for (int i = 0; i < bank_size; ++i) sel.push_back(i);
    } else {
        // the first and the newest slot, then evenly spaced ones between them
        sel.push_back(0);
        sel.push_back(bank_size - 1);
        const int remaining = max_slots - 2;
        if (remaining > 0) {
            const float step = static_cast<float>(bank_size - 2) / static_cast<float>(remaining + 1);
            for (int i = 0; i < remaining; ++i) {
                int idx = 1 + static_cast<int>(static_cast<float>(i + 1) * step);
                sel.push_back(std::min(idx, bank_size - 2));
            }
        }
        std::sort(sel.begin(), sel.end());
        sel.erase(std::unique(sel.begin(), sel.end()), sel.end());
    }
    if (static_cast<int>(sel.size()) > cap) {
        set_error("select_memory_frames: %d slots selected, room for %d", static_cast<int>(sel.size()), cap);
        return -1;
    }
    std::copy(sel.begin(), sel.end(), out);
    return static_cast<int>(sel.size());
}

extern "C" int64_t sam3b200_build_mem_prompt(const sam3b200_mem_prompt_hparams *hp, int n_slots, int slot_tokens,
                                             const float *const *slot_feats, const float *const *slot_pes,
                                             const int32_t *slot_is_cond, int n_ptrs, const float *const *obj_ptrs,
                                             const int32_t *ptr_frames, int cur_frame, const float *tpos_enc,
                                             const float *tpos_proj_w, const float *tpos_proj_b, float *prompt,
                                             float *prompt_pos, int64_t cap_tokens, int32_t *n_ptr_tokens) {
    if (!hp || hp->mem_dim <= 0 || hp->d_model <= 0 || hp->d_model % hp->mem_dim != 0 || hp->d_model % 2 != 0 ||
        hp->num_maskmem < 0 || hp->max_obj_ptrs < 0) {
        set_error("build_mem_prompt: bad hyper-parameters");
        return -1;
    }
    if (n_slots < 0 || slot_tokens < 0 || n_ptrs < 0 || (n_slots > 0 && (!slot_feats || !slot_pes || !slot_is_cond)) ||
        (n_ptrs > 0 && (!obj_ptrs || !ptr_frames)) || !prompt || !prompt_pos || !n_ptr_tokens) {
        set_error("build_mem_prompt: null argument");
        return -1;
    }
    const int MD = hp->mem_dim, D = hp->d_model, split = D / MD;
    const int P = std::min(n_ptrs, hp->max_obj_ptrs);
    const int64_t m_spatial = static_cast<int64_t>(n_slots) * slot_tokens;
    const int64_t m_total = m_spatial + static_cast<int64_t>(P) * split;
    if (m_total > cap_tokens) {
        set_error("build_mem_prompt: %lld prompt tokens, room for %lld", static_cast<long long>(m_total),
                  static_cast<long long>(cap_tokens));
        return -1;
    }
    for (int s = 0; s < n_slots; ++s)
        if (!slot_feats[s] || !slot_pes[s]) {
            set_error("build_mem_prompt: slot %d has no features or positional code", s);
            return -1;
        }
    for (int p = 0; p < P; ++p)
        if (!obj_ptrs[p]) {
            set_error("build_mem_prompt: object pointer %d is null", p);
            return -1;
        }

    // 1. spatial memory tokens: features as they are; positional code = spatial code + the slot's
    //    temporal code (maskmem_tpos_enc[num_maskmem - t - 1] for t in [0, num_maskmem); none beyond)
    //    (a model without the table adds zeros, as the reference does)
    const std::vector<float> zeros(MD, 0.0f);
    for (int s = 0; s < n_slots; ++s) {
        const int t = slot_is_cond[s] ? 0 : n_slots - s;
        const float *te = nullptr;
        if (t >= 0 && t < hp->num_maskmem)
            te = tpos_enc ? tpos_enc + static_cast<int64_t>(hp->num_maskmem - t - 1) * MD : zeros.data();
        const int64_t base = static_cast<int64_t>(s) * slot_tokens * MD;
        std::copy(slot_feats[s], slot_feats[s] + static_cast<int64_t>(slot_tokens) * MD, prompt + base);
        for (int64_t n = 0; n < slot_tokens; ++n)
            for (int d = 0; d < MD; ++d)
                prompt_pos[base + n * MD + d] = te ? slot_pes[s][n * MD + d] + te[d] : slot_pes[s][n * MD + d];
    }

    // 2. object pointers: each D-wide pointer as D / MD tokens; their positional code is the 1-D sine
    //    code of the frame distance / 15 projected D -> MD (obj_ptr_tpos_proj), shared by the pointer's tokens
    std::vector<float> proj(MD);
    int64_t tok = m_spatial;
    for (int p = 0; p < P; ++p) {
        const int rel = std::max(1, std::abs(cur_frame - ptr_frames[p]));
        b200::obj_ptr_pos_row(D, MD, rel, tpos_proj_w, tpos_proj_b, proj.data());
        for (int t = 0; t < split; ++t, ++tok)
            for (int d = 0; d < MD; ++d) {
                prompt[tok * MD + d] = obj_ptrs[p][t * MD + d];
                prompt_pos[tok * MD + d] = proj[d];
            }
    }
    *n_ptr_tokens = P * split;
    return m_total;
}

// sam3_extract_obj_ptr_cpu (sam3.cpp:9347-9420): the object pointer a propagated (or prompted) frame adds
// to the pointer bank -- the decoder's SAM output token through obj_ptr_proj (three D x D layers, ReLU
// after the first two), replaced by no_obj_ptr when the object-score logit says the object is absent
// (SAM3: score <= 0 -> no_obj_ptr, the MLP skipped; SAM2 / EdgeTAM with fixed_no_obj_ptr: the blend
// l * mlp + (1 - l) * no_obj_ptr with l = [score > 0]).  Weights f32 row-major [out][in] (ggml [in, out]).
extern "C" int sam3b200_extract_obj_ptr(int d_model, int blend, const float *sam_token, float obj_score,
                                        const float *const *w, const float *const *b, const float *no_obj_ptr,
                                        float *out) {
    const int D = d_model;
    if (D <= 0 || !sam_token || !w || !b || !no_obj_ptr || !out || !w[0] || !w[1] || !w[2] || !b[0] || !b[1] ||
        !b[2]) {
        set_error("extract_obj_ptr: null argument or bad width");
        return SAM3B200_STATUS_FAILED;
    }
    if (!blend && obj_score <= 0.0f) {
        std::copy(no_obj_ptr, no_obj_ptr + D, out);
        return SAM3B200_STATUS_SUCCESS;
    }
    std::vector<float> h(sam_token, sam_token + D), tmp(D);
    for (int j = 0; j < 3; ++j) {
        for (int o = 0; o < D; ++o) {
            float sum = b[j][o];
            for (int i = 0; i < D; ++i) sum += w[j][static_cast<int64_t>(o) * D + i] * h[i];
            tmp[o] = j < 2 ? std::max(0.0f, sum) : sum;
        }
        std::swap(h, tmp);
    }
    if (blend) {
        const float l = obj_score > 0.0f ? 1.0f : 0.0f;
        for (int i = 0; i < D; ++i) out[i] = l * h[i] + (1.0f - l) * no_obj_ptr[i];
    } else {
        std::copy(h.begin(), h.end(), out);
    }
    return SAM3B200_STATUS_SUCCESS;
}

// sam3_sinusoidal_pe_2d (sam3.cpp:3601-3637): PositionEmbeddingSine with normalised positions
// (p + 1) / n * 2 pi, temperature 1e4; channels [0, d/2) encode y, [d/2, d) encode x; pairs of
// channels share a frequency (sin on even, cos on odd).  out [H][W][d_model].
extern "C" int sam3b200_sinusoidal_pe_2d(int H, int W, int d_model, float *out) {
    if (H <= 0 || W <= 0 || d_model <= 0 || d_model % 2 != 0 || !out) {
        set_error("sinusoidal_pe_2d: bad arguments");
        return SAM3B200_STATUS_FAILED;
    }
    const int half = d_model / 2;
    const float scale = 2.0f * static_cast<float>(M_PI);
    std::vector<float> dim_t(half);
    for (int i = 0; i < half; ++i) dim_t[i] = powf(10000.0f, static_cast<float>(i & ~1) / static_cast<float>(half));
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            const float py = (static_cast<float>(y + 1) / static_cast<float>(H)) * scale;
            const float px = (static_cast<float>(x + 1) / static_cast<float>(W)) * scale;
            float *o = out + (static_cast<int64_t>(y) * W + x) * d_model;
            for (int i = 0; i < half; ++i) {
                o[i] = i % 2 == 0 ? sinf(py / dim_t[i]) : cosf(py / dim_t[i]);
                o[half + i] = i % 2 == 0 ? sinf(px / dim_t[i]) : cosf(px / dim_t[i]);
            }
        }
    return SAM3B200_STATUS_SUCCESS;
}

// The memory of one tracked object in one video stream: the slots sam3_encode_memory stores
// (features [H*H][MD] with the stream's sinusoidal code, frame, conditioning flag; at most num_maskmem,
// evicting the oldest non-conditioning slot first, else slot 1 -- sam3.cpp:11700-11711) and the object
// pointers sam3_store_obj_ptr keeps (at most max_obj_ptrs, oldest first out -- :11716-11734).
struct sam3b200_mem_bank {
    sam3b200_mem_prompt_hparams hp{};
    int H = 0;
    std::vector<float> pe;  // sinusoidal code shared by every slot [H*H][MD]
    struct Slot {
        std::vector<float> feats;
        int frame;
        int cond;
    };
    std::vector<Slot> slots;
    std::vector<std::pair<int, std::vector<float>>> ptrs;
};

extern "C" sam3b200_mem_bank *sam3b200_mem_bank_create(const sam3b200_mem_prompt_hparams *hp, int feat_size) {
    if (!hp || hp->mem_dim <= 0 || hp->d_model <= 0 || hp->d_model % hp->mem_dim != 0 || hp->mem_dim % 2 != 0 ||
        hp->num_maskmem <= 0 || hp->max_obj_ptrs < 0 || feat_size <= 0 || feat_size > 4096) {
        set_error("mem_bank_create: bad hyper-parameters");
        return nullptr;
    }
    auto *b = new sam3b200_mem_bank();
    b->hp = *hp;
    b->H = feat_size;
    b->pe.resize(static_cast<size_t>(feat_size) * feat_size * hp->mem_dim);
    sam3b200_sinusoidal_pe_2d(feat_size, feat_size, hp->mem_dim, b->pe.data());
    return b;
}

extern "C" void sam3b200_mem_bank_free(sam3b200_mem_bank *b) { delete b; }

extern "C" int sam3b200_mem_bank_add_slot(sam3b200_mem_bank *b, const float *feats, int frame, int is_cond) {
    if (!b || !feats) {
        set_error("mem_bank_add_slot: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    const size_t n = static_cast<size_t>(b->H) * b->H * b->hp.mem_dim;
    b->slots.push_back({std::vector<float>(feats, feats + n), frame, is_cond ? 1 : 0});
    while (static_cast<int>(b->slots.size()) > b->hp.num_maskmem) {
        auto it = std::find_if(b->slots.begin(), b->slots.end(), [](const sam3b200_mem_bank::Slot &s) {
            return !s.cond;
        });
        b->slots.erase(it != b->slots.end() ? it : b->slots.begin() + 1);
    }
    return SAM3B200_STATUS_SUCCESS;
}

extern "C" int sam3b200_mem_bank_add_ptr(sam3b200_mem_bank *b, const float *ptr, int frame) {
    if (!b || !ptr) {
        set_error("mem_bank_add_ptr: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    b->ptrs.emplace_back(frame, std::vector<float>(ptr, ptr + b->hp.d_model));
    while (static_cast<int>(b->ptrs.size()) > b->hp.max_obj_ptrs) b->ptrs.erase(b->ptrs.begin());
    return SAM3B200_STATUS_SUCCESS;
}

extern "C" int sam3b200_mem_bank_state(const sam3b200_mem_bank *b, int32_t *slot_frames, int32_t *slot_cond,
                                       int slot_cap, int32_t *ptr_frames, int ptr_cap, int32_t *n_ptrs) {
    if (!b || !n_ptrs) {
        set_error("mem_bank_state: null argument");
        return -1;
    }
    const int ns = static_cast<int>(b->slots.size()), np = static_cast<int>(b->ptrs.size());
    for (int i = 0; i < ns && i < slot_cap; ++i) {
        if (slot_frames) slot_frames[i] = b->slots[i].frame;
        if (slot_cond) slot_cond[i] = b->slots[i].cond;
    }
    for (int i = 0; i < np && i < ptr_cap; ++i)
        if (ptr_frames) ptr_frames[i] = b->ptrs[i].first;
    *n_ptrs = np;
    return ns;
}

extern "C" int64_t sam3b200_mem_bank_prompt(const sam3b200_mem_bank *b, int cur_frame, const float *tpos_enc,
                                            const float *tpos_proj_w, const float *tpos_proj_b, float *prompt,
                                            float *prompt_pos, int64_t cap_tokens, int32_t *n_ptr_tokens) {
    if (!b) {
        set_error("mem_bank_prompt: null bank");
        return -1;
    }
    const int ns = static_cast<int>(b->slots.size());
    std::vector<int32_t> sel(std::max(ns, 2));
    const int n_sel = sam3b200_select_memory_frames(ns, b->hp.num_maskmem, sel.data(), static_cast<int>(sel.size()));
    if (n_sel < 0) return -1;
    std::vector<const float *> feats(n_sel), pes(n_sel);
    std::vector<int32_t> cond(n_sel);
    for (int s = 0; s < n_sel; ++s) {
        feats[s] = b->slots[sel[s]].feats.data();
        pes[s] = b->pe.data();
        cond[s] = b->slots[sel[s]].cond;
    }
    const int np = static_cast<int>(b->ptrs.size());
    std::vector<const float *> ptrs(np);
    std::vector<int32_t> frames(np);
    for (int p = 0; p < np; ++p) {
        ptrs[p] = b->ptrs[p].second.data();
        frames[p] = b->ptrs[p].first;
    }
    return sam3b200_build_mem_prompt(&b->hp, n_sel, b->H * b->H, feats.data(), pes.data(), cond.data(), np,
                                     ptrs.data(), frames.data(), cur_frame, tpos_enc, tpos_proj_w, tpos_proj_b,
                                     prompt, prompt_pos, cap_tokens, n_ptr_tokens);
}

// sam3_compute_axial_cis (sam3.cpp:3559-3590): per position idx of an end_x x end_y map, dim/4 x frequencies
// then dim/4 y frequencies 1 / theta^(4i / dim), stored as (cos, sin) pairs: out [N][dim/2][2].  The
// tracker's RoPE tables (sam3_ensure_tracker_pe_caches, :11140-11152) are this table unchanged.
extern "C" int sam3b200_axial_cis(int dim, int end_x, int end_y, float theta, float scale_pos, float *out) {
    if (dim <= 0 || dim % 4 != 0 || end_x <= 0 || end_y <= 0 || !out) {
        set_error("axial_cis: bad arguments");
        return SAM3B200_STATUS_FAILED;
    }
    const int q = dim / 4;
    std::vector<float> freqs(q);
    for (int i = 0; i < q; ++i) freqs[i] = 1.0f / powf(theta, static_cast<float>(i * 4) / static_cast<float>(dim));
    const int64_t N = static_cast<int64_t>(end_x) * end_y;
    for (int64_t idx = 0; idx < N; ++idx) {
        const float tx = static_cast<float>(idx % end_x) * scale_pos;
        const float ty = static_cast<float>(idx / end_x) * scale_pos;
        float *o = out + idx * dim;
        for (int i = 0; i < q; ++i) {
            o[2 * i] = cosf(tx * freqs[i]);
            o[2 * i + 1] = sinf(tx * freqs[i]);
            o[2 * q + 2 * i] = cosf(ty * freqs[i]);
            o[2 * q + 2 * i + 1] = sinf(ty * freqs[i]);
        }
    }
    return SAM3B200_STATUS_SUCCESS;
}

// The memory attention's RoPE inputs for the bank's current prompt: rope_q = the H x H table of d_model
// (theta 1e4), rope_k = that table once per selected slot (sam3_propagate_single, :11240-11275, standard
// path).  rope_k needs n_selected * H * H * d_model floats; returns the spatial key count (0: no rope_k).
extern "C" int64_t sam3b200_mem_bank_rope(const sam3b200_mem_bank *b, float *rope_q, float *rope_k,
                                          int64_t cap_k_tokens) {
    if (!b || !rope_q) {
        set_error("mem_bank_rope: null argument");
        return -1;
    }
    const int D = b->hp.d_model, HH = b->H * b->H;
    if (sam3b200_axial_cis(D, b->H, b->H, 10000.0f, 1.0f, rope_q) != SAM3B200_STATUS_SUCCESS) return -1;
    const int ns = static_cast<int>(b->slots.size());
    std::vector<int32_t> sel(std::max(ns, 2));
    const int n_sel = sam3b200_select_memory_frames(ns, b->hp.num_maskmem, sel.data(), static_cast<int>(sel.size()));
    if (n_sel < 0) return -1;
    const int64_t m_spatial = static_cast<int64_t>(n_sel) * HH;
    if (m_spatial > 0) {
        if (!rope_k || m_spatial > cap_k_tokens) {
            set_error("mem_bank_rope: %lld spatial keys, room for %lld", static_cast<long long>(m_spatial),
                      static_cast<long long>(rope_k ? cap_k_tokens : 0));
            return -1;
        }
        for (int s = 0; s < n_sel; ++s)
            std::copy(rope_q, rope_q + static_cast<int64_t>(HH) * D, rope_k + static_cast<int64_t>(s) * HH * D);
    }
    return m_spatial;
}
