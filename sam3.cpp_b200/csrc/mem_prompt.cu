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
    std::vector<float> sine(D), proj(MD);
    int64_t tok = m_spatial;
    for (int p = 0; p < P; ++p) {
        const int rel = std::max(1, std::abs(cur_frame - ptr_frames[p]));
        sine_pe_1d(sine.data(), static_cast<float>(rel) / 15.0f, D);
        for (int j = 0; j < MD; ++j) {
            float sum = tpos_proj_b ? tpos_proj_b[j] : 0.0f;
            for (int i = 0; i < D; ++i)
                sum += (tpos_proj_w ? tpos_proj_w[i + static_cast<int64_t>(j) * D] : 0.0f) * sine[i];
            proj[j] = sum;
        }
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
