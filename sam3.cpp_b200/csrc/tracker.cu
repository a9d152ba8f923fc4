// tracker.cu -- the video tracker's frame loop for visual-only models
// (sam3_create_visual_tracker / sam3_tracker_add_instance /
// sam3_propagate_frame, sam3.cpp:12017-12262) on the B200, chaining the
// runners of this library on the device:
//
//   encode (Hiera + FPN)  ->  per tracked instance:
//     memory prompt from the instance's device-resident bank (selected slots'
//     features copied, slot positional codes + temporal codes by a kernel,
//     object-pointer tokens copied, their positional rows from the host)
//     -> memory attention (sam3b200_mem_attn_run_device)
//     -> SAM decoder on the conditioned features (sam3b200_sam_dec_run_tracking)
//     -> kept mask (best of masks 1..3 by IoU for SAM2's multimask_output_in_sam)
//     -> memory encoder on that mask and the frame's features -> new bank slot
//     -> object pointer (3-layer MLP kernel on the kept mask's token) -> pointer bank
//
// Frame 0 (sam3_tracker_add_instance): a PVS decode of the prompts (mask 0),
// the binary mask at the original size turned into +-6 logits at 4H x 4H,
// encoded as a conditioning memory, and the SAM token's pointer.
//
// The host keeps only indices (which slots, frame numbers) and the tiny
// pointer positional rows; every feature stays in HBM.  The host-side
// post-processing of sam3_propagate_frame (hole filling, sprinkle removal,
// overlap resolution, sam3.cpp:12244-12255) is not part of this loop.
#include "../../include/sam3_b200.h"
#include "backend_impl.h"
#include "model_util.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <deque>
#include <memory>
#include <string>
#include <vector>

namespace b200 {
namespace {

// prompt_pos rows of one memory slot: its spatial code plus (optionally) one temporal-code row
__global__ void slot_pos_kernel(const float *__restrict__ pe, const float *__restrict__ te, int64_t n, int md,
                                float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n * md) return;
    out[i] = te ? __fadd_rn(pe[i], te[i % md]) : pe[i];
}

// sam3_tracker_add_instance's synthetic logits: the binary mask (255 / 0, mw x mh) sampled at
// (x * mw / S, y * mh / S) -> +6 / -6 on an S x S grid
__global__ void synth_logits_kernel(const uint8_t *__restrict__ mask, int mw, int mh, int S, float *__restrict__ out) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(S) * S) return;
    const int x = static_cast<int>(i % S), y = static_cast<int>(i / S);
    const int sx = static_cast<int>(static_cast<int64_t>(x) * mw / S), sy = static_cast<int>(static_cast<int64_t>(y) * mh / S);
    out[i] = mask[static_cast<int64_t>(sy) * mw + sx] > 127 ? 6.0f : -6.0f;
}

// sam3_extract_obj_ptr_cpu (sam3.cpp:9347-9420): three D x D layers (ReLU after the first two) on the
// token; blend: lam * mlp + (1 - lam) * no_obj_ptr with lam = [obj > 0]; else no_obj_ptr when obj <= 0.
// One CTA of 256 threads; a warp per output row, its lanes over the inputs (coalesced weight rows).
__global__ void __launch_bounds__(256) obj_ptr_kernel(const float *__restrict__ token, float obj, int D,
                                                      const float *__restrict__ w0, const float *__restrict__ b0,
                                                      const float *__restrict__ w1, const float *__restrict__ b1,
                                                      const float *__restrict__ w2, const float *__restrict__ b2,
                                                      const float *__restrict__ no_ptr, int blend,
                                                      float *__restrict__ out) {
    extern __shared__ float h[];  // [2][D]
    float *cur = h, *nxt = h + D;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    if (!blend && !(obj > 0.0f)) {
        for (int i = threadIdx.x; i < D; i += blockDim.x) out[i] = no_ptr[i];
        return;
    }
    for (int i = threadIdx.x; i < D; i += blockDim.x) cur[i] = token[i];
    __syncthreads();
    const float *ws[3] = {w0, w1, w2}, *bs[3] = {b0, b1, b2};
    for (int j = 0; j < 3; ++j) {
        for (int o = warp; o < D; o += nwarps) {
            const float *row = ws[j] + static_cast<int64_t>(o) * D;
            float sum = 0.0f;
            for (int i = lane; i < D; i += 32) sum = fmaf(row[i], cur[i], sum);
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            if (lane == 0) {
                const float v = __fadd_rn(bs[j][o], sum);
                nxt[o] = j < 2 ? fmaxf(v, 0.0f) : v;
            }
        }
        __syncthreads();
        float *t = cur;
        cur = nxt;
        nxt = t;
    }
    const float lam = obj > 0.0f ? 1.0f : 0.0f;
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        out[i] = blend ? __fadd_rn(__fmul_rn(lam, cur[i]), __fmul_rn(1.0f - lam, no_ptr[i])) : cur[i];
}

unsigned blocks_for(int64_t n) { return static_cast<unsigned>((n + 255) / 256); }

struct Slot {
    int buf = -1;  // index into the instance's slot buffers
    int frame = 0;
    bool cond = false;
};

struct Ptr {
    int buf = -1;
    int frame = 0;
};

struct Instance {
    int id = 0;
    int first_frame = 0, last_seen = 0;
    float last_score = 0.0f, iou = 0.0f, obj = 0.0f;
    std::deque<Slot> slots;
    std::deque<Ptr> ptrs;
    std::vector<DevBuf> slot_bufs;  // num_maskmem + 1 buffers of [N][MD]
    std::vector<int> slot_free;
    std::vector<DevBuf> ptr_bufs;   // max_obj_ptrs + 1 buffers of [D]
    std::vector<int> ptr_free;
    DevBuf mask;                    // kept mask logits of the last add / propagate, [S][S]
    DevBuf token;                   // that mask's output token, [D]
};

}  // namespace

struct Tracker {
    Backend *be = nullptr;
    sam3b200_tracker_hparams hp{};
    sam3b200_hiera *enc = nullptr;
    sam3b200_sam_dec *dec = nullptr;
    sam3b200_mem_attn *attn = nullptr;
    sam3b200_mem_enc *menc = nullptr;
    int H = 0, N = 0, S = 0, D = 0, MD = 0, split = 0;
    int64_t m_max = 0;
    // weights
    DevBuf ptr_w[3], ptr_b[3], no_ptr, tpos_enc;
    std::vector<float> tpos_w, tpos_b;  // host: the pointer positional rows are formed on the host
    bool have_w[3] = {false, false, false}, have_b[3] = {false, false, false}, have_no_ptr = false;
    bool have_tpos_enc = false;
    // constants
    DevBuf src_pos, pe64, rope_q, rope_k;
    // per frame
    DevBuf prompt, prompt_pos, mask_u8, synth, rgb, chw;
    // pinned: the pointer positional rows reach the device without a sync; rewritten by the next
    // instance only after the decoder's readback has synchronised the stream
    float *ptr_pos_host = nullptr;
    ~Tracker() {
        if (ptr_pos_host) cudaFreeHost(ptr_pos_host);
    }
    std::vector<std::unique_ptr<Instance>> inst;
    int next_id = 1;
    int frame_index = 0;
    bool encoded = false;
};

namespace {

bool tl(Tracker *t, cudaError_t e, const char *what, int n = 1) {
    t->be->count(n);
    return cuda_ok(e, what);
}

bool features(Tracker *t, const float **lvl2, const float **lvl0, const float **lvl1) {
    int64_t ne[4];
    if (sam3b200_hiera_output(t->enc, 2, lvl2, ne) != SAM3B200_STATUS_SUCCESS ||
        sam3b200_hiera_output(t->enc, 0, lvl0, ne) != SAM3B200_STATUS_SUCCESS ||
        sam3b200_hiera_output(t->enc, 1, lvl1, ne) != SAM3B200_STATUS_SUCCESS)
        return false;
    return true;
}

Instance *find(Tracker *t, int id) {
    for (auto &p : t->inst)
        if (p->id == id) return p.get();
    return nullptr;
}

bool ready(Tracker *t) {
    std::string miss;
    for (int j = 0; j < 3; ++j) {
        if (!t->have_w[j]) miss += " obj_ptr_proj.layers." + std::to_string(j) + ".weight";
        if (!t->have_b[j]) miss += " obj_ptr_proj.layers." + std::to_string(j) + ".bias";
    }
    if (!t->have_no_ptr) miss += " no_obj_ptr";
    if (!miss.empty()) {
        set_error("tracker: missing tensors:%s", miss.c_str());
        return false;
    }
    return true;
}

// store the memory encoder's output as a new slot (sam3_encode_memory's bank rule: at most
// num_maskmem slots; drop the oldest non-conditioning slot, else slot 1)
bool push_slot(Tracker *t, Instance *in, const float *feats, int frame, bool cond) {
    if (in->slot_free.empty()) {
        set_error("tracker: no free memory slot");
        return false;
    }
    Slot s;
    s.buf = in->slot_free.back();
    in->slot_free.pop_back();
    s.frame = frame;
    s.cond = cond;
    if (!tl(t, cudaMemcpyAsync(in->slot_bufs[s.buf].p, feats, static_cast<size_t>(t->N) * t->MD * 4,
                               cudaMemcpyDeviceToDevice, t->be->stream),
            "tracker slot copy", 0))
        return false;
    in->slots.push_back(s);
    while (static_cast<int>(in->slots.size()) > t->hp.num_maskmem) {
        auto it = std::find_if(in->slots.begin(), in->slots.end(), [](const Slot &x) { return !x.cond; });
        if (it == in->slots.end()) it = in->slots.begin() + 1;
        in->slot_free.push_back(it->buf);
        in->slots.erase(it);
    }
    return true;
}

// sam3_extract_obj_ptr_cpu + sam3_store_obj_ptr: at most max_obj_ptrs pointers, the oldest dropped
bool push_ptr(Tracker *t, Instance *in, const float *token, float obj, int frame) {
    if (in->ptr_free.empty()) {
        set_error("tracker: no free pointer slot");
        return false;
    }
    Ptr p;
    p.buf = in->ptr_free.back();
    in->ptr_free.pop_back();
    p.frame = frame;
    obj_ptr_kernel<<<1, 256, 2 * t->D * sizeof(float), t->be->stream>>>(
        token, obj, t->D, t->ptr_w[0].as<float>(), t->ptr_b[0].as<float>(), t->ptr_w[1].as<float>(),
        t->ptr_b[1].as<float>(), t->ptr_w[2].as<float>(), t->ptr_b[2].as<float>(), t->no_ptr.as<float>(),
        t->hp.fixed_no_obj_ptr, in->ptr_bufs[p.buf].as<float>());
    if (!tl(t, cudaGetLastError(), "tracker object pointer")) return false;
    in->ptrs.push_back(p);
    while (static_cast<int>(in->ptrs.size()) > t->hp.max_obj_ptrs) {
        in->ptr_free.push_back(in->ptrs.front().buf);
        in->ptrs.pop_front();
    }
    return true;
}

// sam3_propagate_single's inputs (sam3.cpp:11175-11233) assembled on the device; returns M_total, the
// pointer-token count in *n_ptr_tok and the spatial-token count in *m_spatial
int64_t build_prompt(Tracker *t, Instance *in, int cur_frame, int *n_ptr_tok, int64_t *m_spatial) {
    const int ns = static_cast<int>(in->slots.size());
    std::vector<int32_t> sel(static_cast<size_t>(std::max(ns, 2)));
    const int n_sel = sam3b200_select_memory_frames(ns, t->hp.num_maskmem, sel.data(), static_cast<int>(sel.size()));
    if (n_sel < 0) return -1;
    cudaStream_t s = t->be->stream;
    const int64_t slot_elems = static_cast<int64_t>(t->N) * t->MD;
    float *prompt = t->prompt.as<float>(), *pos = t->prompt_pos.as<float>();
    for (int k = 0; k < n_sel; ++k) {
        const Slot &sl = in->slots[static_cast<size_t>(sel[k])];
        const int tp = sl.cond ? 0 : n_sel - k;  // temporal position: 0 for a conditioning slot
        const float *te = nullptr;
        if (tp < t->hp.num_maskmem && t->have_tpos_enc)
            te = t->tpos_enc.as<float>() + static_cast<int64_t>(t->hp.num_maskmem - tp - 1) * t->MD;
        if (!tl(t, cudaMemcpyAsync(prompt + k * slot_elems, in->slot_bufs[sl.buf].p, slot_elems * 4,
                                   cudaMemcpyDeviceToDevice, s),
                "tracker prompt copy", 0))
            return -1;
        slot_pos_kernel<<<blocks_for(slot_elems), 256, 0, s>>>(t->pe64.as<float>(), te, t->N, t->MD,
                                                               pos + k * slot_elems);
        if (!tl(t, cudaGetLastError(), "tracker slot positions")) return -1;
    }
    *m_spatial = n_sel * static_cast<int64_t>(t->N);
    const int P = std::min(static_cast<int>(in->ptrs.size()), t->hp.max_obj_ptrs);
    int64_t tok = *m_spatial;
    for (int p = 0; p < P; ++p) {
        const Ptr &pp = in->ptrs[static_cast<size_t>(p)];
        const int rel = std::max(1, std::abs(cur_frame - pp.frame));
        float *row = t->ptr_pos_host + static_cast<size_t>(p) * t->split * t->MD;
        obj_ptr_pos_row(t->D, t->MD, rel, t->tpos_w.empty() ? nullptr : t->tpos_w.data(),
                        t->tpos_b.empty() ? nullptr : t->tpos_b.data(), row);
        for (int k = 1; k < t->split; ++k) std::copy(row, row + t->MD, row + static_cast<size_t>(k) * t->MD);
        // the pointer's D floats are its split tokens of MD, in order
        if (!tl(t, cudaMemcpyAsync(prompt + (tok + static_cast<int64_t>(p) * t->split) * t->MD,
                                   in->ptr_bufs[pp.buf].p, static_cast<size_t>(t->D) * 4, cudaMemcpyDeviceToDevice, s),
                "tracker pointer tokens", 0))
            return -1;
    }
    if (P > 0 && !tl(t, cudaMemcpyAsync(pos + tok * t->MD, t->ptr_pos_host,
                                        static_cast<size_t>(P) * t->split * t->MD * 4, cudaMemcpyHostToDevice, s),
                     "tracker pointer positions", 0))
        return -1;
    *n_ptr_tok = P * t->split;
    return tok + static_cast<int64_t>(P) * t->split;
}

bool keep_mask(Tracker *t, Instance *in, int m) {
    const float *masks = nullptr, *token = nullptr;
    if (sam3b200_sam_dec_outputs(t->dec, &masks, nullptr, nullptr, nullptr) != SAM3B200_STATUS_SUCCESS ||
        sam3b200_sam_dec_mask_token(t->dec, m, &token) != SAM3B200_STATUS_SUCCESS)
        return false;
    cudaStream_t s = t->be->stream;
    const size_t ss = static_cast<size_t>(t->S) * t->S;
    return tl(t, cudaMemcpyAsync(in->mask.p, masks + static_cast<size_t>(m) * ss, ss * 4, cudaMemcpyDeviceToDevice, s),
              "tracker keep mask", 0) &&
           tl(t, cudaMemcpyAsync(in->token.p, token, static_cast<size_t>(t->D) * 4, cudaMemcpyDeviceToDevice, s),
              "tracker keep token", 0);
}

bool new_instance(Tracker *t, Instance *in) {
    in->slot_bufs.resize(static_cast<size_t>(t->hp.num_maskmem) + 1);
    for (size_t i = 0; i < in->slot_bufs.size(); ++i) {
        if (!in->slot_bufs[i].alloc(static_cast<size_t>(t->N) * t->MD * 4)) return false;
        in->slot_free.push_back(static_cast<int>(in->slot_bufs.size() - 1 - i));
    }
    in->ptr_bufs.resize(static_cast<size_t>(t->hp.max_obj_ptrs) + 1);
    for (size_t i = 0; i < in->ptr_bufs.size(); ++i) {
        if (!in->ptr_bufs[i].alloc(static_cast<size_t>(t->D) * 4)) return false;
        in->ptr_free.push_back(static_cast<int>(in->ptr_bufs.size() - 1 - i));
    }
    return in->mask.alloc(static_cast<size_t>(t->S) * t->S * 4) && in->token.alloc(static_cast<size_t>(t->D) * 4);
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" {

sam3b200_tracker *sam3b200_tracker_create(sam3b200_backend *h, const sam3b200_tracker_hparams *hp,
                                          sam3b200_hiera *enc, sam3b200_sam_dec *dec, sam3b200_mem_attn *attn,
                                          sam3b200_mem_enc *menc) {
    auto *be = reinterpret_cast<Backend *>(h);
    if (!be || !hp || !enc || !dec || !attn || !menc) {
        set_error("tracker_create: null argument");
        return nullptr;
    }
    if (hp->feat <= 0 || hp->feat > 256 || hp->d_model <= 0 || hp->mem_dim <= 0 || hp->d_model % hp->mem_dim ||
        hp->d_model % 4 || hp->num_maskmem < 1 || hp->num_maskmem > 64 || hp->max_obj_ptrs < 0 ||
        hp->max_obj_ptrs > 256 || hp->max_instances < 1 || hp->max_keep_alive < 0) {
        set_error("tracker_create: bad hyper-parameters");
        return nullptr;
    }
    cudaSetDevice(be->device);
    auto *t = new Tracker();
    t->be = be;
    t->hp = *hp;
    t->enc = enc;
    t->dec = dec;
    t->attn = attn;
    t->menc = menc;
    t->H = hp->feat;
    t->N = hp->feat * hp->feat;
    t->S = 4 * hp->feat;
    t->D = hp->d_model;
    t->MD = hp->mem_dim;
    t->split = hp->d_model / hp->mem_dim;
    t->m_max = static_cast<int64_t>(hp->num_maskmem) * t->N + static_cast<int64_t>(hp->max_obj_ptrs) * t->split;
    // constant inputs: the 2-D sine codes (d_model for the current frame, mem_dim for the memory slots)
    // and the RoPE tables (sam3_ensure_tracker_pe_caches, sam3.cpp:11140-11152)
    std::vector<float> sp(static_cast<size_t>(t->N) * t->D), pe(static_cast<size_t>(t->N) * t->MD),
        rq(static_cast<size_t>(t->N) * t->D);
    bool ok = sam3b200_sinusoidal_pe_2d(t->H, t->H, t->D, sp.data()) == SAM3B200_STATUS_SUCCESS &&
              sam3b200_sinusoidal_pe_2d(t->H, t->H, t->MD, pe.data()) == SAM3B200_STATUS_SUCCESS &&
              sam3b200_axial_cis(t->D, t->H, t->H, 10000.0f, 1.0f, rq.data()) == SAM3B200_STATUS_SUCCESS;
    std::vector<float> rk;
    if (ok) {
        rk.resize(rq.size() * static_cast<size_t>(hp->num_maskmem));
        for (int k = 0; k < hp->num_maskmem; ++k) std::copy(rq.begin(), rq.end(), rk.begin() + k * rq.size());
    }
    ok = ok && upload(t->src_pos, sp.data(), sp.size() * 4, be->stream) &&
         upload(t->pe64, pe.data(), pe.size() * 4, be->stream) && upload(t->rope_q, rq.data(), rq.size() * 4, be->stream) &&
         upload(t->rope_k, rk.data(), rk.size() * 4, be->stream) &&
         t->prompt.alloc(static_cast<size_t>(t->m_max) * t->MD * 4) &&
         t->prompt_pos.alloc(static_cast<size_t>(t->m_max) * t->MD * 4) &&
         cuda_ok(cudaMallocHost(&t->ptr_pos_host, static_cast<size_t>(hp->max_obj_ptrs + 1) * t->D * 4),
                 "cudaMallocHost(pointer positions)");
    if (!ok) {
        delete t;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_tracker *>(t);
}

void sam3b200_tracker_free(sam3b200_tracker *h) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t) return;
    cudaSetDevice(t->be->device);
    cudaStreamSynchronize(t->be->stream);
    delete t;
}

int sam3b200_tracker_set_tensor(sam3b200_tracker *h, const char *name, int type, const void *data,
                                const int64_t ne[4]) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t || !name || !data || !ne) {
        set_error("tracker_set_tensor: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    const int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
    std::vector<float> v;
    if (!to_f32(type, data, n, v)) return SAM3B200_STATUS_FAILED;
    const std::string nm(name);
    cudaSetDevice(t->be->device);
    cudaStream_t s = t->be->stream;
    auto shape = [&](int64_t a, int64_t b) {
        if (ne[0] == a && ne[1] * ne[2] * ne[3] == b) return true;
        set_error("tracker_set_tensor: %s has ne [%lld, %lld, %lld, %lld], expected [%lld, %lld]", name,
                  (long long)ne[0], (long long)ne[1], (long long)ne[2], (long long)ne[3], (long long)a, (long long)b);
        return false;
    };
    for (int j = 0; j < 3; ++j) {
        const std::string p = "obj_ptr_proj.layers." + std::to_string(j) + ".";
        if (nm == p + "weight") {
            if (!shape(t->D, t->D) || !upload(t->ptr_w[j], v.data(), v.size() * 4, s)) return SAM3B200_STATUS_FAILED;
            t->have_w[j] = true;
            return SAM3B200_STATUS_SUCCESS;
        }
        if (nm == p + "bias") {
            if (!shape(t->D, 1) || !upload(t->ptr_b[j], v.data(), v.size() * 4, s)) return SAM3B200_STATUS_FAILED;
            t->have_b[j] = true;
            return SAM3B200_STATUS_SUCCESS;
        }
    }
    if (nm == "no_obj_ptr") {
        if (!shape(t->D, 1) || !upload(t->no_ptr, v.data(), v.size() * 4, s)) return SAM3B200_STATUS_FAILED;
        t->have_no_ptr = true;
    } else if (nm == "obj_ptr_tpos_proj.weight") {
        if (!shape(t->D, t->MD)) return SAM3B200_STATUS_FAILED;
        t->tpos_w = v;
    } else if (nm == "obj_ptr_tpos_proj.bias") {
        if (!shape(t->MD, 1)) return SAM3B200_STATUS_FAILED;
        t->tpos_b = v;
    } else if (nm == "mem_enc.tpos_enc") {
        if (!shape(t->MD, t->hp.num_maskmem) || !upload(t->tpos_enc, v.data(), v.size() * 4, s))
            return SAM3B200_STATUS_FAILED;
        t->have_tpos_enc = true;
    } else {
        set_error("tracker_set_tensor: unknown tensor %s", name);
        return SAM3B200_STATUS_FAILED;
    }
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_tracker_encode(sam3b200_tracker *h, const float *img_chw_dev) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t || !img_chw_dev) {
        set_error("tracker_encode: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(t->be->device);
    const int st = sam3b200_hiera_encode_device(t->enc, img_chw_dev);
    t->encoded = st == SAM3B200_STATUS_SUCCESS;
    return st;
}

int sam3b200_tracker_encode_image(sam3b200_tracker *h, const uint8_t *rgb, int w, int h_px) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t || !rgb || w <= 0 || h_px <= 0) {
        set_error("tracker_encode_image: bad arguments");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(t->be->device);
    const size_t bytes = static_cast<size_t>(w) * h_px * 3, chw = static_cast<size_t>(3) * t->hp.img * t->hp.img * 4;
    if ((t->rgb.n < bytes && !t->rgb.alloc(bytes)) || (t->chw.n < chw && !t->chw.alloc(chw))) return SAM3B200_STATUS_FAILED;
    auto *hb = reinterpret_cast<sam3b200_backend *>(t->be);
    if (!tl(t, cudaMemcpyAsync(t->rgb.p, rgb, bytes, cudaMemcpyHostToDevice, t->be->stream), "tracker frame upload", 0) ||
        sam3b200_preprocess_sam2(hb, t->rgb.as<uint8_t>(), w, h_px, t->hp.img, t->chw.as<float>()) !=
            SAM3B200_STATUS_SUCCESS)
        return SAM3B200_STATUS_FAILED;
    return sam3b200_tracker_encode(h, t->chw.as<float>());
}

void sam3b200_tracker_reset(sam3b200_tracker *h) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t) return;
    cudaSetDevice(t->be->device);
    cudaStreamSynchronize(t->be->stream);
    t->inst.clear();
    t->next_id = 1;
    t->frame_index = 0;
    t->encoded = false;
}

int sam3b200_tracker_add_instance(sam3b200_tracker *h, const float *coords, const int32_t *labels, int n_prompts,
                                  int orig_w, int orig_h) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t || !coords || !labels || n_prompts < 1 || orig_w <= 0 || orig_h <= 0) {
        set_error("tracker_add_instance: bad arguments");
        return -1;
    }
    if (!t->encoded) {
        set_error("tracker_add_instance: no encoded frame");
        return -1;
    }
    if (static_cast<int>(t->inst.size()) >= t->hp.max_instances) {
        set_error("tracker_add_instance: %d instances already", static_cast<int>(t->inst.size()));
        return -1;
    }
    if (!ready(t)) return -1;
    cudaSetDevice(t->be->device);
    const float *f2, *f0, *f1;
    if (!features(t, &f2, &f0, &f1)) return -1;
    // the PVS decode (mask 0: multimask off, as sam3_tracker_add_instance's callers ask)
    if (sam3b200_sam_dec_run(t->dec, f2, f0, f1, coords, labels, n_prompts, orig_w, orig_h, t->hp.img) !=
        SAM3B200_STATUS_SUCCESS)
        return -1;
    float iou[4], obj = 0.0f;
    if (sam3b200_sam_dec_outputs(t->dec, nullptr, iou, &obj, nullptr) != SAM3B200_STATUS_SUCCESS) return -1;
    auto in = std::unique_ptr<Instance>(new Instance());
    if (!new_instance(t, in.get())) return -1;
    const int fi = std::max(t->frame_index - 1, 0);
    in->id = t->next_id;
    in->first_frame = in->last_seen = fi;
    in->last_score = in->iou = iou[0];
    in->obj = obj;
    cudaStream_t s = t->be->stream;
    const size_t px = static_cast<size_t>(orig_w) * orig_h;
    if (t->mask_u8.n < px && !t->mask_u8.alloc(px)) return -1;
    // binary mask at the original size -> +-6 logits on the 4H grid
    if (!keep_mask(t, in.get(), 0) ||
        !tl(t, launch_mask_resize(in->mask.as<float>(), t->S, orig_w, orig_h, t->mask_u8.as<uint8_t>(), s),
            "tracker mask resize"))
        return -1;
    if (!t->synth.p && !t->synth.alloc(static_cast<size_t>(t->S) * t->S * 4)) return -1;
    synth_logits_kernel<<<blocks_for(static_cast<int64_t>(t->S) * t->S), 256, 0, s>>>(
        t->mask_u8.as<uint8_t>(), orig_w, orig_h, t->S, t->synth.as<float>());
    if (!tl(t, cudaGetLastError(), "tracker synthetic logits")) return -1;
    const float *mem = nullptr;
    if (sam3b200_mem_enc_run_device(t->menc, t->synth.as<float>(), t->S, t->S, f2, obj) != SAM3B200_STATUS_SUCCESS ||
        sam3b200_mem_enc_output(t->menc, &mem) != SAM3B200_STATUS_SUCCESS)
        return -1;
    if (!push_slot(t, in.get(), mem, fi, true) || !push_ptr(t, in.get(), in->token.as<float>(), obj, fi)) return -1;
    if (!cuda_ok(cudaStreamSynchronize(s), "tracker add sync")) return -1;
    t->inst.push_back(std::move(in));
    return t->next_id++;
}

int sam3b200_tracker_propagate(sam3b200_tracker *h) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t) {
        set_error("tracker_propagate: null tracker");
        return SAM3B200_STATUS_FAILED;
    }
    if (!t->encoded) {
        set_error("tracker_propagate: no encoded frame");
        return SAM3B200_STATUS_FAILED;
    }
    if (!ready(t)) return SAM3B200_STATUS_FAILED;
    cudaSetDevice(t->be->device);
    const float *f2, *f0, *f1;
    if (!features(t, &f2, &f0, &f1)) return SAM3B200_STATUS_FAILED;
    const int fi = t->frame_index;
    for (auto &up : t->inst) {
        Instance *in = up.get();
        if (in->slots.empty()) continue;
        int n_ptr_tok = 0;
        int64_t m_spatial = 0;
        const int64_t m_total = build_prompt(t, in, fi, &n_ptr_tok, &m_spatial);
        if (m_total < 0) return SAM3B200_STATUS_FAILED;
        const float *cond = nullptr;
        if (sam3b200_mem_attn_run_device(t->attn, f2, t->src_pos.as<float>(), t->prompt.as<float>(),
                                         t->prompt_pos.as<float>(), t->rope_q.as<float>(),
                                         m_spatial > 0 ? t->rope_k.as<float>() : nullptr, t->N,
                                         static_cast<int>(m_total), n_ptr_tok) != SAM3B200_STATUS_SUCCESS ||
            sam3b200_mem_attn_output(t->attn, &cond) != SAM3B200_STATUS_SUCCESS)
            return SAM3B200_STATUS_FAILED;
        if (sam3b200_sam_dec_run_tracking(t->dec, cond, f0, f1) != SAM3B200_STATUS_SUCCESS)
            return SAM3B200_STATUS_FAILED;
        float iou[4], obj = 0.0f;
        if (sam3b200_sam_dec_outputs(t->dec, nullptr, iou, &obj, nullptr) != SAM3B200_STATUS_SUCCESS)
            return SAM3B200_STATUS_FAILED;
        int best = 0;
        if (t->hp.multimask_in_sam) {  // the best of masks 1..3 by predicted IoU (the first on a tie)
            best = 1;
            for (int m = 2; m < 4; ++m)
                if (iou[m] > iou[best]) best = m;
        }
        // the pointer comes from the kept mask's token (use_multimask_token_for_obj_ptr), else mask 0's
        const int tok = t->hp.multimask_in_sam && t->hp.multimask_token_for_obj_ptr ? best : 0;
        if (!keep_mask(t, in, best)) return SAM3B200_STATUS_FAILED;
        if (tok != best) {
            const float *token = nullptr;
            if (sam3b200_sam_dec_mask_token(t->dec, tok, &token) != SAM3B200_STATUS_SUCCESS ||
                !tl(t, cudaMemcpyAsync(in->token.p, token, static_cast<size_t>(t->D) * 4, cudaMemcpyDeviceToDevice,
                                       t->be->stream),
                    "tracker keep token", 0))
                return SAM3B200_STATUS_FAILED;
        }
        in->iou = in->last_score = iou[best];
        in->obj = obj;
        in->last_seen = fi;
        const float *mem = nullptr;
        if (sam3b200_mem_enc_run_device(t->menc, in->mask.as<float>(), t->S, t->S, f2, obj) !=
                SAM3B200_STATUS_SUCCESS ||
            sam3b200_mem_enc_output(t->menc, &mem) != SAM3B200_STATUS_SUCCESS)
            return SAM3B200_STATUS_FAILED;
        if (!push_slot(t, in, mem, fi, false) || !push_ptr(t, in, in->token.as<float>(), obj, fi))
            return SAM3B200_STATUS_FAILED;
    }
    // sam3_update_tracker: an instance unseen for more than max_keep_alive frames is dropped
    t->inst.erase(std::remove_if(t->inst.begin(), t->inst.end(),
                                 [&](const std::unique_ptr<Instance> &p) {
                                     return fi - p->last_seen > t->hp.max_keep_alive;
                                 }),
                  t->inst.end());
    t->frame_index++;
    return cuda_ok(cudaStreamSynchronize(t->be->stream), "tracker propagate sync") ? SAM3B200_STATUS_SUCCESS
                                                                                   : SAM3B200_STATUS_FAILED;
}

int sam3b200_tracker_frame_index(const sam3b200_tracker *h) {
    auto *t = reinterpret_cast<const Tracker *>(h);
    return t ? t->frame_index : -1;
}

int sam3b200_tracker_instances(const sam3b200_tracker *h, int32_t *ids, int cap) {
    auto *t = reinterpret_cast<const Tracker *>(h);
    if (!t || (cap > 0 && !ids)) return -1;
    const int n = static_cast<int>(t->inst.size());
    for (int i = 0; i < n && i < cap; ++i) ids[i] = t->inst[static_cast<size_t>(i)]->id;
    return n;
}

int sam3b200_tracker_instance(sam3b200_tracker *h, int id, const float **mask_logits_dev, const float **token_dev,
                              float *iou, float *obj_score, int32_t *last_seen) {
    auto *t = reinterpret_cast<Tracker *>(h);
    Instance *in = t ? find(t, id) : nullptr;
    if (!in) {
        set_error("tracker_instance: no instance %d", id);
        return SAM3B200_STATUS_FAILED;
    }
    if (mask_logits_dev) *mask_logits_dev = in->mask.as<float>();
    if (token_dev) *token_dev = in->token.as<float>();
    if (iou) *iou = in->iou;
    if (obj_score) *obj_score = in->obj;
    if (last_seen) *last_seen = in->last_seen;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_tracker_mask(sam3b200_tracker *h, int id, int out_w, int out_h, uint8_t *dst_dev) {
    auto *t = reinterpret_cast<Tracker *>(h);
    Instance *in = t ? find(t, id) : nullptr;
    if (!in || out_w <= 0 || out_h <= 0 || !dst_dev) {
        set_error("tracker_mask: bad arguments");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(t->be->device);
    return tl(t, launch_mask_resize(in->mask.as<float>(), t->S, out_w, out_h, dst_dev, t->be->stream),
              "tracker mask")
               ? SAM3B200_STATUS_SUCCESS
               : SAM3B200_STATUS_FAILED;
}

int sam3b200_tracker_bank(sam3b200_tracker *h, int id, int32_t *slot_frames, int32_t *slot_cond,
                          const float **slot_feats_dev, int slot_cap, int32_t *ptr_frames, const float **ptrs_dev,
                          int ptr_cap, int32_t *n_ptrs) {
    auto *t = reinterpret_cast<Tracker *>(h);
    Instance *in = t ? find(t, id) : nullptr;
    if (!in || !n_ptrs) {
        set_error("tracker_bank: no instance %d", id);
        return -1;
    }
    const int ns = static_cast<int>(in->slots.size()), np = static_cast<int>(in->ptrs.size());
    for (int i = 0; i < ns && i < slot_cap; ++i) {
        const Slot &s = in->slots[static_cast<size_t>(i)];
        if (slot_frames) slot_frames[i] = s.frame;
        if (slot_cond) slot_cond[i] = s.cond ? 1 : 0;
        if (slot_feats_dev) slot_feats_dev[i] = in->slot_bufs[s.buf].as<float>();
    }
    for (int i = 0; i < np && i < ptr_cap; ++i) {
        const Ptr &p = in->ptrs[static_cast<size_t>(i)];
        if (ptr_frames) ptr_frames[i] = p.frame;
        if (ptrs_dev) ptrs_dev[i] = in->ptr_bufs[p.buf].as<float>();
    }
    *n_ptrs = np;
    return ns;
}

int sam3b200_tracker_prompt(sam3b200_tracker *h, const float **prompt_dev, const float **prompt_pos_dev) {
    auto *t = reinterpret_cast<Tracker *>(h);
    if (!t) return SAM3B200_STATUS_FAILED;
    if (prompt_dev) *prompt_dev = t->prompt.as<float>();
    if (prompt_pos_dev) *prompt_pos_dev = t->prompt_pos.as<float>();
    return SAM3B200_STATUS_SUCCESS;
}

}  // extern "C"
