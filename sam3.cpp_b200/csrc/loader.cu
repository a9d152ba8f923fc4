// loader.cu -- sam3.cpp weight files on the B200 backend: the header,
// hyper-parameter and tensor-record format sam3_load_model / sam3_load_tensors
// read (sam3.cpp:3095-3198, 3204-3330; hyper-parameters sam3_load_hparams
// :1481-1525 and sam2_load_hparams :1568-1630), written by
// convert_sam3_to_ggml.py / convert_sam2_to_ggml.py and examples/quantize.cpp.
//
// Opening a file scans the records into a directory (name, type, shape, data
// offset) without reading tensor data.  Loading streams every tensor through
// two pinned staging buffers: a reader thread fills one while the other is
// handed to the runner that owns the tensor's name (whose set_tensor copies it
// to the device), so disk reads overlap the host-to-device copies.  Tensors
// of components this backend does not run are counted and listed as skipped.
#include "../../include/sam3_b200.h"
#include "backend_impl.h"

#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace b200 {
namespace {

constexpr uint32_t kSam3Magic = 0x73616D33;  // "sam3"
constexpr uint32_t kSam2Magic = 0x73616D32;  // "sam2"
constexpr int32_t kSam3Version = 3, kSam2Version = 1;
constexpr int kSam2HparamWords = 57;  // sam2_load_hparams, backbone_type 1 (Hiera)

struct TensorRec {
    std::string name;
    int32_t type = 0, n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int64_t offset = 0, bytes = 0;
};

// bytes of n elements in rows of ne0 (ggml_row_size per row for block types)
int64_t data_bytes(int32_t type, int64_t ne0, int64_t n) {
    switch (type) {
    case SAM3B200_TYPE_F32: return 4 * n;
    case SAM3B200_TYPE_F16: return 2 * n;
    case SAM3B200_TYPE_Q4_0: return ne0 % 32 ? -1 : n / 32 * 18;
    case SAM3B200_TYPE_Q4_1: return ne0 % 32 ? -1 : n / 32 * 20;
    case SAM3B200_TYPE_Q8_0: return ne0 % 32 ? -1 : n / 32 * 34;
    default: return -1;
    }
}

}  // namespace

struct WeightFile {
    FILE *fp = nullptr;
    uint32_t magic = 0;
    int32_t version = 0, ftype = 0, n_tensors = 0;
    int64_t size = 0;
    std::vector<int32_t> hp;
    std::vector<TensorRec> tensors;
    std::vector<std::string> skipped;
    ~WeightFile() {
        if (fp) fclose(fp);
    }
};

namespace {

bool rd32(FILE *fp, void *v) { return fread(v, 4, 1, fp) == 1; }

bool parse(WeightFile *f, const char *path) {
    f->fp = fopen(path, "rb");
    if (!f->fp) {
        set_error("file_open: cannot open %s", path);
        return false;
    }
    if (fseeko(f->fp, 0, SEEK_END) != 0 || (f->size = ftello(f->fp)) < 16 || fseeko(f->fp, 0, SEEK_SET) != 0) {
        set_error("file_open: %s is not a weight file (too short)", path);
        return false;
    }
    if (!rd32(f->fp, &f->magic) || !rd32(f->fp, &f->version) || !rd32(f->fp, &f->ftype) ||
        !rd32(f->fp, &f->n_tensors)) {
        set_error("file_open: truncated header");
        return false;
    }
    if (f->magic == kSam3Magic) {
        if (f->version != kSam3Version) {
            set_error("file_open: unsupported SAM3 version %d (expected %d)", f->version, kSam3Version);
            return false;
        }
        // 8 words, n_global_attn indices (at most 4), 27 words (sam3_load_hparams)
        f->hp.resize(8);
        for (int i = 0; i < 8; ++i)
            if (!rd32(f->fp, &f->hp[i])) return set_error("file_open: truncated hyperparameters"), false;
        const int ng = f->hp[7] < 0 ? 0 : f->hp[7] < 4 ? f->hp[7] : 4;
        f->hp.resize(8 + ng + 27);
        for (int i = 8; i < 8 + ng + 27; ++i)
            if (!rd32(f->fp, &f->hp[i])) return set_error("file_open: truncated hyperparameters"), false;
    } else if (f->magic == kSam2Magic) {
        if (f->version != kSam2Version) {
            set_error("file_open: unsupported SAM2 version %d (expected %d)", f->version, kSam2Version);
            return false;
        }
        f->hp.resize(kSam2HparamWords);
        for (int i = 0; i < kSam2HparamWords; ++i)
            if (!rd32(f->fp, &f->hp[i])) return set_error("file_open: truncated hyperparameters"), false;
        if (f->hp[1] != 1) {
            set_error("file_open: backbone type %d (only Hiera, 1, is supported; EdgeTAM is 2)", f->hp[1]);
            return false;
        }
    } else {
        set_error("file_open: unknown magic 0x%08x (sam3 0x%08x, sam2 0x%08x)", f->magic, kSam3Magic, kSam2Magic);
        return false;
    }
    if (f->ftype != 0 && f->ftype != 1 && f->ftype != 2 && f->ftype != 3 && f->ftype != 8) {
        set_error("file_open: unsupported ftype %d", f->ftype);
        return false;
    }
    if (f->n_tensors < 0 || f->n_tensors > (1 << 20)) {
        set_error("file_open: implausible tensor count %d", f->n_tensors);
        return false;
    }
    f->tensors.reserve(static_cast<size_t>(f->n_tensors));
    for (int t = 0; t < f->n_tensors; ++t) {
        TensorRec r;
        int32_t name_len = 0;
        if (!rd32(f->fp, &r.n_dims) || !rd32(f->fp, &name_len) || !rd32(f->fp, &r.type)) {
            set_error("file_open: truncated record %d", t);
            return false;
        }
        if (r.n_dims < 1 || r.n_dims > 4 || name_len < 1 || name_len > 4096) {
            set_error("file_open: bad record %d (%d dims, name length %d)", t, r.n_dims, name_len);
            return false;
        }
        int64_t n = 1;
        for (int i = 0; i < r.n_dims; ++i) {
            int32_t d = 0;
            if (!rd32(f->fp, &d) || d <= 0) {
                set_error("file_open: bad shape in record %d", t);
                return false;
            }
            r.ne[i] = d;
            n *= d;
        }
        r.name.resize(static_cast<size_t>(name_len));
        if (fread(&r.name[0], 1, static_cast<size_t>(name_len), f->fp) != static_cast<size_t>(name_len)) {
            set_error("file_open: truncated name in record %d", t);
            return false;
        }
        const int64_t pos = ftello(f->fp);
        r.offset = pos + (32 - pos % 32) % 32;  // data starts 32-byte aligned
        r.bytes = data_bytes(r.type, r.ne[0], n);
        if (r.bytes < 0) {
            set_error("file_open: %s: type %d with ne0 %lld is not supported", r.name.c_str(), r.type,
                      (long long)r.ne[0]);
            return false;
        }
        if (r.offset + r.bytes > f->size) {
            set_error("file_open: %s: data runs past the end of the file", r.name.c_str());
            return false;
        }
        if (fseeko(f->fp, r.offset + r.bytes, SEEK_SET) != 0) {
            set_error("file_open: seek failed after %s", r.name.c_str());
            return false;
        }
        f->tensors.push_back(std::move(r));
    }
    return true;
}

bool starts(const std::string &s, const char *p) { return s.compare(0, strlen(p), p) == 0; }

// the runner that owns a tensor name (nullptr: not run by this backend)
int route(const sam3b200_model_parts *m, const std::string &n, int type, const void *data, const int64_t *ne,
          bool *taken) {
    *taken = true;
    if (m->vit && (starts(n, "vit.") || starts(n, "neck.trk.") || starts(n, "neck.det.")))
        return sam3b200_vit_set_tensor(m->vit, n.c_str(), type, data, ne);
    if (m->hiera && (starts(n, "hiera.") || starts(n, "fpn.")))
        return sam3b200_hiera_set_tensor(m->hiera, n.c_str(), type, data, ne);
    if (m->text && starts(n, "text.")) return sam3b200_text_set_tensor(m->text, n.c_str(), type, data, ne);
    if (m->sam_dec && (starts(n, "sam_pe.") || starts(n, "sam_dec.") || n == "no_mem_embed"))
        return sam3b200_sam_dec_set_tensor(m->sam_dec, n.c_str(), type, data, ne);
    if (m->mem_attn && starts(n, "mem_attn.")) return sam3b200_mem_attn_set_tensor(m->mem_attn, n.c_str(), type, data, ne);
    if (m->mem_enc && (starts(n, "mem_enc.") || n == "no_obj_embed_spatial"))
        return sam3b200_mem_enc_set_tensor(m->mem_enc, n.c_str(), type, data, ne);
    if (m->fenc && starts(n, "fenc.")) return sam3b200_fenc_set_tensor(m->fenc, n.c_str(), type, data, ne);
    if (m->ddec && (starts(n, "ddec.") || starts(n, "scoring.")))
        return sam3b200_ddec_set_tensor(m->ddec, n.c_str(), type, data, ne);
    if (m->seg && starts(n, "seg.")) return sam3b200_seg_set_tensor(m->seg, n.c_str(), type, data, ne);
    if (m->geom && (starts(n, "geom.layers.") || starts(n, "geom.encode_norm.")))
        return sam3b200_geom_set_tensor(m->geom, n.c_str(), type, data, ne);
    *taken = false;
    return SAM3B200_STATUS_SUCCESS;
}

}  // namespace
}  // namespace b200

using namespace b200;

sam3b200_file *sam3b200_file_open(const char *path) {
    if (!path) return nullptr;
    auto *f = new WeightFile();
    if (!parse(f, path)) {
        delete f;
        return nullptr;
    }
    return reinterpret_cast<sam3b200_file *>(f);
}

void sam3b200_file_close(sam3b200_file *hf) { delete reinterpret_cast<WeightFile *>(hf); }

int sam3b200_file_info(const sam3b200_file *hf, uint32_t *magic, int32_t *version, int32_t *ftype,
                       int32_t *n_tensors) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f) return SAM3B200_STATUS_FAILED;
    if (magic) *magic = f->magic;
    if (version) *version = f->version;
    if (ftype) *ftype = f->ftype;
    if (n_tensors) *n_tensors = f->n_tensors;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_file_hparams(const sam3b200_file *hf, int32_t *words, int cap) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f) return -1;
    const int n = static_cast<int>(f->hp.size());
    for (int i = 0; words && i < n && i < cap; ++i) words[i] = f->hp[i];
    return n;
}

int sam3b200_file_tensor(const sam3b200_file *hf, int i, char *name, int name_cap, int32_t *type, int64_t *ne,
                         int64_t *offset, int64_t *bytes) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f || i < 0 || i >= static_cast<int>(f->tensors.size())) return SAM3B200_STATUS_FAILED;
    const TensorRec &r = f->tensors[static_cast<size_t>(i)];
    if (name && name_cap > 0) snprintf(name, static_cast<size_t>(name_cap), "%s", r.name.c_str());
    if (type) *type = r.type;
    if (ne)
        for (int d = 0; d < 4; ++d) ne[d] = r.ne[d];
    if (offset) *offset = r.offset;
    if (bytes) *bytes = r.bytes;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_file_vit_hparams(const sam3b200_file *hf, sam3b200_vit_hparams *out) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f || !out || f->magic != kSam3Magic) {
        set_error("file_vit_hparams: not a SAM3 file");
        return SAM3B200_STATUS_FAILED;
    }
    const std::vector<int32_t> &h = f->hp;
    const int ng = h[7] < 0 ? 0 : h[7] < 4 ? h[7] : 4;
    sam3b200_vit_hparams v{};
    v.img = h[0];
    v.patch = h[1];
    v.embed = h[2];
    v.depth = h[3];
    v.heads = h[4];
    v.mlp = static_cast<int>(static_cast<float>(h[2]) * (static_cast<float>(h[5]) / 1000.0f));
    v.window = h[6];
    v.n_global = ng;
    for (int i = 0; i < 4; ++i) v.global_idx[i] = i < ng ? h[8 + i] : -1;
    v.neck_dim = h[8 + ng + 6];
    v.pos_grid = 0;
    v.wtype = -1;
    for (const TensorRec &r : f->tensors) {
        if (r.name == "vit.pos_embed") v.pos_grid = static_cast<int>(r.ne[1]);
        if (r.name == "vit.blocks.0.attn.qkv.weight") v.wtype = r.type;
    }
    if (v.pos_grid <= 0 || v.wtype < 0) {
        set_error("file_vit_hparams: vit.pos_embed or vit.blocks.0.attn.qkv.weight missing");
        return SAM3B200_STATUS_FAILED;
    }
    *out = v;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_file_text_hparams(const sam3b200_file *hf, sam3b200_text_hparams *out) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f || !out || f->magic != kSam3Magic) {
        set_error("file_text_hparams: not a SAM3 file");
        return SAM3B200_STATUS_FAILED;
    }
    const int ng = f->hp[7] < 0 ? 0 : f->hp[7] < 4 ? f->hp[7] : 4;
    const int32_t *t = f->hp.data() + 8 + ng;  // text_width .. text_out_dim
    *out = sam3b200_text_hparams{t[0], t[1], t[2], t[3], t[4], t[5]};
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_file_hiera_hparams(const sam3b200_file *hf, sam3b200_hiera_hparams *out) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f || !out || f->magic != kSam2Magic) {
        set_error("file_hiera_hparams: not a SAM2 file");
        return SAM3B200_STATUS_FAILED;
    }
    const int32_t *h = f->hp.data();  // sam2_load_hparams word order
    sam3b200_hiera_hparams v{};
    v.img = h[0];
    v.embed = h[2];
    v.heads = h[3];
    for (int i = 0; i < 4; ++i) v.stages[i] = h[5 + i];
    v.n_global = h[9];
    for (int i = 0; i < 8; ++i) v.global_idx[i] = h[10 + i];
    v.q_pool = h[18];
    for (int i = 0; i < 4; ++i) v.window_spec[i] = h[19 + i];
    v.bkg_h = h[23];
    v.bkg_w = h[24];
    v.scalp = h[25];
    v.neck_dim = h[26];
    v.fpn_top_down_n = h[27];
    for (int i = 0; i < 4; ++i) v.fpn_top_down_levels[i] = h[28 + i];
    *out = v;
    return SAM3B200_STATUS_SUCCESS;
}

int sam3b200_file_load(sam3b200_file *hf, sam3b200_backend *hb, const sam3b200_model_parts *parts,
                       int64_t *n_loaded, int64_t *n_skipped) {
    auto *f = reinterpret_cast<WeightFile *>(hf);
    auto *be = reinterpret_cast<Backend *>(hb);
    if (!f || !be || !parts) {
        set_error("file_load: null argument");
        return SAM3B200_STATUS_FAILED;
    }
    cudaSetDevice(be->device);
    f->skipped.clear();
    int64_t max_bytes = 16;
    for (const TensorRec &r : f->tensors) max_bytes = r.bytes > max_bytes ? r.bytes : max_bytes;
    void *slot[2] = {nullptr, nullptr};
    for (auto &s : slot)
        if (!cuda_ok(cudaHostAlloc(&s, static_cast<size_t>(max_bytes), cudaHostAllocDefault), "pinned staging")) {
            for (auto &t : slot)
                if (t) cudaFreeHost(t);
            return SAM3B200_STATUS_ALLOC_FAILED;
        }
    // reader thread: tensor i goes to slot i % 2 once the consumer released it
    std::mutex mu;
    std::condition_variable cv;
    int64_t ready = -1, consumed = -1;  // last tensor read / last tensor handed off
    bool read_failed = false, stop = false;
    const int64_t nt = static_cast<int64_t>(f->tensors.size());
    std::thread reader([&] {
        for (int64_t i = 0; i < nt; ++i) {
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return stop || consumed >= i - 2; });  // slot i % 2 is free again
                if (stop) return;
            }
            const TensorRec &r = f->tensors[static_cast<size_t>(i)];
            const bool ok = fseeko(f->fp, r.offset, SEEK_SET) == 0 &&
                            fread(slot[i % 2], 1, static_cast<size_t>(r.bytes), f->fp) == static_cast<size_t>(r.bytes);
            std::lock_guard<std::mutex> lk(mu);
            if (!ok) {
                read_failed = true;
                cv.notify_all();
                return;
            }
            ready = i;
            cv.notify_all();
        }
    });
    int status = SAM3B200_STATUS_SUCCESS;
    int64_t loaded = 0;
    for (int64_t i = 0; i < nt && status == SAM3B200_STATUS_SUCCESS; ++i) {
        {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return ready >= i || read_failed; });
            if (ready < i) {
                set_error("file_load: read of %s failed", f->tensors[static_cast<size_t>(i)].name.c_str());
                status = SAM3B200_STATUS_FAILED;
                break;
            }
        }
        const TensorRec &r = f->tensors[static_cast<size_t>(i)];
        bool taken = false;
        status = route(parts, r.name, r.type, slot[i % 2], r.ne, &taken);
        if (taken && status == SAM3B200_STATUS_SUCCESS) ++loaded;
        if (!taken) f->skipped.push_back(r.name);
        {
            std::lock_guard<std::mutex> lk(mu);
            consumed = i;
        }
        cv.notify_all();
    }
    {
        std::lock_guard<std::mutex> lk(mu);
        stop = true;
    }
    cv.notify_all();
    reader.join();
    for (auto &s : slot) cudaFreeHost(s);
    if (n_loaded) *n_loaded = loaded;
    if (n_skipped) *n_skipped = static_cast<int64_t>(f->skipped.size());
    return status;
}

int sam3b200_file_skipped(const sam3b200_file *hf, char *buf, int cap) {
    const auto *f = reinterpret_cast<const WeightFile *>(hf);
    if (!f) return -1;
    std::string all;
    for (const auto &s : f->skipped) all += s + "\n";
    if (buf && cap > 0) snprintf(buf, static_cast<size_t>(cap), "%s", all.c_str());
    return static_cast<int>(f->skipped.size());
}
