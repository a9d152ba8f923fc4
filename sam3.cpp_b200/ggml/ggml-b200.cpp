// ggml-b200.cpp -- the B200 ggml backend: ggml's backend, buffer-type, buffer
// and device interfaces (ggml-backend-impl.h) filled over the C ABI of
// libsam3_b200.so (include/sam3_b200.h).  This is what sam3.cpp selects in
// place of ggml_backend_metal_init / ggml_backend_cpu_init
// (sam3.cpp:3279-3287); its weights go into this backend's buffers
// (sam3.cpp:3320) and its graphs through ggml_backend_graph_compute
// (sam3.cpp:1019-1030).
//
// The backend translates, nothing more:
//   - buffers are device allocations of sam3b200_buffer_alloc; tensor
//     set / get / memset are the ABI's synchronous copies;
//   - graph_compute flattens each node and its sources into sam3b200_tensor
//     records (ops mapped by name) and hands them to sam3b200_graph_compute,
//     which checks every node before launching any kernel and returns the
//     ggml_status;
//   - a MUL_MAT whose src0 is a 2-D Q8_0 / Q4_0 / Q4_1 / F16 leaf of a B200
//     buffer (a weight) runs on the tensor-core layout of that weight, made
//     once from the buffer's bytes (sam3b200_weight_upload from device memory)
//     and cached in the buffer until the tensor is written again.
// C++14; no exceptions cross the ggml interface.
#include "ggml-b200.h"

#include "ggml-backend-impl.h"
#include "ggml.h"

#include "../../include/sam3_b200.h"

#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace {

constexpr int kMaxDevices = 16;
constexpr size_t kAlignment = 256;

struct Device {
    int id = -1;
    sam3b200_backend *copier_ = nullptr;  // stream for buffer copies and weight layouts, made on first use
    ggml_backend_buffer_type buft;
    ggml_backend_device dev;
    char name[32] = {0};

    sam3b200_backend *copier();
};

struct BufferCtx {
    Device *d = nullptr;
    void *base = nullptr;
    size_t size = 0;
    std::unordered_map<const ggml_tensor *, sam3b200_weight *> weights;  // tensor-core layouts of weight leafs
};

struct BackendCtx {
    Device *d = nullptr;
    sam3b200_backend *be = nullptr;  // own stream for graph compute
    char name[48] = {0};
};

std::mutex g_mutex;
Device g_devices[kMaxDevices];
ggml_guid g_guid = {{0x73, 0x61, 0x6d, 0x33, 0x62, 0x32, 0x30, 0x30, 0x67, 0x67, 0x6d, 0x6c, 0x2d, 0x62, 0x32, 0x30}};

void report(const char *what) { std::fprintf(stderr, "ggml-b200: %s: %s\n", what, sam3b200_last_error()); }

// ---- buffers ------------------------------------------------------------------------------------

BufferCtx *buf_ctx(ggml_backend_buffer_t b) { return static_cast<BufferCtx *>(b->context); }

void drop_weight(BufferCtx *c, const ggml_tensor *t) {
    const ggml_tensor *base = t->view_src ? t->view_src : t;
    for (const ggml_tensor *k : {t, base}) {
        auto it = c->weights.find(k);
        if (it != c->weights.end()) {
            sam3b200_weight_free(c->d->copier(), it->second);
            c->weights.erase(it);
        }
    }
}

void buffer_free(ggml_backend_buffer_t b) {
    BufferCtx *c = buf_ctx(b);
    for (auto &kv : c->weights) sam3b200_weight_free(c->d->copier(), kv.second);
    sam3b200_buffer_free(c->d->copier(), c->base);
    delete c;
}

void *buffer_get_base(ggml_backend_buffer_t b) { return buf_ctx(b)->base; }

ggml_status buffer_init_tensor(ggml_backend_buffer_t, ggml_tensor *) { return GGML_STATUS_SUCCESS; }

void buffer_memset_tensor(ggml_backend_buffer_t b, ggml_tensor *t, uint8_t value, size_t offset, size_t size) {
    BufferCtx *c = buf_ctx(b);
    drop_weight(c, t);
    if (sam3b200_tensor_memset(c->d->copier(), t->data, value, offset, size) != SAM3B200_STATUS_SUCCESS)
        report("memset_tensor");
}

void buffer_set_tensor(ggml_backend_buffer_t b, ggml_tensor *t, const void *data, size_t offset, size_t size) {
    BufferCtx *c = buf_ctx(b);
    drop_weight(c, t);
    if (sam3b200_tensor_set(c->d->copier(), t->data, data, offset, size) != SAM3B200_STATUS_SUCCESS)
        report("set_tensor");
}

void buffer_get_tensor(ggml_backend_buffer_t b, const ggml_tensor *t, void *data, size_t offset, size_t size) {
    BufferCtx *c = buf_ctx(b);
    if (sam3b200_tensor_get(c->d->copier(), t->data, data, offset, size) != SAM3B200_STATUS_SUCCESS)
        report("get_tensor");
}

bool buffer_cpy_tensor(ggml_backend_buffer_t, const ggml_tensor *, ggml_tensor *) { return false; }

void buffer_clear(ggml_backend_buffer_t b, uint8_t value) {
    BufferCtx *c = buf_ctx(b);
    for (auto &kv : c->weights) sam3b200_weight_free(c->d->copier(), kv.second);
    c->weights.clear();
    if (sam3b200_tensor_memset(c->d->copier(), c->base, value, 0, c->size) != SAM3B200_STATUS_SUCCESS)
        report("buffer clear");
}

ggml_backend_buffer_i buffer_iface() {
    ggml_backend_buffer_i i;
    std::memset(&i, 0, sizeof i);
    i.free_buffer = buffer_free;
    i.get_base = buffer_get_base;
    i.init_tensor = buffer_init_tensor;
    i.memset_tensor = buffer_memset_tensor;
    i.set_tensor = buffer_set_tensor;
    i.get_tensor = buffer_get_tensor;
    i.cpy_tensor = buffer_cpy_tensor;
    i.clear = buffer_clear;
    i.reset = nullptr;
    return i;
}

// ---- buffer type --------------------------------------------------------------------------------

Device *buft_device(ggml_backend_buffer_type_t buft) { return static_cast<Device *>(buft->context); }

const char *buft_get_name(ggml_backend_buffer_type_t buft) { return buft_device(buft)->name; }

ggml_backend_buffer_t buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size) {
    Device *d = buft_device(buft);
    const size_t bytes = size < kAlignment ? kAlignment : size;
    void *base = sam3b200_buffer_alloc(d->copier(), bytes);
    if (!base) {
        report("alloc_buffer");
        return nullptr;
    }
    auto *c = new BufferCtx();
    c->d = d;
    c->base = base;
    c->size = bytes;
    return ggml_backend_buffer_init(buft, buffer_iface(), c, size);
}

size_t buft_get_alignment(ggml_backend_buffer_type_t) { return kAlignment; }
size_t buft_get_max_size(ggml_backend_buffer_type_t) { return SIZE_MAX; }
size_t buft_get_alloc_size(ggml_backend_buffer_type_t, const ggml_tensor *t) { return ggml_nbytes(t); }
bool buft_is_host(ggml_backend_buffer_type_t) { return false; }

bool is_b200_buffer(const ggml_backend_buffer *b) {
    return b && b->buft && b->buft->iface.alloc_buffer == buft_alloc_buffer;
}

// ---- graph translation --------------------------------------------------------------------------

int map_unary(ggml_unary_op u) {
    switch (u) {
        case GGML_UNARY_OP_RELU: return SAM3B200_UNARY_RELU;
        case GGML_UNARY_OP_SIGMOID: return SAM3B200_UNARY_SIGMOID;
        case GGML_UNARY_OP_GELU_ERF: return SAM3B200_UNARY_GELU_ERF;
        case GGML_UNARY_OP_GELU: return SAM3B200_UNARY_GELU;
        default: return -1;
    }
}

// ggml op -> sam3b200 op by name; -1 for an op this backend does not execute
int map_op(ggml_op op) {
    switch (op) {
        case GGML_OP_NONE: return SAM3B200_OP_NONE;
        case GGML_OP_VIEW: case GGML_OP_RESHAPE: case GGML_OP_PERMUTE: case GGML_OP_TRANSPOSE: return SAM3B200_OP_VIEW;
        case GGML_OP_MUL_MAT: return SAM3B200_OP_MUL_MAT;
        case GGML_OP_ADD: return SAM3B200_OP_ADD;
        case GGML_OP_SUB: return SAM3B200_OP_SUB;
        case GGML_OP_MUL: return SAM3B200_OP_MUL;
        case GGML_OP_SCALE: return SAM3B200_OP_SCALE;
        case GGML_OP_NORM: return SAM3B200_OP_NORM;
        case GGML_OP_GROUP_NORM: return SAM3B200_OP_GROUP_NORM;
        case GGML_OP_SOFT_MAX: return SAM3B200_OP_SOFT_MAX;
        case GGML_OP_UNARY: return SAM3B200_OP_UNARY;
        case GGML_OP_CONT: case GGML_OP_CPY: case GGML_OP_DUP: return SAM3B200_OP_CONT;
        case GGML_OP_REPEAT: return SAM3B200_OP_REPEAT;
        case GGML_OP_CONCAT: return SAM3B200_OP_CONCAT;
        case GGML_OP_WIN_PART: return SAM3B200_OP_WIN_PART;
        case GGML_OP_WIN_UNPART: return SAM3B200_OP_WIN_UNPART;
        case GGML_OP_FLASH_ATTN_EXT: return SAM3B200_OP_FLASH_ATTN_EXT;
        case GGML_OP_GET_ROWS: return SAM3B200_OP_GET_ROWS;
        case GGML_OP_IM2COL: return SAM3B200_OP_IM2COL;
        case GGML_OP_CONV_2D: return SAM3B200_OP_CONV_2D;
        case GGML_OP_CONV_2D_DW: return SAM3B200_OP_CONV_2D_DW;
        case GGML_OP_CONV_TRANSPOSE_2D: return SAM3B200_OP_CONV_TRANSPOSE_2D;
        case GGML_OP_POOL_2D: return SAM3B200_OP_POOL_2D;
        case GGML_OP_PAD: return SAM3B200_OP_PAD;
        case GGML_OP_UPSCALE: return SAM3B200_OP_UPSCALE;
        default: return -1;
    }
}

// A 2-D weight the MUL_MAT reads through its tensor-core layout: a leaf in a B200 buffer.
bool weight_leaf(const ggml_tensor *a) {
    const bool quant = a->type == GGML_TYPE_Q8_0 || a->type == GGML_TYPE_Q4_0 || a->type == GGML_TYPE_Q4_1;
    return (quant || a->type == GGML_TYPE_F16) && a->op == GGML_OP_NONE && !a->view_src && a->data &&
           is_b200_buffer(a->buffer) && a->ne[2] == 1 && a->ne[3] == 1 && ggml_is_contiguous(a) &&
           a->ne[0] % (quant ? 32 : 8) == 0;
}

sam3b200_weight *weight_of(const ggml_tensor *a) {
    BufferCtx *c = buf_ctx(a->buffer);
    auto it = c->weights.find(a);
    if (it != c->weights.end()) return it->second;
    sam3b200_weight *w = sam3b200_weight_upload(c->d->copier(), a->type, a->data, a->ne[0], a->ne[1]);
    if (!w) {
        report("weight layout");
        return nullptr;
    }
    c->weights.emplace(a, w);
    return w;
}

struct Records {
    std::vector<sam3b200_tensor> recs;
    std::unordered_map<const ggml_tensor *, size_t> index;
    std::vector<sam3b200_tensor *> nodes;

    void reserve(size_t n) { recs.reserve(n); }

    size_t add(const ggml_tensor *t) {
        auto it = index.find(t);
        if (it != index.end()) return it->second;
        sam3b200_tensor r;
        std::memset(&r, 0, sizeof r);
        r.type = t->type;
        r.op = map_op(t->op);
        std::memcpy(r.ne, t->ne, sizeof r.ne);
        for (int d = 0; d < 4; ++d) r.nb[d] = t->nb[d];
        std::memcpy(r.op_params, t->op_params, sizeof r.op_params);
        r.flags = t->flags;
        r.data = t->data;
        if (t->op == GGML_OP_UNARY) r.op_params[0] = map_unary(static_cast<ggml_unary_op>(t->op_params[0]));
        if (t->op == GGML_OP_UNARY && r.op_params[0] < 0) r.op = -1;
        // sources beyond the four the record holds (attention sinks and the like) are not executed here
        for (int s = 4; s < GGML_MAX_SRC; ++s)
            if (t->src[s]) r.op = -1;
        index.emplace(t, recs.size());
        recs.push_back(r);
        return recs.size() - 1;
    }

    // one record per node and per source of a node, the sources linked; false if a weight layout failed
    bool build(ggml_cgraph *g, bool make_weights) {
        const int n = ggml_graph_n_nodes(g);
        reserve(static_cast<size_t>(n) * 5);
        std::vector<size_t> order;
        for (int i = 0; i < n; ++i) {
            const ggml_tensor *t = ggml_graph_node(g, i);
            order.push_back(add(t));
            const int nsrc = t->op == GGML_OP_CPY ? 1 : 4;  // ggml_cpy's src1 is its destination, not an input
            for (int s = 0; s < nsrc; ++s)
                if (t->src[s]) add(t->src[s]);
        }
        for (const auto &kv : index) {
            const ggml_tensor *t = kv.first;
            sam3b200_tensor &r = recs[kv.second];
            const int nsrc = t->op == GGML_OP_CPY ? 1 : 4;
            for (int s = 0; s < nsrc; ++s) {
                auto it = t->src[s] ? index.find(t->src[s]) : index.end();
                r.src[s] = it != index.end() ? &recs[it->second] : nullptr;
            }
            if (t->op == GGML_OP_MUL_MAT && t->src[0] && weight_leaf(t->src[0]) && make_weights) {
                sam3b200_weight *w = weight_of(t->src[0]);
                if (!w) return false;
                recs[index.at(t->src[0])].extra = w;
            }
        }
        for (size_t i : order) nodes.push_back(&recs[i]);
        return true;
    }
};

// ---- backend ------------------------------------------------------------------------------------

BackendCtx *be_ctx(ggml_backend_t b) { return static_cast<BackendCtx *>(b->context); }

const char *backend_get_name(ggml_backend_t b) { return be_ctx(b)->name; }

void backend_free(ggml_backend_t b) {
    BackendCtx *c = be_ctx(b);
    sam3b200_backend_free(c->be);
    delete c;
    delete b;
}

void backend_synchronize(ggml_backend_t b) {
    if (sam3b200_backend_synchronize(be_ctx(b)->be) != SAM3B200_STATUS_SUCCESS) report("synchronize");
}

ggml_status backend_graph_compute(ggml_backend_t b, ggml_cgraph *g) {
    Records r;
    if (!r.build(g, true)) return GGML_STATUS_ALLOC_FAILED;
    const int st = sam3b200_graph_compute(be_ctx(b)->be, r.nodes.data(), static_cast<int>(r.nodes.size()));
    if (st != SAM3B200_STATUS_SUCCESS) report("graph_compute");
    return static_cast<ggml_status>(st);
}

// ---- device -------------------------------------------------------------------------------------

Device *dev_device(ggml_backend_dev_t dev) { return static_cast<Device *>(dev->context); }

const char *dev_get_name(ggml_backend_dev_t dev) { return dev_device(dev)->name; }
const char *dev_get_description(ggml_backend_dev_t dev) { return sam3b200_backend_name(dev_device(dev)->copier()); }

void dev_get_memory(ggml_backend_dev_t dev, size_t *free, size_t *total) {
    if (sam3b200_device_memory(dev_device(dev)->id, free, total) != SAM3B200_STATUS_SUCCESS) *free = *total = 0;
}

ggml_backend_dev_type dev_get_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_GPU; }

ggml_backend_t dev_init_backend(ggml_backend_dev_t dev, const char *) {
    return ggml_backend_b200_init(dev_device(dev)->id);
}

ggml_backend_buffer_type_t dev_get_buffer_type(ggml_backend_dev_t dev) { return &dev_device(dev)->buft; }

// The op and its sources as records, checked by the library's node rules.  Weights have no layout
// yet here; the rules do not need one.
bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor *op) {
    Records r;
    r.add(op);
    const int nsrc = op->op == GGML_OP_CPY ? 1 : 4;
    for (int s = 0; s < nsrc; ++s)
        if (op->src[s]) r.add(op->src[s]);
    sam3b200_tensor &rec = r.recs[0];
    for (int s = 0; s < nsrc; ++s)
        rec.src[s] = op->src[s] ? &r.recs[r.index.at(op->src[s])] : nullptr;
    return sam3b200_supports_op(&rec) != 0;
}

bool dev_supports_buft(ggml_backend_dev_t dev, ggml_backend_buffer_type_t buft) {
    return buft == &dev_device(dev)->buft;
}

bool dev_offload_op(ggml_backend_dev_t, const ggml_tensor *) { return false; }

sam3b200_backend *Device::copier() {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!copier_) {
        copier_ = sam3b200_backend_init(id);
        if (!copier_) report("backend init");
    }
    return copier_;
}

// The device record needs no GPU until a buffer or a backend is made on it: op support is decided on
// the host.
Device *get_device(int id) {
    if (id < 0 || id >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    Device &d = g_devices[id];
    if (d.id == id) return &d;
    d.id = id;
    std::snprintf(d.name, sizeof d.name, "B200_%d", id);
    std::memset(&d.buft, 0, sizeof d.buft);
    d.buft.iface.get_name = buft_get_name;
    d.buft.iface.alloc_buffer = buft_alloc_buffer;
    d.buft.iface.get_alignment = buft_get_alignment;
    d.buft.iface.get_max_size = buft_get_max_size;
    d.buft.iface.get_alloc_size = buft_get_alloc_size;
    d.buft.iface.is_host = buft_is_host;
    d.buft.device = &d.dev;
    d.buft.context = &d;
    std::memset(&d.dev, 0, sizeof d.dev);
    d.dev.iface.get_name = dev_get_name;
    d.dev.iface.get_description = dev_get_description;
    d.dev.iface.get_memory = dev_get_memory;
    d.dev.iface.get_type = dev_get_type;
    d.dev.iface.init_backend = dev_init_backend;
    d.dev.iface.get_buffer_type = dev_get_buffer_type;
    d.dev.iface.supports_op = dev_supports_op;
    d.dev.iface.supports_buft = dev_supports_buft;
    d.dev.iface.offload_op = dev_offload_op;
    d.dev.reg = nullptr;
    d.dev.context = &d;
    return &d;
}

}  // namespace

extern "C" {

ggml_backend_t ggml_backend_b200_init(int device) {
    Device *d = get_device(device);
    if (!d) return nullptr;
    auto *c = new BackendCtx();
    c->d = d;
    c->be = sam3b200_backend_init(device);
    if (!c->be) {
        report("backend init");
        delete c;
        return nullptr;
    }
    std::snprintf(c->name, sizeof c->name, "B200_%d", device);
    auto *b = new ggml_backend();
    std::memset(&b->iface, 0, sizeof b->iface);
    b->guid = &g_guid;
    b->iface.get_name = backend_get_name;
    b->iface.free = backend_free;
    b->iface.synchronize = backend_synchronize;
    b->iface.graph_compute = backend_graph_compute;
    b->device = &d->dev;
    b->context = c;
    return b;
}

bool ggml_backend_is_b200(ggml_backend_t backend) {
    return backend && backend->iface.graph_compute == backend_graph_compute;
}

ggml_backend_buffer_type_t ggml_backend_b200_buffer_type(int device) {
    Device *d = get_device(device);
    return d ? &d->buft : nullptr;
}

int ggml_backend_b200_get_device_count(void) {
    int n = 0;
    return sam3b200_device_count(&n) == SAM3B200_STATUS_SUCCESS ? n : 0;
}

void *ggml_backend_b200_get_handle(ggml_backend_t backend) {
    return ggml_backend_is_b200(backend) ? be_ctx(backend)->be : nullptr;
}

}  // extern "C"
