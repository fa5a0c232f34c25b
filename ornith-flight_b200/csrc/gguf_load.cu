// gguf_load.cu — GGUF file -> HBM: the MoE layer's tensors uploaded as
// stored (raw Q4_K / Q6_K blocks, F32 router and gate vector), so every
// expert stays resident on the device instead of being streamed from disk
// per token (the reference reads slices with pread per token,
// engine/src/gguf.c:588-601, and caches them in host memory).
//
// The parser follows the GGUF container format (version <= 3): magic, version,
// tensor count, metadata count, metadata (key, type, value; arrays nested),
// tensor infos (name, dims, type, offset), data at the next multiple of
// general.alignment (default 32). Parameters are looked up with the
// architecture prefix (general.architecture + "." + name), as
// engine/src/gguf.c:726-744 does. Tensor bytes are read with pread into a
// pinned staging buffer and copied to the device in chunks (two buffers, so
// reading the next chunk overlaps the copy of the previous one).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

struct TensorInfo {
    std::string name;
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t offset;  // from the start of the data section
    uint64_t n_elems;
    uint64_t n_bytes;  // 0 when the type's size is not known here
};

struct MetaU {
    std::string key;
    uint32_t type;
    uint64_t u;      // integer values
    double f;        // float values
    std::string s;   // string values
};

// Bytes of n elements of a ggml type (block types: bytes per block / block).
uint64_t type_bytes(uint32_t t, uint64_t n) {
    switch (t) {
    case 0: return n * 4;                      // F32
    case 1: return n * 2;                      // F16
    case 30: return n * 2;                     // BF16
    case 2: return n % 32 ? 0 : n / 32 * 18;   // Q4_0
    case 3: return n % 32 ? 0 : n / 32 * 20;   // Q4_1
    case 8: return n % 32 ? 0 : n / 32 * 34;   // Q8_0
    case 10: return n % 256 ? 0 : n / 256 * 84;   // Q2_K
    case 11: return n % 256 ? 0 : n / 256 * 110;  // Q3_K
    case 12: return n % 256 ? 0 : n / 256 * 144;  // Q4_K
    case 13: return n % 256 ? 0 : n / 256 * 176;  // Q5_K
    case 14: return n % 256 ? 0 : n / 256 * 210;  // Q6_K
    case 15: return n % 256 ? 0 : n / 256 * 292;  // Q8_K
    default: return 0;
    }
}

}  // namespace

struct ofb_gguf {
    int fd = -1;
    uint64_t file_size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32, data_offset = 0;
    std::string arch;
    std::vector<MetaU> meta;
    std::vector<TensorInfo> tensors;
};

namespace {

struct Reader {
    int fd;
    uint64_t pos, size;
    bool ok = true;
    bool get(void *dst, size_t n) {
        if (!ok || pos + n > size) { ok = false; return false; }
        if (pread(fd, dst, n, (off_t)pos) != (ssize_t)n) { ok = false; return false; }
        pos += n;
        return true;
    }
    uint32_t u32() { uint32_t v = 0; get(&v, 4); return v; }
    uint64_t u64() { uint64_t v = 0; get(&v, 8); return v; }
    std::string str() {
        const uint64_t n = u64();
        if (!ok || n > (1u << 20)) { ok = false; return {}; }
        std::string s(n, '\0');
        get(&s[0], n);
        return s;
    }
};

// One metadata value of type t; scalars kept, arrays skipped.
bool read_value(Reader &r, uint32_t t, MetaU &m, int depth = 0) {
    switch (t) {
    case 0: case 1: case 7: { uint8_t v = 0; r.get(&v, 1); m.u = v; break; }
    case 2: case 3: { uint16_t v = 0; r.get(&v, 2); m.u = v; break; }
    case 4: case 5: m.u = r.u32(); break;
    case 6: { float v = 0; r.get(&v, 4); m.f = v; break; }
    case 8: m.s = r.str(); break;
    case 9: {
        if (depth > 4) return false;
        const uint32_t et = r.u32();
        const uint64_t n = r.u64();
        MetaU tmp;
        for (uint64_t i = 0; i < n && r.ok; i++)
            if (!read_value(r, et, tmp, depth + 1)) return false;
        break;
    }
    case 10: case 11: m.u = r.u64(); break;
    case 12: { double v = 0; r.get(&v, 8); m.f = v; break; }
    default: return false;
    }
    return r.ok;
}

const TensorInfo *find(const ofb_gguf *g, const char *name) {
    for (const TensorInfo &t : g->tensors)
        if (t.name == name) return &t;
    return nullptr;
}

}  // namespace

using namespace ofb;

extern "C" int ofb_gguf_open(const char *path, ofb_gguf **out) {
    if (!path || !out) { set_error("ofb_gguf_open: NULL argument"); return OFB_EINVAL; }
    const int fd = open(path, O_RDONLY);
    if (fd < 0) { set_error("ofb_gguf_open: cannot open %s", path); return OFB_EINVAL; }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); set_error("ofb_gguf_open: fstat failed"); return OFB_EINVAL; }
    ofb_gguf *g = new ofb_gguf;
    g->fd = fd;
    g->file_size = (uint64_t)st.st_size;
    Reader r{fd, 0, g->file_size};
    uint32_t magic = r.u32();
    g->version = r.u32();
    const uint64_t nt = r.u64(), nm = r.u64();
    if (!r.ok || magic != 0x46554747u || g->version < 1 || g->version > 3 || nt > (1u << 24) || nm > (1u << 24)) {
        delete g;
        close(fd);
        set_error("ofb_gguf_open: %s is not a GGUF file of version 1-3", path);
        return OFB_EINVAL;
    }
    for (uint64_t i = 0; i < nm && r.ok; i++) {
        MetaU m;
        m.key = r.str();
        m.type = r.u32();
        m.u = 0;
        m.f = 0;
        if (!read_value(r, m.type, m)) { r.ok = false; break; }
        if (m.key == "general.architecture" && m.type == 8) g->arch = m.s;
        if (m.key == "general.alignment" && m.type == 4 && m.u) g->alignment = m.u;
        g->meta.push_back(std::move(m));
    }
    for (uint64_t i = 0; i < nt && r.ok; i++) {
        TensorInfo t;
        t.name = r.str();
        t.n_dims = r.u32();
        if (t.n_dims > 4) { r.ok = false; break; }
        t.n_elems = 1;
        for (int d = 0; d < 4; d++) {
            t.dims[d] = d < (int)t.n_dims ? r.u64() : 1;
            t.n_elems *= t.dims[d];
        }
        t.type = r.u32();
        t.offset = r.u64();
        t.n_bytes = type_bytes(t.type, t.n_elems);
        g->tensors.push_back(std::move(t));
    }
    if (!r.ok) {
        delete g;
        close(fd);
        set_error("ofb_gguf_open: %s is truncated or malformed", path);
        return OFB_EINVAL;
    }
    g->data_offset = (r.pos + g->alignment - 1) / g->alignment * g->alignment;
    for (const TensorInfo &t : g->tensors)
        if (t.n_bytes && g->data_offset + t.offset + t.n_bytes > g->file_size) {
            set_error("ofb_gguf_open: tensor %s runs past the end of the file", t.name.c_str());
            close(fd);
            delete g;
            return OFB_EINVAL;
        }
    *out = g;
    return OFB_OK;
}

extern "C" int ofb_gguf_close(ofb_gguf *g) {
    if (!g) return OFB_OK;
    if (g->fd >= 0) close(g->fd);
    delete g;
    return OFB_OK;
}

extern "C" int ofb_gguf_tensor(const ofb_gguf *g, const char *name, int *type, int *n_dims, uint64_t dims[4],
                               uint64_t *file_offset, uint64_t *n_bytes) {
    if (!g || !name) { set_error("ofb_gguf_tensor: NULL argument"); return OFB_EINVAL; }
    const TensorInfo *t = find(g, name);
    if (!t) { set_error("ofb_gguf_tensor: no tensor %s", name); return OFB_EINVAL; }
    if (type) *type = (int)t->type;
    if (n_dims) *n_dims = (int)t->n_dims;
    if (dims) for (int d = 0; d < 4; d++) dims[d] = t->dims[d];
    if (file_offset) *file_offset = g->data_offset + t->offset;
    if (n_bytes) *n_bytes = t->n_bytes;
    return OFB_OK;
}

extern "C" int ofb_gguf_param_u32(const ofb_gguf *g, const char *param, uint32_t *value) {
    if (!g || !param || !value) { set_error("ofb_gguf_param_u32: NULL argument"); return OFB_EINVAL; }
    const std::string key = (g->arch.empty() ? std::string("unknown") : g->arch) + "." + param;
    for (const MetaU &m : g->meta)
        if (m.key == key && (m.type == 4 || m.type == 5)) {
            *value = (uint32_t)m.u;
            return OFB_OK;
        }
    set_error("ofb_gguf_param_u32: no %s", key.c_str());
    return OFB_EINVAL;
}

extern "C" int ofb_gguf_upload(const ofb_gguf *g, const char *name, void *dst, uint64_t capacity, void *stream) {
    if (!g || !name || !dst) { set_error("ofb_gguf_upload: NULL argument"); return OFB_EINVAL; }
    const TensorInfo *t = find(g, name);
    if (!t) { set_error("ofb_gguf_upload: no tensor %s", name); return OFB_EINVAL; }
    if (!t->n_bytes) { set_error("ofb_gguf_upload: %s has a type (%u) this loader cannot size", name, t->type); return OFB_EUNSUPPORTED; }
    if (t->n_bytes > capacity) { set_error("ofb_gguf_upload: %s needs %llu bytes", name, (unsigned long long)t->n_bytes); return OFB_ETOOLARGE; }
    constexpr size_t CHUNK = 32u << 20;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t *stage = nullptr;
    cudaError_t e = cudaHostAlloc((void **)&stage, 2 * CHUNK, cudaHostAllocDefault);
    if (e != cudaSuccess) return cuda_status(e, "ofb_gguf_upload: staging");
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (int i = 0; i < 2 && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
    const uint64_t base = g->data_offset + t->offset;
    int st = OFB_OK;
    for (uint64_t off = 0, k = 0; e == cudaSuccess && off < t->n_bytes; off += CHUNK, k++) {
        const size_t n = (size_t)std::min<uint64_t>(CHUNK, t->n_bytes - off);
        uint8_t *buf = stage + (k & 1) * CHUNK;
        if (k >= 2) e = cudaEventSynchronize(done[k & 1]);  // this half's previous copy is done
        if (e != cudaSuccess) break;
        if (pread(g->fd, buf, n, (off_t)(base + off)) != (ssize_t)n) {
            set_error("ofb_gguf_upload: read of %s failed", name);
            st = OFB_EINVAL;
            break;
        }
        e = cudaMemcpyAsync(static_cast<uint8_t *>(dst) + off, buf, n, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaEventRecord(done[k & 1], s);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    for (int i = 0; i < 2; i++) if (done[i]) cudaEventDestroy(done[i]);
    cudaFreeHost(stage);
    if (st) return st;
    return e == cudaSuccess ? OFB_OK : cuda_status(e, "ofb_gguf_upload");
}

// The MoE tensors of one layer, allocated on the current device and uploaded.
extern "C" int ofb_gguf_upload_moe_layer(const ofb_gguf *g, int layer, int layout, ofb_gguf_moe_layer *out,
                                         void *stream) {
    if (!g || !out || layer < 0 || (layout != OFB_LAYOUT_CONTIGUOUS && layout != OFB_LAYOUT_INTERLEAVED)) {
        set_error("ofb_gguf_upload_moe_layer: bad arguments");
        return OFB_EINVAL;
    }
    memset(out, 0, sizeof(*out));
    char nm[128];
    auto tname = [&](const char *what) { snprintf(nm, sizeof(nm), "blk.%d.%s", layer, what); return nm; };
    const TensorInfo *tg = find(g, tname("ffn_gate_exps.weight"));
    const TensorInfo *tu = find(g, tname("ffn_up_exps.weight"));
    const TensorInfo *td = find(g, tname("ffn_down_exps.weight"));
    const TensorInfo *tr = find(g, tname("ffn_gate_inp.weight"));
    if (!tg || !tu || !td || tg->type != OFB_TYPE_Q4_K || tu->type != OFB_TYPE_Q4_K || td->type != OFB_TYPE_Q6_K) {
        set_error("ofb_gguf_upload_moe_layer: layer %d lacks Q4_K gate/up and Q6_K down expert tensors", layer);
        return OFB_EUNSUPPORTED;
    }
    uint32_t D = 0, H = 0, E = 0, K = 0;
    ofb_gguf_param_u32(g, "embedding_length", &D);
    ofb_gguf_param_u32(g, "expert_feed_forward_length", &H);
    ofb_gguf_param_u32(g, "expert_count", &E);
    ofb_gguf_param_u32(g, "expert_used_count", &K);
    if (!D) D = (uint32_t)tg->dims[0];
    if (!E) E = (uint32_t)tg->dims[2];
    if (!H) H = E ? (uint32_t)(tg->n_elems / ((uint64_t)D * E)) : 0;
    if (!K) K = 8;
    if ((uint64_t)D * H * E != tg->n_elems || tu->n_elems != tg->n_elems || td->n_elems != tg->n_elems) {
        set_error("ofb_gguf_upload_moe_layer: expert tensors do not match d_model %u x hidden %u x %u experts", D, H, E);
        return OFB_EINVAL;
    }
    if (tr && (tr->type != OFB_TYPE_F32 || tr->n_elems != (uint64_t)D * E)) {
        set_error("ofb_gguf_upload_moe_layer: router must be F32 [%u x %u]", D, E);
        return OFB_EUNSUPPORTED;
    }
    out->cfg = ofb_moe_config{(int)D, (int)H, (int)E, (int)K, layout, OFB_ROUTE_FORWARD, 1, 1};
    const void **slots[8] = {(const void **)&out->weights.router, &out->weights.gate_exps, &out->weights.up_exps,
                             &out->weights.down_exps, &out->weights.gate_shexp, &out->weights.up_shexp,
                             &out->weights.down_shexp, (const void **)&out->weights.shexp_gate};
    const char *names[8] = {"ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                            "ffn_down_exps.weight", "ffn_gate_shexp.weight", "ffn_up_shexp.weight",
                            "ffn_down_shexp.weight", "ffn_gate_inp_shexp.weight"};
    int st = OFB_OK;
    for (int i = 0; i < 8 && !st; i++) {
        const TensorInfo *t = find(g, tname(names[i]));
        if (!t) continue;  // router, shared expert and its gate are optional
        if (!t->n_bytes) { set_error("ofb_gguf_upload_moe_layer: %s has an unsupported type", nm); st = OFB_EUNSUPPORTED; break; }
        void *p = nullptr;
        cudaError_t e = cudaMalloc(&p, t->n_bytes);
        if (e != cudaSuccess) { st = cuda_status(e, "ofb_gguf_upload_moe_layer: cudaMalloc"); break; }
        *slots[i] = p;
        st = ofb_gguf_upload(g, nm, p, t->n_bytes, stream);
    }
    const bool sh = out->weights.gate_shexp || out->weights.up_shexp || out->weights.down_shexp;
    if (!st && sh && !(out->weights.gate_shexp && out->weights.up_shexp && out->weights.down_shexp)) {
        set_error("ofb_gguf_upload_moe_layer: layer %d has an incomplete shared expert", layer);
        st = OFB_EINVAL;
    }
    out->cfg.shared_gate = out->weights.shexp_gate != nullptr;
    if (st) ofb_gguf_free_moe_layer(out);
    return st;
}

extern "C" int ofb_gguf_free_moe_layer(ofb_gguf_moe_layer *l) {
    if (!l) return OFB_OK;
    const void *p[8] = {l->weights.router, l->weights.gate_exps, l->weights.up_exps, l->weights.down_exps,
                        l->weights.gate_shexp, l->weights.up_shexp, l->weights.down_shexp, l->weights.shexp_gate};
    for (int i = 0; i < 8; i++)
        if (p[i]) cudaFree(const_cast<void *>(p[i]));
    memset(l, 0, sizeof(*l));
    return OFB_OK;
}
