// gguf.inl — cpq_gguf_*: GGUF v1-v3 reader and tensor-parallel shard loader (host).
//
// The file side of codpiece-gguf (crates/codpiece-gguf/src/lib.rs:346-460:
// header, metadata KVs, tensor directory, no tensor data read at open) with
// the same checks: magic "GGUF", version 1..3, caps on counts, string and
// array lengths and dimensions, power-of-two alignment (general.alignment,
// default 32), and every tensor's [offset, offset + bytes) aligned, in order,
// non-overlapping and inside the data section. Then the loading side of
// Weights::load (crates/codpiece-model/src/lib.rs:128-311), which reads each
// tensor whole and lets ggml's meta backend slice it per device: here a shard
// is cut on the host by the split state (cpq_tp_split_state, split.rs) and
// written once, dense, to its device.

struct cpq_gguf {
    std::string path;
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_start = 0;
    uint64_t file_len = 0;
    struct Tensor {
        std::string name;
        int32_t type;
        int32_t n_dims;
        int64_t ne[4];
        uint64_t offset;  // from data_start
        uint64_t bytes;   // 0: unknown type
    };
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, uint64_t> kv_u64;     // non-negative integer values
    std::unordered_map<std::string, std::string> kv_str;  // string values
};

namespace cpq {

// Elements per block and bytes per block of the ggml types the directory can size.
static bool gguf_type_size(int32_t t, uint64_t *blk, uint64_t *bytes) {
    static const struct { int32_t t; uint64_t blk, bytes; } tab[] = {
        {0, 1, 4},    {1, 1, 2},    {2, 32, 18},  {3, 32, 20},  {6, 32, 22},  {7, 32, 24},   {8, 32, 34},
        {9, 32, 36},  {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176}, {14, 256, 210},
        {15, 256, 292}, {16, 256, 66}, {17, 256, 74}, {18, 256, 98}, {19, 256, 50}, {20, 32, 18},
        {21, 256, 110}, {22, 256, 82}, {23, 256, 136}, {24, 1, 1}, {25, 1, 2}, {26, 1, 4}, {27, 1, 8},
        {28, 1, 8}, {29, 256, 56}, {30, 1, 2}, {34, 256, 54}, {35, 256, 66}, {39, 32, 17},
    };
    for (const auto &e : tab)
        if (e.t == t) {
            *blk = e.blk;
            *bytes = e.bytes;
            return true;
        }
    return false;
}

struct GgufReader {
    FILE *f;
    bool wide;  // v2+: 64-bit lengths and counts
    bool ok = true;
    bool read(void *p, size_t n) {
        if (ok && std::fread(p, 1, n, f) != n) ok = false;
        return ok;
    }
    uint8_t u8() { uint8_t v = 0; read(&v, 1); return v; }
    uint16_t u16() { uint16_t v = 0; read(&v, 2); return v; }
    uint32_t u32() { uint32_t v = 0; read(&v, 4); return v; }
    uint64_t u64() { uint64_t v = 0; read(&v, 8); return v; }
    uint64_t len() { return wide ? u64() : u32(); }
    bool skip(uint64_t n) {
        if (ok && std::fseek(f, long(n), SEEK_CUR) != 0) ok = false;
        return ok;
    }
};

constexpr uint64_t kGgufMaxTensors = uint64_t(1) << 20;
constexpr uint64_t kGgufMaxKvs = uint64_t(1) << 20;
constexpr uint64_t kGgufMaxString = uint64_t(256) << 20;
constexpr uint32_t kGgufMaxDims = 8;

static cpq_status gguf_bad(const cpq_gguf *g, const char *fmt, const char *what = "") {
    return fail(CPQ_ERR_INVALID_ARG, "malformed GGUF %s: %s%s", g->path.c_str(), fmt, what);
}

// One metadata value of type ty (recorded under key when it is a
// non-negative integer or a string; arrays are skipped element by element).
static cpq_status gguf_value(GgufReader &r, cpq_gguf *g, const std::string &key, uint32_t ty, int depth) {
    auto put_u = [&](uint64_t v) { if (depth == 0) g->kv_u64[key] = v; };
    switch (ty) {
    case 0: put_u(r.u8()); break;
    case 1: { const int8_t v = int8_t(r.u8()); if (v >= 0) put_u(uint64_t(v)); break; }
    case 2: put_u(r.u16()); break;
    case 3: { const int16_t v = int16_t(r.u16()); if (v >= 0) put_u(uint64_t(v)); break; }
    case 4: put_u(r.u32()); break;
    case 5: { const int32_t v = int32_t(r.u32()); if (v >= 0) put_u(uint64_t(v)); break; }
    case 6: r.u32(); break;
    case 7: r.u8(); break;
    case 8: {
        const uint64_t n = r.len();
        if (n > kGgufMaxString) return gguf_bad(g, "string length exceeds the cap");
        if (depth == 0) {
            std::string s(size_t(n), '\0');
            r.read(&s[0], size_t(n));
            g->kv_str[key] = s;
        } else {
            r.skip(n);
        }
        break;
    }
    case 9: {
        if (depth > 2) return gguf_bad(g, "array nesting too deep");
        const uint32_t et = r.u32();
        const uint64_t n = r.len();
        if (n > kGgufMaxString) return gguf_bad(g, "array length exceeds the cap");
        static const int fixed[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (et < 13 && fixed[et] > 0) {
            r.skip(n * uint64_t(fixed[et]));
        } else {
            for (uint64_t i = 0; i < n && r.ok; i++) {
                cpq_status rc = gguf_value(r, g, key, et, depth + 1);
                if (rc) return rc;
            }
        }
        break;
    }
    case 10: put_u(r.u64()); break;
    case 11: { const int64_t v = int64_t(r.u64()); if (v >= 0) put_u(uint64_t(v)); break; }
    case 12: r.u64(); break;
    default: return gguf_bad(g, "unknown metadata value type");
    }
    return r.ok ? CPQ_SUCCESS : gguf_bad(g, "file ends inside the metadata");
}

}  // namespace cpq

extern "C" cpq_status cpq_gguf_open(const char *path, cpq_gguf **out) {
    using namespace cpq;
    if (!path || !out) return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_open: null argument");
    *out = nullptr;
    FILE *f = std::fopen(path, "rb");
    if (!f) return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_open: cannot open %s", path);
    std::unique_ptr<FILE, int (*)(FILE *)> closer(f, std::fclose);
    std::unique_ptr<cpq_gguf> g(new cpq_gguf);
    g->path = path;
    std::fseek(f, 0, SEEK_END);
    g->file_len = uint64_t(std::ftell(f));
    std::fseek(f, 0, SEEK_SET);
    GgufReader r{f, true};
    const uint32_t magic = r.u32();
    if (!r.ok || magic != 0x46554747u)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_open: %s: bad magic 0x%08x (not a GGUF file)", path, magic);
    g->version = r.u32();
    if (g->version < 1 || g->version > 3)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_gguf_open: %s: unsupported GGUF version %u", path, g->version);
    r.wide = g->version >= 2;
    const uint64_t n_tensors = r.len(), n_kvs = r.len();
    if (!r.ok) return gguf_bad(g.get(), "file ends inside the header");
    if (n_tensors > kGgufMaxTensors || n_kvs > kGgufMaxKvs) return gguf_bad(g.get(), "implausible tensor or KV count");
    for (uint64_t i = 0; i < n_kvs; i++) {
        const uint64_t n = r.len();
        if (!r.ok || n > kGgufMaxString) return gguf_bad(g.get(), "bad KV key");
        std::string key(size_t(n), '\0');
        r.read(&key[0], size_t(n));
        const uint32_t ty = r.u32();
        if (!r.ok) return gguf_bad(g.get(), "file ends inside the metadata");
        cpq_status rc = gguf_value(r, g.get(), key, ty, 0);
        if (rc) return rc;
    }
    auto al = g->kv_u64.find("general.alignment");
    if (al != g->kv_u64.end()) g->alignment = al->second;
    if (g->alignment == 0 || (g->alignment & (g->alignment - 1))) return gguf_bad(g.get(), "alignment is not a power of two");
    g->tensors.reserve(size_t(n_tensors));
    for (uint64_t i = 0; i < n_tensors; i++) {
        cpq_gguf::Tensor t;
        const uint64_t n = r.len();
        if (!r.ok || n > kGgufMaxString) return gguf_bad(g.get(), "bad tensor name");
        t.name.assign(size_t(n), '\0');
        r.read(&t.name[0], size_t(n));
        const uint32_t nd = r.u32();
        if (!r.ok || nd > kGgufMaxDims) return gguf_bad(g.get(), "too many dimensions in tensor ", t.name.c_str());
        if (nd > 4) return fail(CPQ_ERR_UNSUPPORTED, "cpq_gguf_open: tensor %s has %u dimensions", t.name.c_str(), nd);
        t.n_dims = int32_t(nd);
        uint64_t elems = 1;
        for (int d = 0; d < 4; d++) t.ne[d] = 1;
        for (uint32_t d = 0; d < nd; d++) {
            const uint64_t v = r.len();
            if (v > (uint64_t(1) << 40) || (v && elems > (uint64_t(1) << 50) / v))
                return gguf_bad(g.get(), "implausible dimensions in tensor ", t.name.c_str());
            t.ne[d] = int64_t(v);
            elems *= v;
        }
        t.type = int32_t(r.u32());
        t.offset = r.u64();
        if (!r.ok) return gguf_bad(g.get(), "file ends inside the tensor directory");
        uint64_t blk = 0, bb = 0;
        t.bytes = gguf_type_size(t.type, &blk, &bb) && elems % blk == 0 ? elems / blk * bb : 0;
        g->tensors.push_back(std::move(t));
    }
    const uint64_t pos = uint64_t(std::ftell(f));
    g->data_start = (pos + g->alignment - 1) / g->alignment * g->alignment;
    if (g->data_start > g->file_len) return gguf_bad(g.get(), "data section starts past the end of the file");
    const uint64_t data_len = g->file_len - g->data_start;
    uint64_t prev_end = 0;
    for (const auto &t : g->tensors) {
        if (t.offset % g->alignment) return gguf_bad(g.get(), "offset not aligned: tensor ", t.name.c_str());
        if (t.offset < prev_end) return gguf_bad(g.get(), "overlaps the previous tensor: ", t.name.c_str());
        if (t.bytes) {
            if (t.offset + t.bytes > data_len) return gguf_bad(g.get(), "exceeds the data section: ", t.name.c_str());
            prev_end = t.offset + t.bytes;
        } else {
            prev_end = t.offset;
        }
    }
    *out = g.release();
    return CPQ_SUCCESS;
}

extern "C" void cpq_gguf_close(cpq_gguf *g) { delete g; }

extern "C" int64_t cpq_gguf_n_tensors(const cpq_gguf *g) { return g ? int64_t(g->tensors.size()) : -1; }

extern "C" int64_t cpq_gguf_find_tensor(const cpq_gguf *g, const char *name) {
    if (!g || !name) return -1;
    for (size_t i = 0; i < g->tensors.size(); i++)
        if (g->tensors[i].name == name) return int64_t(i);
    return -1;
}

extern "C" cpq_status cpq_gguf_tensor_at(const cpq_gguf *g, int64_t i, cpq_gguf_tensor *out) {
    using namespace cpq;
    if (!g || !out || i < 0 || i >= int64_t(g->tensors.size()))
        return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_tensor_at: bad handle or index %lld", (long long)i);
    const auto &t = g->tensors[size_t(i)];
    out->name = t.name.c_str();
    out->type = t.type;
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; d++) out->ne[d] = t.ne[d];
    out->offset = g->data_start + t.offset;
    out->bytes = t.bytes;
    return CPQ_SUCCESS;
}

extern "C" cpq_status cpq_gguf_get_u64(const cpq_gguf *g, const char *key, uint64_t *out) {
    using namespace cpq;
    if (!g || !key || !out) return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_get_u64: null argument");
    auto it = g->kv_u64.find(key);
    if (it == g->kv_u64.end()) return fail(CPQ_ERR_INVALID_ARG, "GGUF key %s: absent or not a non-negative integer", key);
    *out = it->second;
    return CPQ_SUCCESS;
}

extern "C" cpq_status cpq_gguf_get_str(const cpq_gguf *g, const char *key, const char **out) {
    using namespace cpq;
    if (!g || !key || !out) return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_get_str: null argument");
    auto it = g->kv_str.find(key);
    if (it == g->kv_str.end()) return fail(CPQ_ERR_INVALID_ARG, "GGUF key %s: absent or not a string", key);
    *out = it->second.c_str();
    return CPQ_SUCCESS;
}

namespace cpq {

// The [start, length) pieces of an axis of `extent` elements that device d of
// n holds under split state st (NULL or MIRRORED: the whole axis): the axis is
// the sequence of segments s, each repeated nr[s] times, and every repetition
// is divided among the devices in device order (ne[s * n + d] elements each),
// the meta backend's layout (crates/codpiece-model/src/meta.rs:50-121).
static cpq_status shard_pieces(const cpq_split_state *st, int n, int d, int64_t extent,
                               std::vector<std::pair<int64_t, int64_t>> &pieces) {
    pieces.clear();
    if (!st || st->axis == CPQ_SPLIT_MIRRORED) {
        pieces.emplace_back(0, extent);
        return CPQ_SUCCESS;
    }
    if (n < 1 || d < 0 || d >= n || st->n_segments < 1 || st->n_segments > 16 || int64_t(st->n_segments) * n > 256)
        return fail(CPQ_ERR_INVALID_ARG, "shard: device %d of %d, %u segments", d, n, st->n_segments);
    int64_t pos = 0;
    for (uint32_t s = 0; s < st->n_segments; s++) {
        int64_t per = 0, off = 0;
        for (int q = 0; q < n; q++) {
            if (st->ne[s * n + q] < 0) return fail(CPQ_ERR_INVALID_ARG, "shard: negative extent");
            if (q < d) off += st->ne[s * n + q];
            per += st->ne[s * n + q];
        }
        const int64_t len = st->ne[s * n + d];
        for (uint32_t rep = 0; rep < st->nr[s]; rep++) {
            if (len > 0) pieces.emplace_back(pos + off, len);
            pos += per;
        }
    }
    if (pos != extent)
        return fail(CPQ_ERR_INVALID_ARG, "shard: the split covers %lld of %lld elements", (long long)pos, (long long)extent);
    return CPQ_SUCCESS;
}

// Shape of device d's shard of tensor t (2-D view: ne0 contiguous, ne1 rows).
static cpq_status gguf_shard_geometry(const cpq_gguf *g, int64_t i, const cpq_split_state *st, int n, int d,
                                      std::vector<std::pair<int64_t, int64_t>> &pieces, int64_t *ne0, int64_t *ne1,
                                      uint64_t *blk, uint64_t *bb) {
    if (!g || i < 0 || i >= int64_t(g->tensors.size())) return fail(CPQ_ERR_INVALID_ARG, "gguf shard: bad handle or index");
    const auto &t = g->tensors[size_t(i)];
    if (!t.bytes || !gguf_type_size(t.type, blk, bb))
        return fail(CPQ_ERR_UNSUPPORTED, "gguf shard: tensor %s has a type of unknown size", t.name.c_str());
    if (t.ne[2] != 1 || t.ne[3] != 1) return fail(CPQ_ERR_UNSUPPORTED, "gguf shard: tensor %s is not 2-D", t.name.c_str());
    const int axis = st ? st->axis : CPQ_SPLIT_MIRRORED;
    if (axis != CPQ_SPLIT_AXIS_0 && axis != CPQ_SPLIT_AXIS_1 && axis != CPQ_SPLIT_MIRRORED)
        return fail(CPQ_ERR_UNSUPPORTED, "gguf shard: split axis %d", axis);
    const int64_t extent = axis == CPQ_SPLIT_AXIS_1 ? t.ne[1] : t.ne[0];
    cpq_status rc = shard_pieces(axis == CPQ_SPLIT_MIRRORED ? nullptr : st, n, d, extent, pieces);
    if (rc) return rc;
    int64_t total = 0;
    for (const auto &p : pieces) {
        if (axis == CPQ_SPLIT_AXIS_0 && (p.first % int64_t(*blk) || p.second % int64_t(*blk)))
            return fail(CPQ_ERR_INVALID_ARG, "gguf shard: tensor %s: a K piece cuts a quant block", t.name.c_str());
        total += p.second;
    }
    *ne0 = axis == CPQ_SPLIT_AXIS_0 ? total : t.ne[0];
    *ne1 = axis == CPQ_SPLIT_AXIS_1 ? total : t.ne[1];
    return CPQ_SUCCESS;
}

// Reads device d's shard of tensor i into host memory (dense rows).
static cpq_status gguf_read_shard(const cpq_gguf *g, int64_t i, const cpq_split_state *st, int n, int d, uint8_t *dst,
                                  size_t dst_bytes) {
    std::vector<std::pair<int64_t, int64_t>> pieces;
    int64_t ne0 = 0, ne1 = 0;
    uint64_t blk = 1, bb = 1;
    cpq_status rc = gguf_shard_geometry(g, i, st, n, d, pieces, &ne0, &ne1, &blk, &bb);
    if (rc) return rc;
    const auto &t = g->tensors[size_t(i)];
    const size_t row = size_t(t.ne[0] / int64_t(blk)) * bb;  // bytes of a whole row in the file
    const size_t srow = size_t(ne0 / int64_t(blk)) * bb;     // bytes of a shard row
    if (!dst || dst_bytes < srow * size_t(ne1))
        return fail(CPQ_ERR_INVALID_ARG, "gguf shard: destination of %zu B < %zu B", dst_bytes, srow * size_t(ne1));
    FILE *f = std::fopen(g->path.c_str(), "rb");
    if (!f) return fail(CPQ_ERR_INVALID_ARG, "gguf shard: cannot reopen %s", g->path.c_str());
    std::unique_ptr<FILE, int (*)(FILE *)> closer(f, std::fclose);
    const uint64_t base = g->data_start + t.offset;
    auto read_at = [&](uint64_t off, void *p, size_t bytes) {
        return std::fseek(f, long(base + off), SEEK_SET) == 0 && std::fread(p, 1, bytes, f) == bytes;
    };
    const int axis = st ? st->axis : CPQ_SPLIT_MIRRORED;
    if (axis != CPQ_SPLIT_AXIS_0) {  // whole rows: one read per piece
        size_t at = 0;
        for (const auto &p : pieces) {
            const int64_t r0 = axis == CPQ_SPLIT_AXIS_1 ? p.first : 0, nr = axis == CPQ_SPLIT_AXIS_1 ? p.second : t.ne[1];
            if (!read_at(uint64_t(r0) * row, dst + at, size_t(nr) * row))
                return fail(CPQ_ERR_INVALID_ARG, "gguf shard: short read of %s", t.name.c_str());
            at += size_t(nr) * row;
        }
        return CPQ_SUCCESS;
    }
    // K pieces of every row: whole rows through a bounded staging buffer, then gathered
    const size_t batch = std::max<size_t>(1, (size_t(64) << 20) / row);
    std::vector<uint8_t> stage(batch * row);
    for (int64_t r0 = 0; r0 < t.ne[1]; r0 += int64_t(batch)) {
        const int64_t nr = std::min<int64_t>(int64_t(batch), t.ne[1] - r0);
        if (!read_at(uint64_t(r0) * row, stage.data(), size_t(nr) * row))
            return fail(CPQ_ERR_INVALID_ARG, "gguf shard: short read of %s", t.name.c_str());
        for (int64_t r = 0; r < nr; r++) {
            uint8_t *out = dst + size_t(r0 + r) * srow;
            for (const auto &p : pieces) {
                const size_t b0 = size_t(p.first / int64_t(blk)) * bb, nbytes = size_t(p.second / int64_t(blk)) * bb;
                std::memcpy(out, stage.data() + size_t(r) * row + b0, nbytes);
                out += nbytes;
            }
        }
    }
    return CPQ_SUCCESS;
}

}  // namespace cpq

extern "C" cpq_status cpq_gguf_shard_shape(const cpq_gguf *g, int64_t i, const cpq_split_state *split, int n_devices,
                                           int device_index, int64_t *ne0, int64_t *ne1, size_t *bytes) {
    using namespace cpq;
    if (!ne0 || !ne1 || !bytes) return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_shard_shape: null output");
    std::vector<std::pair<int64_t, int64_t>> pieces;
    uint64_t blk = 1, bb = 1;
    cpq_status rc = gguf_shard_geometry(g, i, split, n_devices, device_index, pieces, ne0, ne1, &blk, &bb);
    if (rc) return rc;
    *bytes = size_t(*ne0 / int64_t(blk)) * bb * size_t(*ne1);
    return CPQ_SUCCESS;
}

extern "C" cpq_status cpq_gguf_read_shard(const cpq_gguf *g, int64_t i, const cpq_split_state *split, int n_devices,
                                          int device_index, void *host_dst, size_t dst_bytes) {
    return cpq::gguf_read_shard(g, i, split, n_devices, device_index, static_cast<uint8_t *>(host_dst), dst_bytes);
}

extern "C" cpq_status cpq_gguf_load_shard(const cpq_gguf *g, int64_t i, const cpq_split_state *split, int n_devices,
                                          int device_index, void *device_dst, size_t dst_bytes) {
    using namespace cpq;
    int64_t ne0 = 0, ne1 = 0;
    size_t bytes = 0;
    cpq_status rc = cpq_gguf_shard_shape(g, i, split, n_devices, device_index, &ne0, &ne1, &bytes);
    if (rc) return rc;
    if (!device_dst || dst_bytes < bytes)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_gguf_load_shard: destination of %zu B < %zu B", dst_bytes, bytes);
    std::vector<uint8_t> host(bytes);
    if ((rc = gguf_read_shard(g, i, split, n_devices, device_index, host.data(), bytes))) return rc;
    const cudaError_t e = cudaMemcpy(device_dst, host.data(), bytes, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_gguf_load_shard: copy to the device");
}
