// GGUF model files: the header reader of crates/model/src/gguf.rs (key-value metadata and the
// tensor index, split models merged, gguf.rs:236-400) and the tensor loader of
// load_weights (crates/model/src/qwen3moe.rs:2498-2584), which streams the bytes of a tensor --
// or of a contiguous run of its experts (TensorInfo::slab, gguf.rs:76-86) -- from the file into
// device memory.  Host code only.
//
// Format (GGUF version 3, little endian): "GGUF", u32 version, u64 n_tensors, u64 n_kv; n_kv
// entries {string key, u32 type, value}; n_tensors entries {string name, u32 n_dims, u64 ne[n_dims],
// u32 ggml type, u64 offset}; the data section starts at the next multiple of general.alignment
// (default 32) and each tensor's offset is relative to it.  Strings are u64 length + bytes.
#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/tmoe.h"

struct tmoe_gguf {
    struct KV {
        std::string key;
        int32_t kind = 0;
        uint64_t u = 0;
        int64_t i = 0;
        double f = 0.0;
        std::string s;
        uint64_t n = 0;  // array length
    };
    struct Tensor {
        std::string name;
        int32_t type = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        int32_t shard = 0;
        uint64_t offset = 0;  // absolute, in its shard file
        uint64_t nbytes = 0;
    };
    std::vector<std::string> paths;
    std::vector<int> fds;
    std::vector<KV> kv;  // the first shard's metadata
    std::unordered_map<std::string, size_t> kv_by_key;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
    uint64_t alignment = 32, data_offset = 0;
    // the loader's two pinned bounce buffers (portable), made on first use and kept until close
    mutable void *bounce[2] = {nullptr, nullptr};
    mutable uint64_t bounce_bytes = 0;
    ~tmoe_gguf() {
        for (void *b : bounce)
            if (b) cudaFreeHost(b);
        for (int fd : fds)
            if (fd >= 0) close(fd);
    }
};

namespace {

thread_local std::string g_error;

int gfail(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
    return code;
}

// ggml's type table as the format defines it: block size (elements) and bytes per block, by type
// id; ids that ggml removed have no entry (the reference's Type::from_id rejects them).
struct TypeSize {
    int32_t id;
    int32_t blck, bytes;
};
constexpr TypeSize kTypes[] = {
    {0, 1, 4},      {1, 1, 2},      {2, 32, 18},    {3, 32, 20},    {6, 32, 22},    {7, 32, 24},
    {8, 32, 34},    {9, 32, 40},    {10, 256, 84},  {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
    {14, 256, 210}, {15, 256, 292}, {16, 256, 66},  {17, 256, 74},  {18, 256, 98},  {19, 256, 50},
    {20, 32, 18},   {21, 256, 110}, {22, 256, 82},  {23, 256, 136}, {24, 1, 1},     {25, 1, 2},
    {26, 1, 4},     {27, 1, 8},     {28, 1, 8},     {29, 256, 56},  {30, 1, 2},     {34, 256, 54},
    {35, 256, 66},  {39, 32, 17},   {40, 64, 36},   {41, 128, 18},
};

const TypeSize *type_size(int32_t id) {
    for (const TypeSize &t : kTypes)
        if (t.id == id) return &t;
    return nullptr;
}

// Sequential little-endian reader over a file descriptor, buffered.
struct Reader {
    int fd;
    std::vector<uint8_t> buf = std::vector<uint8_t>(1 << 16);
    size_t pos = 0, len = 0;
    uint64_t consumed = 0;  // file offset of buf[pos]
    bool bad = false;
    explicit Reader(int f) : fd(f) {}
    bool fill() {
        if (pos < len) return true;
        const ssize_t r = ::read(fd, buf.data(), buf.size());
        if (r <= 0) return false;
        pos = 0, len = (size_t)r;
        return true;
    }
    bool bytes(void *dst, uint64_t n) {
        uint8_t *d = static_cast<uint8_t *>(dst);
        while (n) {
            if (!fill()) return bad = true, false;
            const size_t k = (size_t)std::min<uint64_t>(n, len - pos);
            if (d) memcpy(d, buf.data() + pos, k), d += k;
            pos += k, n -= k, consumed += k;
        }
        return true;
    }
    bool skip(uint64_t n) { return bytes(nullptr, n); }
    template <typename T>
    T get() {
        T v{};
        bytes(&v, sizeof(T));
        return v;
    }
    bool str(std::string &s, uint64_t cap = 1ull << 30) {
        const uint64_t n = get<uint64_t>();
        if (bad || n > cap) return bad = true, false;
        s.resize((size_t)n);
        return bytes(s.data(), n);
    }
};

// One value of kind `ty` (gguf.rs:181-216): integers widen to u64 (unsigned) or i64 (signed),
// floats to f64; arrays keep only their length.
bool read_value(Reader &r, uint32_t ty, tmoe_gguf::KV &v, std::string &err) {
    switch (ty) {
    case 0: v.kind = TMOE_GGUF_U64, v.u = r.get<uint8_t>(); break;
    case 1: v.kind = TMOE_GGUF_I64, v.i = r.get<int8_t>(); break;
    case 2: v.kind = TMOE_GGUF_U64, v.u = r.get<uint16_t>(); break;
    case 3: v.kind = TMOE_GGUF_I64, v.i = r.get<int16_t>(); break;
    case 4: v.kind = TMOE_GGUF_U64, v.u = r.get<uint32_t>(); break;
    case 5: v.kind = TMOE_GGUF_I64, v.i = r.get<int32_t>(); break;
    case 6: v.kind = TMOE_GGUF_F64, v.f = (double)r.get<float>(); break;
    case 7: v.kind = TMOE_GGUF_BOOL, v.u = r.get<uint8_t>() != 0; break;
    case 8: v.kind = TMOE_GGUF_STR; r.str(v.s); break;
    case 9: {
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        v.kind = TMOE_GGUF_ARRAY, v.n = n;
        uint64_t w = 0;
        if (et == 0 || et == 1 || et == 7) w = 1;
        else if (et == 2 || et == 3) w = 2;
        else if (et >= 4 && et <= 6) w = 4;
        else if (et >= 10 && et <= 12) w = 8;
        else if (et == 8) {
            for (uint64_t k = 0; k < n && !r.bad; k++) r.skip(r.get<uint64_t>());
            break;
        } else {
            err = "array of type " + std::to_string(et);
            return false;
        }
        if (n > (1ull << 40)) return r.bad = true, false;
        r.skip(n * w);
        break;
    }
    case 10: v.kind = TMOE_GGUF_U64, v.u = r.get<uint64_t>(); break;
    case 11: v.kind = TMOE_GGUF_I64, v.i = r.get<int64_t>(); break;
    case 12: v.kind = TMOE_GGUF_F64, v.f = r.get<double>(); break;
    default: err = "value type " + std::to_string(ty); return false;
    }
    return !r.bad;
}

struct Parsed {
    std::vector<tmoe_gguf::KV> kv;
    std::vector<tmoe_gguf::Tensor> tensors;
    uint64_t alignment = 32, data_offset = 0;
};

// parse_file (gguf.rs:326-400).  On failure returns a TMOE_E_* code with the message set.
int parse_file(int fd, const std::string &path, int shard, Parsed &out) {
    Reader r(fd);
    char magic[4];
    if (!r.bytes(magic, 4) || memcmp(magic, "GGUF", 4) != 0) return gfail(TMOE_E_INVALID, "%s: not a GGUF file (bad magic)", path.c_str());
    const uint32_t version = r.get<uint32_t>();
    if (version != 3) return gfail(TMOE_E_UNSUPPORTED, "%s: unsupported GGUF version %u", path.c_str(), version);
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (r.bad || n_tensors > (1u << 20) || n_kv > (1u << 20))
        return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: implausible counts", path.c_str());
    std::string err;
    for (uint64_t k = 0; k < n_kv; k++) {
        tmoe_gguf::KV v;
        if (!r.str(v.key, 1 << 16)) return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: truncated metadata", path.c_str());
        const uint32_t ty = r.get<uint32_t>();
        if (!read_value(r, ty, v, err))
            return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: %s", path.c_str(),
                         err.empty() ? "truncated metadata" : err.c_str());
        if (v.key == "general.alignment" && v.kind == TMOE_GGUF_U64 && v.u > 0) out.alignment = v.u;
        out.kv.push_back(std::move(v));
    }
    struct Raw {
        std::string name;
        int64_t ne[4];
        uint32_t type;
        uint64_t off;
    };
    std::vector<Raw> raw((size_t)n_tensors);
    for (Raw &t : raw) {
        if (!r.str(t.name, 1 << 16)) return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: truncated tensor index", path.c_str());
        const uint32_t nd = r.get<uint32_t>();
        if (nd < 1 || nd > 4)
            return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: tensor `%s` has %u dims", path.c_str(), t.name.c_str(), nd);
        for (int d = 0; d < 4; d++) t.ne[d] = d < (int)nd ? (int64_t)r.get<uint64_t>() : 1;
        t.type = r.get<uint32_t>();
        t.off = r.get<uint64_t>();
        if (r.bad) return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: truncated tensor index", path.c_str());
    }
    out.data_offset = (r.consumed + out.alignment - 1) / out.alignment * out.alignment;
    for (Raw &t : raw) {
        const TypeSize *ts = type_size((int32_t)t.type);
        if (!ts)
            return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: tensor `%s` has type id %u", path.c_str(), t.name.c_str(),
                         t.type);
        if (t.ne[0] <= 0 || t.ne[0] % ts->blck != 0)
            return gfail(TMOE_E_INVALID, "%s: corrupt GGUF: tensor `%s` row is not block aligned", path.c_str(),
                         t.name.c_str());
        tmoe_gguf::Tensor x;
        x.name = std::move(t.name);
        x.type = (int32_t)t.type;
        memcpy(x.ne, t.ne, sizeof(x.ne));
        x.shard = shard;
        x.offset = out.data_offset + t.off;
        x.nbytes = (uint64_t)(t.ne[0] / ts->blck) * (uint64_t)ts->bytes * (uint64_t)t.ne[1] * (uint64_t)t.ne[2] *
                   (uint64_t)t.ne[3];
        out.tensors.push_back(std::move(x));
    }
    return TMOE_OK;
}

// The entry of `key`; a repeated key: the last one (the reference's map keeps the last insert).
const tmoe_gguf::KV *find_kv(const std::vector<tmoe_gguf::KV> &kv, const char *key) {
    for (size_t i = kv.size(); i-- > 0;)
        if (kv[i].key == key) return &kv[i];
    return nullptr;
}

// kv_int (gguf.rs:120-126): an unsigned value, or a non-negative signed one.
bool kv_int(const std::vector<tmoe_gguf::KV> &kv, const char *key, uint64_t &out) {
    const tmoe_gguf::KV *v = find_kv(kv, key);
    if (!v) return false;
    if (v->kind == TMOE_GGUF_U64) return out = v->u, true;
    if (v->kind == TMOE_GGUF_I64 && v->i >= 0) return out = (uint64_t)v->i, true;
    return false;
}

// shard_path (gguf.rs:130-141): `<prefix>-00001-of-0000N.gguf` -> `<prefix>-0000k-of-0000N.gguf`.
bool shard_path(const std::string &first, uint64_t count, uint64_t no, std::string &out) {
    char suffix[64];
    snprintf(suffix, sizeof(suffix), "-%05u-of-%05llu.gguf", 1u, (unsigned long long)count);
    const size_t slash = first.find_last_of('/');
    const std::string dir = slash == std::string::npos ? "" : first.substr(0, slash + 1);
    const std::string name = slash == std::string::npos ? first : first.substr(slash + 1);
    const size_t sl = strlen(suffix);
    if (name.size() < sl || name.compare(name.size() - sl, sl, suffix) != 0) return false;
    char tail[64];
    snprintf(tail, sizeof(tail), "-%05llu-of-%05llu.gguf", (unsigned long long)(no + 1), (unsigned long long)count);
    out = dir + name.substr(0, name.size() - sl) + tail;
    return true;
}

int open_fd(const std::string &path, int &fd) {
    fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) return gfail(TMOE_E_INVALID, "cannot read GGUF `%s`: %s", path.c_str(), strerror(errno));
    return TMOE_OK;
}

// pread of exactly n bytes.
int read_at(int fd, uint64_t off, void *dst, uint64_t n, const char *what) {
    uint8_t *d = static_cast<uint8_t *>(dst);
    while (n) {
        const size_t k = (size_t)std::min<uint64_t>(n, 1ull << 30);
        const ssize_t r = pread(fd, d, k, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return gfail(TMOE_E_INVALID, "reading %s: %s", what, r < 0 ? strerror(errno) : "unexpected end of file");
        d += r, off += (uint64_t)r, n -= (uint64_t)r;
    }
    return TMOE_OK;
}

// read_at over up to kReadThreads threads, each a contiguous slice (page-cache copies scale with
// cores; one thread is bound by one core's copy rate).
constexpr int kReadThreads = 8;
constexpr uint64_t kSliceMin = 8ull << 20;

int read_parallel(int fd, uint64_t off, uint8_t *dst, uint64_t n, const char *what) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int T = (int)std::min<uint64_t>({(uint64_t)kReadThreads, (uint64_t)hw, std::max<uint64_t>(1, n / kSliceMin)});
    if (T <= 1) return read_at(fd, off, dst, n, what);
    std::vector<int> err(T, 0);
    std::vector<std::thread> th;
    const uint64_t slice = (n / T + 4095) & ~4095ull;
    for (int i = 0; i < T; i++) {
        const uint64_t a = std::min(n, (uint64_t)i * slice), b = std::min(n, a + slice);
        th.emplace_back([=, &err] {
            uint64_t o = a;
            while (o < b) {
                const ssize_t r = pread(fd, dst + o, (size_t)std::min<uint64_t>(b - o, 1ull << 30), (off_t)(off + o));
                if (r < 0 && errno == EINTR) continue;
                if (r <= 0) {
                    err[i] = r < 0 ? errno : -1;
                    return;
                }
                o += (uint64_t)r;
            }
        });
    }
    for (auto &t : th) t.join();
    for (int e : err)
        if (e) return gfail(TMOE_E_INVALID, "reading %s: %s", what, e > 0 ? strerror(e) : "unexpected end of file");
    return TMOE_OK;
}

int check_range(const tmoe_gguf *g, int64_t t, uint64_t off, uint64_t n) {
    if (!g || t < 0 || t >= (int64_t)g->tensors.size()) return gfail(TMOE_E_INVALID, "no tensor %lld", (long long)t);
    const tmoe_gguf::Tensor &x = g->tensors[(size_t)t];
    if (off > x.nbytes || n > x.nbytes - off)
        return gfail(TMOE_E_INVALID, "bytes [%llu, +%llu) outside tensor `%s` (%llu bytes)", (unsigned long long)off,
                     (unsigned long long)n, x.name.c_str(), (unsigned long long)x.nbytes);
    return TMOE_OK;
}

}  // namespace

extern "C" {

const char *tmoe_gguf_last_error(void) { return g_error.c_str(); }

int tmoe_gguf_open(const char *path, tmoe_gguf **out) {
    if (!path || !out) return gfail(TMOE_E_INVALID, "null argument");
    *out = nullptr;
    tmoe_gguf *g = new tmoe_gguf;
    auto bail = [&](int rc) {
        delete g;
        return rc;
    };
    int fd = -1;
    int rc = open_fd(path, fd);
    if (rc) return bail(rc);
    g->fds.push_back(fd);
    g->paths.push_back(path);
    Parsed first;
    if ((rc = parse_file(fd, path, 0, first))) return bail(rc);
    uint64_t count = 1;
    kv_int(first.kv, "split.count", count);
    if (count == 0) count = 1;
    if (count > 1) {  // gguf.rs:241-279
        uint64_t no = 1;
        if (!kv_int(first.kv, "split.no", no) || no != 0)
            return bail(gfail(TMOE_E_INVALID, "split GGUF: `%s` is not the first shard; open the -00001-of-%05llu file",
                              path, (unsigned long long)count));
        if (count > (1u << 16)) return bail(gfail(TMOE_E_INVALID, "split GGUF: %llu shards", (unsigned long long)count));
        for (uint64_t k = 1; k < count; k++) {
            std::string p;
            if (!shard_path(path, count, k, p))
                return bail(gfail(TMOE_E_INVALID, "split GGUF: `%s` should be named `<prefix>-00001-of-%05llu.gguf`",
                                  path, (unsigned long long)count));
            int sfd = -1;
            if ((rc = open_fd(p, sfd))) return bail(rc);
            g->fds.push_back(sfd);
            g->paths.push_back(p);
            Parsed sh;
            if ((rc = parse_file(sfd, p, (int)k, sh))) return bail(rc);
            uint64_t sno = ~0ull, scount = 0;
            if (!kv_int(sh.kv, "split.no", sno) || sno != k || !kv_int(sh.kv, "split.count", scount) || scount != count)
                return bail(gfail(TMOE_E_INVALID, "split GGUF: `%s` is not shard %llu of %llu", p.c_str(),
                                  (unsigned long long)(k + 1), (unsigned long long)count));
            for (auto &t : sh.tensors) first.tensors.push_back(std::move(t));
        }
        uint64_t declared = 0;
        if (!kv_int(first.kv, "split.tensors.count", declared) || declared != first.tensors.size())
            return bail(gfail(TMOE_E_INVALID, "split GGUF: %zu tensors in the shards, split.tensors.count says %llu",
                              first.tensors.size(), (unsigned long long)declared));
    }
    g->kv = std::move(first.kv);
    g->tensors = std::move(first.tensors);
    g->alignment = first.alignment;
    g->data_offset = first.data_offset;
    for (size_t i = 0; i < g->kv.size(); i++) g->kv_by_key[g->kv[i].key] = i;  // a repeated key: the last wins
    for (size_t i = 0; i < g->tensors.size(); i++)
        if (!g->by_name.emplace(g->tensors[i].name, i).second)
            return bail(gfail(TMOE_E_INVALID, "corrupt GGUF: duplicate tensor `%s`", g->tensors[i].name.c_str()));
    // every tensor lies inside its file
    for (const auto &t : g->tensors) {
        struct stat st;
        if (fstat(g->fds[(size_t)t.shard], &st) != 0 || t.offset + t.nbytes > (uint64_t)st.st_size)
            return bail(gfail(TMOE_E_INVALID, "corrupt GGUF: tensor `%s` runs past the end of `%s`", t.name.c_str(),
                              g->paths[(size_t)t.shard].c_str()));
    }
    *out = g;
    return TMOE_OK;
}

void tmoe_gguf_close(tmoe_gguf *g) { delete g; }

int32_t tmoe_gguf_n_shards(const tmoe_gguf *g) { return g ? (int32_t)g->paths.size() : TMOE_E_INVALID; }

int64_t tmoe_gguf_n_tensors(const tmoe_gguf *g) { return g ? (int64_t)g->tensors.size() : TMOE_E_INVALID; }

int64_t tmoe_gguf_find_tensor(const tmoe_gguf *g, const char *name) {
    if (!g || !name) return TMOE_E_INVALID;
    const auto it = g->by_name.find(name);
    return it == g->by_name.end() ? -1 : (int64_t)it->second;
}

int tmoe_gguf_tensor_info(const tmoe_gguf *g, int64_t i, const char **name, int32_t *type, int64_t *ne,
                          int32_t *shard, uint64_t *offset, uint64_t *nbytes) {
    if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return gfail(TMOE_E_INVALID, "no tensor %lld", (long long)i);
    const tmoe_gguf::Tensor &t = g->tensors[(size_t)i];
    if (name) *name = t.name.c_str();
    if (type) *type = t.type;
    if (ne) memcpy(ne, t.ne, sizeof(t.ne));
    if (shard) *shard = t.shard;
    if (offset) *offset = t.offset;
    if (nbytes) *nbytes = t.nbytes;
    return TMOE_OK;
}

int64_t tmoe_gguf_n_kv(const tmoe_gguf *g) { return g ? (int64_t)g->kv.size() : TMOE_E_INVALID; }

int tmoe_gguf_kv_key(const tmoe_gguf *g, int64_t i, const char **key) {
    if (!g || !key || i < 0 || i >= (int64_t)g->kv.size()) return gfail(TMOE_E_INVALID, "no key-value entry %lld", (long long)i);
    *key = g->kv[(size_t)i].key.c_str();
    return TMOE_OK;
}

int tmoe_gguf_kv(const tmoe_gguf *g, const char *key, int32_t *kind, uint64_t *u, int64_t *i, double *f,
                 const char **s, uint64_t *n) {
    if (!g || !key) return gfail(TMOE_E_INVALID, "null argument");
    const auto it = g->kv_by_key.find(key);
    if (it == g->kv_by_key.end()) return gfail(TMOE_E_NOTFOUND, "missing key `%s`", key);
    const tmoe_gguf::KV &v = g->kv[it->second];
    if (kind) *kind = v.kind;
    if (u) *u = v.u;
    if (i) *i = v.i;
    if (f) *f = v.f;
    if (s) *s = v.s.c_str();
    if (n) *n = v.n;
    return TMOE_OK;
}

int tmoe_gguf_type_size(int32_t type, int32_t *block_elems, int32_t *block_bytes) {
    const TypeSize *ts = type_size(type);
    if (!ts) return gfail(TMOE_E_UNSUPPORTED, "ggml type id %d", type);
    if (block_elems) *block_elems = ts->blck;
    if (block_bytes) *block_bytes = ts->bytes;
    return TMOE_OK;
}

int tmoe_gguf_read(const tmoe_gguf *g, int64_t tensor, uint64_t offset, uint64_t nbytes, void *dst) {
    int rc = check_range(g, tensor, offset, nbytes);
    if (rc) return rc;
    if (nbytes && !dst) return gfail(TMOE_E_INVALID, "null destination");
    const tmoe_gguf::Tensor &t = g->tensors[(size_t)tensor];
    return read_parallel(g->fds[(size_t)t.shard], t.offset + offset, static_cast<uint8_t *>(dst), nbytes,
                         t.name.c_str());
}

// File -> device through the handle's two pinned bounce buffers: chunk k+1 is read from the file
// (by several threads) while chunk k crosses the host link (one cudaMemcpyAsync per chunk on
// `stream`, an event per buffer).  Returns when the last copy has landed.
int tmoe_gguf_load(const tmoe_gguf *g, int64_t tensor, uint64_t offset, uint64_t nbytes, void *dst, int32_t device,
                   void *stream) {
    int rc = check_range(g, tensor, offset, nbytes);
    if (rc) return rc;
    if (nbytes == 0) return TMOE_OK;
    if (!dst) return gfail(TMOE_E_INVALID, "null destination");
    const tmoe_gguf::Tensor &t = g->tensors[(size_t)tensor];
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return gfail(TMOE_E_CUDA, "cudaSetDevice(%d)", device);
    }
    cudaStream_t st = (cudaStream_t)stream;
    const uint64_t chunk = 64ull << 20;
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaError_t e = cudaSuccess;
    if (g->bounce_bytes < chunk) {
        for (int b = 0; b < 2 && e == cudaSuccess; b++) {
            if (g->bounce[b]) cudaFreeHost(g->bounce[b]), g->bounce[b] = nullptr;
            e = cudaHostAlloc(&g->bounce[b], (size_t)chunk, cudaHostAllocPortable);
        }
        g->bounce_bytes = e == cudaSuccess ? chunk : 0;
    }
    void *const bounce[2] = {g->bounce[0], g->bounce[1]};
    for (int b = 0; b < 2 && e == cudaSuccess; b++) e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
    uint64_t pos = 0;
    int k = 0;
    while (e == cudaSuccess && rc == TMOE_OK && pos < nbytes) {
        const int b = k & 1;
        const uint64_t n = std::min(chunk, nbytes - pos);
        if (k >= 2) e = cudaEventSynchronize(done[b]);  // the copy that last used this buffer
        if (e != cudaSuccess) break;
        rc = read_parallel(g->fds[(size_t)t.shard], t.offset + offset + pos, static_cast<uint8_t *>(bounce[b]), n,
                           t.name.c_str());
        if (rc) break;
        e = cudaMemcpyAsync(static_cast<uint8_t *>(dst) + pos, bounce[b], (size_t)n, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaEventRecord(done[b], st);
        pos += n, k++;
    }
    const cudaError_t es = cudaStreamSynchronize(st);  // no copy still reads a buffer when this returns
    if (e == cudaSuccess) e = es;
    for (int b = 0; b < 2; b++)
        if (done[b]) cudaEventDestroy(done[b]);
    cudaSetDevice(prev);
    if (rc) return rc;
    if (e != cudaSuccess) {
        cudaGetLastError();
        return gfail(TMOE_E_CUDA, "loading `%s`: %s", t.name.c_str(), cudaGetErrorString(e));
    }
    return TMOE_OK;
}

}  // extern "C"
