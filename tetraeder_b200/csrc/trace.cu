// Routing traces, the `tetraeder-routing` v1 format of crates/memory/src/replay/trace.rs: one JSON
// header line (TraceHeader, serialised by serde_json), then little-endian binary records:
//   kind u8 (0 layer step, 1 hot-set refresh), step u32; a layer step goes on with layer u16,
//   n_tokens u32, flags u8 (bit 0 predicted, bit 1 predicted2), the routed ids (n_tokens * n_used,
//   token-major, id_bytes each: 1 when n_expert <= 256, else 2), then the predicted and depth-2
//   predicted ids when flagged.
// The reader replays recorded routing into the layer (the ids are returned as int32, as the
// kernels take them); the writer records the routing of a run.  Host code only.
#include <errno.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <utility>
#include <vector>

#include "../../include/tmoe.h"

namespace {

constexpr const char *kFormat = "tetraeder-routing";
constexpr uint32_t kVersion = 1;
constexpr uint32_t kMaxStepTokens = 1u << 20;  // MAX_STEP_TOKENS: a larger count is a corrupt record
constexpr uint8_t kKindStep = 0, kKindRefresh = 1, kFlagPredicted = 1, kFlagPredicted2 = 2;

thread_local std::string t_error;

int tfail(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_error = buf;
    return code;
}

// ---------------------------------------------------------------- a small JSON reader (RFC 8259)
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    bool is_uint = false;  // an integer literal without sign, fraction or exponent that fits u64
    uint64_t u = 0;
    std::string s;
    std::vector<Json> a;
    std::vector<std::pair<std::string, Json>> o;
};

struct Parser {
    const char *p, *end;
    std::string err;
    int depth = 0;
    bool fail(const char *m) {
        if (err.empty()) err = m;
        return false;
    }
    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    static void put_utf8(std::string &out, uint32_t c) {
        if (c < 0x80) out += (char)c;
        else if (c < 0x800) out += (char)(0xc0 | (c >> 6)), out += (char)(0x80 | (c & 0x3f));
        else if (c < 0x10000)
            out += (char)(0xe0 | (c >> 12)), out += (char)(0x80 | ((c >> 6) & 0x3f)), out += (char)(0x80 | (c & 0x3f));
        else
            out += (char)(0xf0 | (c >> 18)), out += (char)(0x80 | ((c >> 12) & 0x3f)),
                out += (char)(0x80 | ((c >> 6) & 0x3f)), out += (char)(0x80 | (c & 0x3f));
    }
    bool hex4(uint32_t &v) {
        if (end - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string &out) {
        if (p >= end || *p != '"') return fail("expected a string");
        p++;
        while (p < end && *p != '"') {
            const unsigned char c = (unsigned char)*p;
            if (c < 0x20) return fail("control character in a string");
            if (c != '\\') {
                out += (char)c, p++;
                continue;
            }
            if (++p >= end) return fail("truncated escape");
            const char e = *p++;
            switch (e) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                uint32_t v;
                if (!hex4(v)) return false;
                if (v >= 0xd800 && v < 0xdc00) {  // a surrogate pair
                    uint32_t lo;
                    if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
                    p += 2;
                    if (!hex4(lo) || lo < 0xdc00 || lo >= 0xe000) return fail("bad surrogate pair");
                    v = 0x10000 + ((v - 0xd800) << 10) + (lo - 0xdc00);
                } else if (v >= 0xdc00 && v < 0xe000) {
                    return fail("lone surrogate");
                }
                put_utf8(out, v);
                break;
            }
            default: return fail("bad escape");
            }
        }
        if (p >= end) return fail("unterminated string");
        p++;
        return true;
    }
    bool number(Json &j) {
        const char *s = p;
        bool neg = false, frac = false;
        if (p < end && *p == '-') neg = true, p++;
        if (p >= end || *p < '0' || *p > '9') return fail("bad number");
        if (*p == '0') p++;
        else
            while (p < end && *p >= '0' && *p <= '9') p++;
        if (p < end && *p == '.') {
            frac = true, p++;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            frac = true, p++;
            if (p < end && (*p == '+' || *p == '-')) p++;
            if (p >= end || *p < '0' || *p > '9') return fail("bad number");
            while (p < end && *p >= '0' && *p <= '9') p++;
        }
        j.kind = Json::Num;
        if (!neg && !frac) {
            uint64_t v = 0;
            bool fits = true;
            for (const char *q = s; q < p; q++) {
                const uint64_t d = (uint64_t)(*q - '0');
                if (v > (UINT64_MAX - d) / 10) fits = false;
                v = v * 10 + d;
            }
            j.is_uint = fits, j.u = v;
        }
        return true;
    }
    bool lit(const char *w) {
        const size_t n = strlen(w);
        if ((size_t)(end - p) < n || memcmp(p, w, n) != 0) return fail("bad literal");
        p += n;
        return true;
    }
    bool value(Json &j) {
        if (++depth > 64) return fail("nested too deeply");
        ws();
        if (p >= end) return fail("unexpected end");
        bool ok;
        switch (*p) {
        case '{': ok = object(j); break;
        case '[': ok = array(j); break;
        case '"': j.kind = Json::Str, ok = string(j.s); break;
        case 't': j.kind = Json::Bool, j.b = true, ok = lit("true"); break;
        case 'f': j.kind = Json::Bool, j.b = false, ok = lit("false"); break;
        case 'n': j.kind = Json::Null, ok = lit("null"); break;
        default: ok = number(j);
        }
        depth--;
        return ok;
    }
    bool array(Json &j) {
        j.kind = Json::Arr, p++;
        ws();
        if (p < end && *p == ']') return p++, true;
        for (;;) {
            j.a.emplace_back();
            if (!value(j.a.back())) return false;
            ws();
            if (p < end && *p == ',') {
                p++;
                continue;
            }
            if (p < end && *p == ']') return p++, true;
            return fail("expected , or ]");
        }
    }
    bool object(Json &j) {
        j.kind = Json::Obj, p++;
        ws();
        if (p < end && *p == '}') return p++, true;
        for (;;) {
            ws();
            std::string k;
            if (!string(k)) return false;
            ws();
            if (p >= end || *p != ':') return fail("expected :");
            p++;
            Json v;
            if (!value(v)) return false;
            j.o.emplace_back(std::move(k), std::move(v));
            ws();
            if (p < end && *p == ',') {
                p++;
                continue;
            }
            if (p < end && *p == '}') return p++, true;
            return fail("expected , or }");
        }
    }
};

// ---------------------------------------------------------------- TraceHeader
struct Header {
    std::string format, model, hot_source, prompt_hash;
    uint32_t version = 0, n_layer = 0, n_expert = 0, n_used = 0, vram_slots = 0, ram_slots = 0, prefetch_depth = 0,
             ubatch = 0;
    uint32_t id_bytes = 0;
    std::vector<uint64_t> expert_bytes;
    bool has_profile = false;
    std::vector<std::vector<uint64_t>> profile;
};

uint32_t id_bytes_for(uint32_t n_expert) { return n_expert <= 256 ? 1 : 2; }

// The header from its JSON (serde's rules for TraceHeader: every field but `profile` required,
// unknown fields ignored, a repeated field an error, integers in their type's range), then
// TraceHeader::check (trace.rs:75-89).
bool parse_header(const std::string &text, Header &h, std::string &err) {
    Parser ps{text.data(), text.data() + text.size()};
    Json j;
    if (!ps.value(j)) return err = "trace header: " + ps.err, false;
    ps.ws();
    if (ps.p != ps.end) return err = "trace header: trailing characters", false;
    if (j.kind != Json::Obj) return err = "trace header: not an object", false;
    const char *names[] = {"format",         "version",    "model",       "n_layer",    "n_expert",
                           "n_used",         "id_bytes",   "vram_slots",  "ram_slots",  "prefetch_depth",
                           "hot_source",     "ubatch",     "prompt_hash", "expert_bytes", "profile"};
    constexpr int NF = 15;
    const Json *f[NF] = {};
    for (const auto &kv : j.o)
        for (int i = 0; i < NF; i++)
            if (kv.first == names[i]) {
                if (f[i]) return err = std::string("trace header: duplicate field `") + names[i] + "`", false;
                f[i] = &kv.second;
            }
    for (int i = 0; i < NF - 1; i++)
        if (!f[i]) return err = std::string("trace header: missing field `") + names[i] + "`", false;
    auto str = [&](int i, std::string &out) {
        if (f[i]->kind != Json::Str) return err = std::string("trace header: `") + names[i] + "` is not a string", false;
        out = f[i]->s;
        return true;
    };
    auto uint = [&](const Json &v, uint64_t max, uint64_t &out, const char *name) {
        if (v.kind != Json::Num || !v.is_uint || v.u > max)
            return err = std::string("trace header: `") + name + "` is not an integer in range", false;
        out = v.u;
        return true;
    };
    uint64_t t;
    uint32_t *u32s[] = {&h.version,   &h.n_layer,        &h.n_expert, &h.n_used, &h.vram_slots,
                        &h.ram_slots, &h.prefetch_depth, &h.ubatch};
    const int u32i[] = {1, 3, 4, 5, 7, 8, 9, 11};
    for (int k = 0; k < 8; k++) {
        if (!uint(*f[u32i[k]], UINT32_MAX, t, names[u32i[k]])) return false;
        *u32s[k] = (uint32_t)t;
    }
    if (!uint(*f[6], 255, t, "id_bytes")) return false;
    h.id_bytes = (uint32_t)t;
    if (!str(0, h.format) || !str(2, h.model) || !str(10, h.hot_source) || !str(12, h.prompt_hash)) return false;
    if (f[13]->kind != Json::Arr) return err = "trace header: `expert_bytes` is not an array", false;
    for (const Json &v : f[13]->a) {
        if (!uint(v, UINT64_MAX, t, "expert_bytes")) return false;
        h.expert_bytes.push_back(t);
    }
    if (f[14] && f[14]->kind != Json::Null) {
        if (f[14]->kind != Json::Arr) return err = "trace header: `profile` is not an array", false;
        h.has_profile = true;
        for (const Json &row : f[14]->a) {
            if (row.kind != Json::Arr) return err = "trace header: `profile` is not an array of arrays", false;
            h.profile.emplace_back();
            for (const Json &v : row.a) {
                if (!uint(v, UINT64_MAX, t, "profile")) return false;
                h.profile.back().push_back(t);
            }
        }
    }
    // TraceHeader::check
    if (h.format != kFormat || h.version != kVersion) {
        char b[256];
        snprintf(b, sizeof(b), "not a %s v%u trace (%s v%u)", kFormat, kVersion, h.format.c_str(), h.version);
        return err = b, false;
    }
    if (h.id_bytes != id_bytes_for(h.n_expert) || h.n_used == 0)
        return err = "inconsistent header (id_bytes or n_used)", false;
    if (h.expert_bytes.size() != h.n_layer) return err = "expert_bytes must have one entry per layer", false;
    return true;
}

// serde_json's compact form of a string (escapes: quote, backslash, the short control escapes,
// other control characters as \u00XX; everything else, non-ASCII included, as is).
void put_json_string(std::string &out, const std::string &s) {
    out += '"';
    for (unsigned char c : s) {
        switch (c) {
        case '"': out += "\\\""; break;
        case '\\': out += "\\\\"; break;
        case '\b': out += "\\b"; break;
        case '\f': out += "\\f"; break;
        case '\n': out += "\\n"; break;
        case '\r': out += "\\r"; break;
        case '\t': out += "\\t"; break;
        default:
            if (c < 0x20) {
                char b[8];
                snprintf(b, sizeof(b), "\\u%04x", c);
                out += b;
            } else {
                out += (char)c;
            }
        }
    }
    out += '"';
}

// The header as serde_json writes TraceHeader: fields in declaration order, `profile` left out
// when absent.
std::string header_json(const Header &h) {
    std::string o = "{\"format\":";
    put_json_string(o, h.format);
    auto num = [&](const char *k, uint64_t v) { o += ",\""; o += k; o += "\":"; o += std::to_string(v); };
    num("version", h.version);
    o += ",\"model\":";
    put_json_string(o, h.model);
    num("n_layer", h.n_layer);
    num("n_expert", h.n_expert);
    num("n_used", h.n_used);
    num("id_bytes", h.id_bytes);
    num("vram_slots", h.vram_slots);
    num("ram_slots", h.ram_slots);
    num("prefetch_depth", h.prefetch_depth);
    o += ",\"hot_source\":";
    put_json_string(o, h.hot_source);
    num("ubatch", h.ubatch);
    o += ",\"prompt_hash\":";
    put_json_string(o, h.prompt_hash);
    o += ",\"expert_bytes\":[";
    for (size_t i = 0; i < h.expert_bytes.size(); i++) o += (i ? "," : "") + std::to_string(h.expert_bytes[i]);
    o += "]";
    if (h.has_profile) {
        o += ",\"profile\":[";
        for (size_t r = 0; r < h.profile.size(); r++) {
            o += r ? ",[" : "[";
            for (size_t i = 0; i < h.profile[r].size(); i++) o += (i ? "," : "") + std::to_string(h.profile[r][i]);
            o += "]";
        }
        o += "]";
    }
    o += "}";
    return o;
}

}  // namespace

struct tmoe_trace {
    FILE *f = nullptr;
    Header h;
    std::string line;  // the header line as read
    // the current record
    int32_t kind = -1, flags = 0, layer = 0;
    uint32_t step = 0, n_tokens = 0;
    std::vector<int32_t> ids[3];
    bool broken = false;  // a record failed: the stream position is unknown
    ~tmoe_trace() {
        if (f) fclose(f);
    }
};

struct tmoe_trace_writer {
    FILE *f = nullptr;
    Header h;
    std::string path;
    ~tmoe_trace_writer() {
        if (f) fclose(f);
    }
};

namespace {

bool read_exact(FILE *f, void *dst, size_t n) { return fread(dst, 1, n, f) == n; }

// read_ids (trace.rs:265-285): n ids of id_bytes each; only what the file holds is allocated.
int read_ids(tmoe_trace *t, size_t n, std::vector<int32_t> &out) {
    const size_t w = t->h.id_bytes;
    out.clear();
    uint8_t buf[4096];
    while (out.size() < n) {
        const size_t k = std::min(n - out.size(), sizeof(buf) / w);
        if (!read_exact(t->f, buf, k * w)) return tfail(TMOE_E_INVALID, "routing trace: unexpected end of file");
        for (size_t i = 0; i < k; i++) {
            const uint32_t e = w == 1 ? buf[i] : (uint32_t)buf[2 * i] | ((uint32_t)buf[2 * i + 1] << 8);
            if (e >= t->h.n_expert) return tfail(TMOE_E_INVALID, "routing trace: expert id out of range");
            out.push_back((int32_t)e);
        }
    }
    return TMOE_OK;
}

}  // namespace

extern "C" {

const char *tmoe_trace_last_error(void) { return t_error.c_str(); }

int tmoe_trace_open(const char *path, tmoe_trace **out) {
    if (!path || !out) return tfail(TMOE_E_INVALID, "null argument");
    *out = nullptr;
    FILE *f = fopen(path, "rb");
    if (!f) return tfail(TMOE_E_INVALID, "cannot read routing trace `%s`: %s", path, strerror(errno));
    tmoe_trace *t = new tmoe_trace;
    t->f = f;
    for (;;) {  // the header line (TraceReader::new, trace.rs:236-254)
        const int c = fgetc(f);
        if (c == EOF) {
            delete t;
            return tfail(TMOE_E_INVALID, "routing trace `%s`: unexpected end of file in the header", path);
        }
        if (c == '\n') break;
        t->line += (char)c;
        if (t->line.size() > (64u << 20)) {
            delete t;
            return tfail(TMOE_E_INVALID, "trace header too long");
        }
    }
    std::string err;
    if (!parse_header(t->line, t->h, err)) {
        delete t;
        return tfail(TMOE_E_INVALID, "%s", err.c_str());
    }
    *out = t;
    return TMOE_OK;
}

void tmoe_trace_close(tmoe_trace *t) { delete t; }

int tmoe_trace_header(const tmoe_trace *t, tmoe_trace_info *info) {
    if (!t || !info) return tfail(TMOE_E_INVALID, "null argument");
    const Header &h = t->h;
    info->version = h.version, info->n_layer = h.n_layer, info->n_expert = h.n_expert, info->n_used = h.n_used;
    info->id_bytes = h.id_bytes, info->vram_slots = h.vram_slots, info->ram_slots = h.ram_slots;
    info->prefetch_depth = h.prefetch_depth, info->ubatch = h.ubatch, info->has_profile = h.has_profile;
    return TMOE_OK;
}

const char *tmoe_trace_header_json(const tmoe_trace *t) { return t ? t->line.c_str() : nullptr; }

const char *tmoe_trace_header_str(const tmoe_trace *t, const char *field) {
    if (!t || !field) return nullptr;
    if (!strcmp(field, "format")) return t->h.format.c_str();
    if (!strcmp(field, "model")) return t->h.model.c_str();
    if (!strcmp(field, "hot_source")) return t->h.hot_source.c_str();
    if (!strcmp(field, "prompt_hash")) return t->h.prompt_hash.c_str();
    return nullptr;
}

int tmoe_trace_expert_bytes(const tmoe_trace *t, uint64_t *out) {
    if (!t || !out) return tfail(TMOE_E_INVALID, "null argument");
    memcpy(out, t->h.expert_bytes.data(), t->h.expert_bytes.size() * 8);
    return TMOE_OK;
}

int tmoe_trace_profile(const tmoe_trace *t, int64_t *rows, int64_t *cols, uint64_t *out) {
    if (!t) return tfail(TMOE_E_INVALID, "null argument");
    if (!t->h.has_profile) return tfail(TMOE_E_NOTFOUND, "the trace carries no routing profile");
    const int64_t r = (int64_t)t->h.profile.size();
    int64_t c = r ? (int64_t)t->h.profile[0].size() : 0;
    for (const auto &row : t->h.profile)
        if ((int64_t)row.size() != c) c = -1;
    if (rows) *rows = r;
    if (cols) *cols = c;
    if (c < 0) return tfail(TMOE_E_INVALID, "the routing profile is ragged");
    if (out)
        for (int64_t i = 0; i < r; i++) memcpy(out + i * c, t->h.profile[(size_t)i].data(), (size_t)c * 8);
    return TMOE_OK;
}

int tmoe_trace_next(tmoe_trace *t, int32_t *kind, uint32_t *step, int32_t *layer, uint32_t *n_tokens,
                    int32_t *flags) {
    if (!t) return tfail(TMOE_E_INVALID, "null argument");
    if (t->broken) return tfail(TMOE_E_INVALID, "routing trace: a previous record was corrupt");
    t->kind = -1;
    for (auto &v : t->ids) v.clear();
    const int k = fgetc(t->f);
    if (k == EOF) return 0;  // a clean end at a record boundary
    t->broken = true;        // until the record is complete
    uint32_t s;
    if (!read_exact(t->f, &s, 4)) return tfail(TMOE_E_INVALID, "routing trace: unexpected end of file");
    if (k == kKindRefresh) {
        t->kind = 1, t->step = s, t->n_tokens = 0, t->flags = 0, t->layer = 0;
    } else if (k == kKindStep) {
        uint16_t l;
        uint32_t n;
        uint8_t fl;
        if (!read_exact(t->f, &l, 2) || !read_exact(t->f, &n, 4))
            return tfail(TMOE_E_INVALID, "routing trace: unexpected end of file");
        if (n > kMaxStepTokens) return tfail(TMOE_E_INVALID, "%u tokens in one step", n);
        if (!read_exact(t->f, &fl, 1)) return tfail(TMOE_E_INVALID, "routing trace: unexpected end of file");
        const size_t cnt = (size_t)n * t->h.n_used;
        int rc = read_ids(t, cnt, t->ids[0]);
        if (!rc && (fl & kFlagPredicted)) rc = read_ids(t, cnt, t->ids[1]);
        if (!rc && (fl & kFlagPredicted2)) rc = read_ids(t, cnt, t->ids[2]);
        if (rc) return rc;
        t->kind = 0, t->step = s, t->layer = l, t->n_tokens = n;
        t->flags = fl & (kFlagPredicted | kFlagPredicted2);
    } else {
        return tfail(TMOE_E_INVALID, "unknown record kind %d", k);
    }
    t->broken = false;
    if (kind) *kind = t->kind;
    if (step) *step = t->step;
    if (layer) *layer = t->layer;
    if (n_tokens) *n_tokens = t->n_tokens;
    if (flags) *flags = t->flags;
    return 1;
}

int tmoe_trace_ids(const tmoe_trace *t, int32_t which, int32_t *out) {
    if (!t || !out || which < 0 || which > 2) return tfail(TMOE_E_INVALID, "bad argument");
    if (t->kind != 0) return tfail(TMOE_E_INVALID, "the current record is not a layer step");
    if (which > 0 && !(t->flags & (which == 1 ? kFlagPredicted : kFlagPredicted2)))
        return tfail(TMOE_E_NOTFOUND, "the step carries no %s ids", which == 1 ? "predicted" : "predicted2");
    memcpy(out, t->ids[which].data(), t->ids[which].size() * 4);
    return TMOE_OK;
}

int tmoe_trace_create(const char *path, const char *header_json_text, tmoe_trace_writer **out) {
    if (!path || !header_json_text || !out) return tfail(TMOE_E_INVALID, "null argument");
    *out = nullptr;
    tmoe_trace_writer *w = new tmoe_trace_writer;
    std::string err;
    if (!parse_header(header_json_text, w->h, err)) {
        delete w;
        return tfail(TMOE_E_INVALID, "%s", err.c_str());
    }
    w->f = fopen(path, "wb");
    if (!w->f) {
        delete w;
        return tfail(TMOE_E_INVALID, "cannot create routing trace `%s`: %s", path, strerror(errno));
    }
    const std::string line = header_json(w->h) + "\n";
    if (fwrite(line.data(), 1, line.size(), w->f) != line.size()) {
        delete w;
        return tfail(TMOE_E_INVALID, "writing routing trace `%s`: %s", path, strerror(errno));
    }
    w->path = path;
    *out = w;
    return TMOE_OK;
}

// TraceWriter::layer_step (trace.rs:141-170): ids and predictions are n_tokens * n_used int32,
// token-major; ids outside [0, n_expert) are an error and nothing is written.
int tmoe_trace_write_step(tmoe_trace_writer *w, uint32_t step, int32_t layer, uint32_t n_tokens, const int32_t *ids,
                          const int32_t *predicted, const int32_t *predicted2) {
    if (!w || (!ids && n_tokens)) return tfail(TMOE_E_INVALID, "null argument");
    if (layer < 0 || layer > 65535) return tfail(TMOE_E_INVALID, "layer %d out of range", layer);
    if (n_tokens > kMaxStepTokens) return tfail(TMOE_E_INVALID, "%u tokens in one step", n_tokens);
    const size_t n = (size_t)n_tokens * w->h.n_used;
    const int32_t *vs[3] = {ids, predicted, predicted2};
    std::string rec;
    rec += (char)kKindStep;
    rec.append(reinterpret_cast<const char *>(&step), 4);
    const uint16_t l = (uint16_t)layer;
    rec.append(reinterpret_cast<const char *>(&l), 2);
    rec.append(reinterpret_cast<const char *>(&n_tokens), 4);
    rec += (char)((predicted ? kFlagPredicted : 0) | (predicted2 ? kFlagPredicted2 : 0));
    for (const int32_t *v : vs) {
        if (!v) continue;
        for (size_t i = 0; i < n; i++) {
            const int32_t e = v[i];
            if (e < 0 || (uint32_t)e >= w->h.n_expert) return tfail(TMOE_E_INVALID, "expert id %d out of range", e);
            rec += (char)(e & 0xff);
            if (w->h.id_bytes == 2) rec += (char)((e >> 8) & 0xff);
        }
    }
    if (fwrite(rec.data(), 1, rec.size(), w->f) != rec.size())
        return tfail(TMOE_E_INVALID, "writing routing trace `%s`: %s", w->path.c_str(), strerror(errno));
    return TMOE_OK;
}

int tmoe_trace_write_refresh(tmoe_trace_writer *w, uint32_t step) {
    if (!w) return tfail(TMOE_E_INVALID, "null argument");
    char rec[5];
    rec[0] = (char)kKindRefresh;
    memcpy(rec + 1, &step, 4);
    if (fwrite(rec, 1, 5, w->f) != 5)
        return tfail(TMOE_E_INVALID, "writing routing trace `%s`: %s", w->path.c_str(), strerror(errno));
    return TMOE_OK;
}

int tmoe_trace_finish(tmoe_trace_writer *w) {
    if (!w) return tfail(TMOE_E_INVALID, "null argument");
    const bool ok = fflush(w->f) == 0;
    const int e = errno;
    const std::string path = w->path;
    delete w;
    return ok ? TMOE_OK : tfail(TMOE_E_INVALID, "writing routing trace `%s`: %s", path.c_str(), strerror(e));
}

}  // extern "C"
