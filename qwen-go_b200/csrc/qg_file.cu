// On-disk quantised MoE layers: a read-only mapping of a safetensors file
// and the qgmoe_desc of one layer pointing into it (host code only).
//
// The reference loads quantised linears as <name>.qweight / <name>.scale
// pairs named in quant.json (model/load.go:478-582) and its MoE loader takes
// the stacked expert tensors only as f32 or bf16 blobs (model/load.go:
// 415-456).  This file reads the same naming extended to the stacked expert
// codes and scales, so qgmoe_create can copy a quantised layer from the
// mapping straight to the device.
//
// Safetensors: an 8-byte little-endian header length N, N bytes of JSON
// {"name": {"dtype": "F16", "shape": [..], "data_offsets": [begin, end]},
// "__metadata__": {...}}, then the data (offsets relative to its start).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "qg_common.cuh"

struct qgmoe_file {
    struct Tensor {
        int dtype = QGMOE_DT_OTHER;
        int rank = 0;
        int64_t shape[8] = {};
        uint64_t begin = 0, end = 0;
    };
    int fd = -1;
    void *map = nullptr;
    size_t size = 0;
    const uint8_t *data = nullptr;  // start of the tensor data
    uint64_t data_size = 0;
    std::unordered_map<std::string, Tensor> tensors;
    // float32 copies of bf16 vectors the descriptor needs as float32 (router,
    // shared-expert gate), owned by the handle
    mutable std::unordered_map<std::string, std::vector<float>> widened;
};

namespace qg {
namespace {

// Minimal JSON reader for safetensors headers: objects, arrays, strings,
// integers; other values are skipped.
struct Json {
    const char *p, *e;
    bool ok = true;

    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool eat(char c) {
        ws();
        if (p < e && *p == c) {
            p++;
            return true;
        }
        return false;
    }
    void expect(char c) {
        if (!eat(c)) ok = false;
    }
    static void put_utf8(std::string &o, unsigned cp) {
        if (cp < 0x80) {
            o += (char)cp;
        } else if (cp < 0x800) {
            o += (char)(0xC0 | (cp >> 6));
            o += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            o += (char)(0xE0 | (cp >> 12));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        } else {
            o += (char)(0xF0 | (cp >> 18));
            o += (char)(0x80 | ((cp >> 12) & 0x3F));
            o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(unsigned &v) {
        if (e - p < 4) return false;
        v = 0;
        for (int i = 0; i < 4; i++) {
            const char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    std::string str() {
        std::string o;
        ws();
        if (p >= e || *p != '"') {
            ok = false;
            return o;
        }
        p++;
        while (p < e && *p != '"') {
            if (*p != '\\') {
                o += *p++;
                continue;
            }
            if (++p >= e) break;
            const char c = *p++;
            switch (c) {
            case '"': o += '"'; break;
            case '\\': o += '\\'; break;
            case '/': o += '/'; break;
            case 'b': o += '\b'; break;
            case 'f': o += '\f'; break;
            case 'n': o += '\n'; break;
            case 'r': o += '\r'; break;
            case 't': o += '\t'; break;
            case 'u': {
                unsigned cp = 0;
                if (!hex4(cp)) {
                    ok = false;
                    return o;
                }
                if (cp >= 0xD800 && cp < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                    p += 2;
                    unsigned lo = 0;
                    if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) {
                        ok = false;
                        return o;
                    }
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                }
                put_utf8(o, cp);
                break;
            }
            default: ok = false; return o;
            }
        }
        if (p >= e) {
            ok = false;
            return o;
        }
        p++;  // closing quote
        return o;
    }
    int64_t integer() {
        ws();
        bool neg = false;
        if (p < e && *p == '-') {
            neg = true;
            p++;
        }
        if (p >= e || *p < '0' || *p > '9') {
            ok = false;
            return 0;
        }
        int64_t v = 0;
        while (p < e && *p >= '0' && *p <= '9') {
            if (v > (INT64_MAX - 9) / 10) {
                ok = false;
                return 0;
            }
            v = v * 10 + (*p++ - '0');
        }
        if (p < e && (*p == '.' || *p == 'e' || *p == 'E')) ok = false;  // not an integer
        return neg ? -v : v;
    }
    void skip(int depth = 0) {
        ws();
        if (p >= e || depth > 64) {
            ok = false;
            return;
        }
        if (*p == '"') {
            str();
        } else if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            p++;
            if (eat(close)) return;
            do {
                if (obj) {
                    str();
                    expect(':');
                }
                skip(depth + 1);
            } while (ok && eat(','));
            expect(close);
        } else {
            // number, true, false, null
            while (p < e && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n' &&
                   *p != '\r' && *p != '\t')
                p++;
        }
    }
};

int dtype_code(const std::string &s) {
    if (s == "F32") return QGMOE_DT_F32;
    if (s == "F16") return QGMOE_DT_F16;
    if (s == "BF16") return QGMOE_DT_BF16;
    if (s == "I8") return QGMOE_DT_I8;
    if (s == "U8") return QGMOE_DT_U8;
    if (s == "I32") return QGMOE_DT_I32;
    return QGMOE_DT_OTHER;
}

int dtype_bytes(int dt) {
    switch (dt) {
    case QGMOE_DT_F32: case QGMOE_DT_I32: return 4;
    case QGMOE_DT_F16: case QGMOE_DT_BF16: return 2;
    case QGMOE_DT_I8: case QGMOE_DT_U8: return 1;
    default: return 0;
    }
}

int parse_header(qgmoe_file *f, const char *h, size_t n) {
    Json j{h, h + n};
    j.expect('{');
    if (!j.ok) return set_error(QGMOE_ERR_INVALID_ARG, "safetensors header is not a JSON object");
    if (j.eat('}')) return QGMOE_OK;
    do {
        const std::string name = j.str();
        j.expect(':');
        if (!j.ok) break;
        if (name == "__metadata__") {
            j.skip();
            continue;
        }
        qgmoe_file::Tensor t;
        bool have_dt = false, have_shape = false, have_off = false;
        j.expect('{');
        if (!j.eat('}')) {
            do {
                const std::string key = j.str();
                j.expect(':');
                if (key == "dtype") {
                    t.dtype = dtype_code(j.str());
                    have_dt = true;
                } else if (key == "shape") {
                    j.expect('[');
                    if (!j.eat(']')) {
                        do {
                            const int64_t d = j.integer();
                            if (t.rank >= 8 || d < 0) j.ok = false;
                            else t.shape[t.rank++] = d;
                        } while (j.ok && j.eat(','));
                        j.expect(']');
                    }
                    have_shape = true;
                } else if (key == "data_offsets") {
                    j.expect('[');
                    const int64_t b = j.integer();
                    j.expect(',');
                    const int64_t en = j.integer();
                    j.expect(']');
                    if (b < 0 || en < b) j.ok = false;
                    t.begin = (uint64_t)b;
                    t.end = (uint64_t)en;
                    have_off = true;
                } else {
                    j.skip();
                }
            } while (j.ok && j.eat(','));
            j.expect('}');
        }
        if (!j.ok) break;
        if (!have_dt || !have_shape || !have_off)
            return set_error(QGMOE_ERR_INVALID_ARG, "tensor %s: dtype, shape or data_offsets missing",
                             name.c_str());
        if (t.end > f->data_size)
            return set_error(QGMOE_ERR_INVALID_ARG, "tensor %s: data beyond the end of the file",
                             name.c_str());
        const int eb = dtype_bytes(t.dtype);
        if (eb) {
            uint64_t numel = 1;
            for (int i = 0; i < t.rank; i++) {
                if (t.shape[i] && numel > UINT64_MAX / (uint64_t)t.shape[i])
                    return set_error(QGMOE_ERR_INVALID_ARG, "tensor %s: shape overflows", name.c_str());
                numel *= (uint64_t)t.shape[i];
            }
            if (numel > UINT64_MAX / (uint64_t)eb)
                return set_error(QGMOE_ERR_INVALID_ARG, "tensor %s: byte size overflows",
                                 name.c_str());
            if (numel * (uint64_t)eb != t.end - t.begin)
                return set_error(QGMOE_ERR_INVALID_ARG, "tensor %s: %llu bytes for its shape, %llu stored",
                                 name.c_str(), (unsigned long long)(numel * eb),
                                 (unsigned long long)(t.end - t.begin));
        }
        f->tensors[name] = t;
    } while (j.ok && j.eat(','));
    if (j.ok) j.expect('}');
    if (!j.ok) return set_error(QGMOE_ERR_INVALID_ARG, "malformed safetensors header");
    return QGMOE_OK;
}

const qgmoe_file::Tensor *find(const qgmoe_file *f, const std::string &name) {
    auto it = f->tensors.find(name);
    return it == f->tensors.end() ? nullptr : &it->second;
}

// One linear stack [G, O, K] (G = experts, or absent for a single linear):
// quantised <base>.qweight (I8/U8 [.., O, K] int8 or U8 [.., O, K/2] int4) +
// <base>.scale (F16/F32 [.., O, K/32]), or raw <base>.weight (BF16 -> bits
// 16, F32 -> bits 32; model/load.go:419-449 reads the stacked experts so).
struct LinStack {
    const void *w = nullptr, *s = nullptr;
    int bits = 0, sdt = -1;
    int64_t lead = 1, O = 0, K = 0;
};

int lin_stack(const qgmoe_file *f, const std::string &base, int want_rank, LinStack &o) {
    const auto *q = find(f, base + ".qweight");
    if (!q) {
        const auto *w = find(f, base + ".weight");
        if (!w)
            return set_error(QGMOE_ERR_INVALID_ARG, "%s.qweight / .weight not in the file",
                             base.c_str());
        if (w->rank != want_rank || (w->dtype != QGMOE_DT_BF16 && w->dtype != QGMOE_DT_F32))
            return set_error(QGMOE_ERR_INVALID_ARG, "%s.weight: BF16 or F32 of rank %d expected",
                             base.c_str(), want_rank);
        o.lead = 1;
        for (int i = 0; i < want_rank - 2; i++) o.lead *= w->shape[i];
        o.O = w->shape[want_rank - 2];
        o.K = w->shape[want_rank - 1];
        o.bits = w->dtype == QGMOE_DT_BF16 ? 16 : 32;
        o.w = f->data + w->begin;
        o.s = nullptr;
        o.sdt = -1;
        return QGMOE_OK;
    }
    const auto *s = find(f, base + ".scale");
    if (!s) return set_error(QGMOE_ERR_INVALID_ARG, "%s.scale not in the file", base.c_str());
    if (q->rank != want_rank || s->rank != want_rank)
        return set_error(QGMOE_ERR_INVALID_ARG, "%s: expected rank %d", base.c_str(), want_rank);
    if (q->dtype != QGMOE_DT_I8 && q->dtype != QGMOE_DT_U8)
        return set_error(QGMOE_ERR_INVALID_ARG, "%s.qweight: I8 or U8 expected", base.c_str());
    if (s->dtype != QGMOE_DT_F16 && s->dtype != QGMOE_DT_F32)
        return set_error(QGMOE_ERR_INVALID_ARG, "%s.scale: F16 or F32 expected", base.c_str());
    for (int i = 0; i < want_rank - 1; i++)
        if (q->shape[i] != s->shape[i])
            return set_error(QGMOE_ERR_INVALID_ARG, "%s: code and scale shapes disagree", base.c_str());
    o.lead = 1;
    for (int i = 0; i < want_rank - 2; i++) o.lead *= q->shape[i];
    o.O = q->shape[want_rank - 2];
    o.K = s->shape[want_rank - 1] * QG_GROUP;
    const int64_t qk = q->shape[want_rank - 1];
    if (qk == o.K) {
        o.bits = 8;
    } else if (2 * qk == o.K && q->dtype == QGMOE_DT_U8) {
        o.bits = 4;
    } else {
        return set_error(QGMOE_ERR_INVALID_ARG,
                         "%s: codes of width %lld do not match scales for %lld inputs",
                         base.c_str(), (long long)qk, (long long)o.K);
    }
    o.w = f->data + q->begin;
    o.s = f->data + s->begin;
    o.sdt = s->dtype == QGMOE_DT_F16 ? QGMOE_SCALE_F16 : QGMOE_SCALE_F32;
    return QGMOE_OK;
}

// A float32 vector the descriptor needs (router rows, shared-expert gate):
// F32 in the mapping as is, BF16 widened once into a buffer the handle owns.
const float *f32_view(const qgmoe_file *f, const std::string &name, const qgmoe_file::Tensor *t) {
    if (t->dtype == QGMOE_DT_F32) return reinterpret_cast<const float *>(f->data + t->begin);
    auto &v = f->widened[name];
    if (v.empty()) {
        const uint64_t n = (t->end - t->begin) / 2;
        v.resize(n);
        const uint8_t *b = f->data + t->begin;
        for (uint64_t i = 0; i < n; i++) {
            const uint32_t u = ((uint32_t)b[2 * i] | ((uint32_t)b[2 * i + 1] << 8)) << 16;
            memcpy(&v[i], &u, 4);
        }
    }
    return v.data();
}

}  // namespace
}  // namespace qg

using namespace qg;

extern "C" {

int qgmoe_file_open(const char *path, qgmoe_file_t **out) {
    if (!path || !out) return set_error(QGMOE_ERR_INVALID_ARG, "null path/out");
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(QGMOE_ERR_INVALID_ARG, "cannot open %s: %s", path, strerror(errno));
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size < 8) {
        close(fd);
        return set_error(QGMOE_ERR_INVALID_ARG, "%s: not a safetensors file (too short)", path);
    }
    void *map = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) {
        close(fd);
        return set_error(QGMOE_ERR_INVALID_ARG, "mmap %s: %s", path, strerror(errno));
    }
    qgmoe_file *f = new qgmoe_file();
    f->fd = fd;
    f->map = map;
    f->size = (size_t)st.st_size;
    const uint8_t *b = static_cast<const uint8_t *>(map);
    uint64_t n = 0;
    for (int i = 7; i >= 0; i--) n = (n << 8) | b[i];
    if (n > f->size - 8) {
        qgmoe_file_close(f);
        return set_error(QGMOE_ERR_INVALID_ARG, "%s: header length %llu beyond the file", path,
                         (unsigned long long)n);
    }
    f->data = b + 8 + n;
    f->data_size = f->size - 8 - n;
    const int rc = parse_header(f, reinterpret_cast<const char *>(b + 8), (size_t)n);
    if (rc) {
        qgmoe_file_close(f);
        return rc;
    }
    *out = f;
    return QGMOE_OK;
}

int qgmoe_file_close(qgmoe_file_t *f) {
    if (!f) return QGMOE_OK;
    if (f->map) munmap(f->map, f->size);
    if (f->fd >= 0) close(f->fd);
    delete f;
    return QGMOE_OK;
}

int qgmoe_file_tensor(const qgmoe_file_t *f, const char *name, int32_t *dtype, int32_t *rank,
                      int64_t *shape, const void **data, int64_t *nbytes) {
    if (!f || !name) return set_error(QGMOE_ERR_INVALID_ARG, "null file/name");
    const auto *t = find(f, name);
    if (!t) return set_error(QGMOE_ERR_INVALID_ARG, "no tensor %s", name);
    if (dtype) *dtype = t->dtype;
    if (rank) *rank = t->rank;
    if (shape)
        for (int i = 0; i < t->rank; i++) shape[i] = t->shape[i];
    if (data) *data = f->data + t->begin;
    if (nbytes) *nbytes = (int64_t)(t->end - t->begin);
    return QGMOE_OK;
}

int qgmoe_file_layer_desc(const qgmoe_file_t *f, const char *prefix, int32_t top_k,
                          int32_t router_mode, int32_t device, qgmoe_desc *d) {
    if (!f || !d) return set_error(QGMOE_ERR_INVALID_ARG, "null file/desc");
    const std::string pre = prefix ? prefix : "";
    // router: float rows (gate.weight, F32 or BF16) or a quantised linear
    // (gate.qweight / gate.scale: routerQuant, model/load.go:651-652)
    LinStack rq;
    const auto *router = find(f, pre + "gate.weight");
    const bool router_quant = find(f, pre + "gate.qweight") != nullptr;
    int64_t E = 0, H = 0;
    int rc = 0;
    if (router_quant) {
        if ((rc = lin_stack(f, pre + "gate", 2, rq))) return rc;
        E = rq.O;
        H = rq.K;
    } else {
        if (!router)
            return set_error(QGMOE_ERR_INVALID_ARG, "%sgate.weight not in the file", pre.c_str());
        if ((router->dtype != QGMOE_DT_F32 && router->dtype != QGMOE_DT_BF16) || router->rank != 2)
            return set_error(QGMOE_ERR_INVALID_ARG, "%sgate.weight: F32 or BF16 [E, H] expected",
                             pre.c_str());
        E = router->shape[0];
        H = router->shape[1];
    }
    LinStack gu, dn;
    rc = lin_stack(f, pre + "experts.gate_up_proj", 3, gu);
    if (!rc) rc = lin_stack(f, pre + "experts.down_proj", 3, dn);
    if (rc) return rc;
    const int64_t I = gu.O / 2;
    if (gu.lead != E || gu.O % 2 || gu.K != H || dn.lead != E || dn.O != H || dn.K != I)
        return set_error(QGMOE_ERR_INVALID_ARG,
                         "expert stacks [%lld, %lld, %lld] / [%lld, %lld, %lld] do not fit E=%lld "
                         "H=%lld", (long long)gu.lead, (long long)gu.O, (long long)gu.K,
                         (long long)dn.lead, (long long)dn.O, (long long)dn.K, (long long)E,
                         (long long)H);
    if (gu.bits != dn.bits || gu.sdt != dn.sdt)
        return set_error(QGMOE_ERR_INVALID_ARG, "expert stacks differ in format or scale dtype");
    const bool has_shared = find(f, pre + "shared_expert.gate_proj.qweight") ||
                            find(f, pre + "shared_expert.up_proj.qweight") ||
                            find(f, pre + "shared_expert.down_proj.qweight") ||
                            find(f, pre + "shared_expert.gate_proj.weight") ||
                            find(f, pre + "shared_expert.up_proj.weight") ||
                            find(f, pre + "shared_expert.down_proj.weight");
    LinStack sg, su, sd;
    int64_t Is = 0;
    const float *gate_vec = nullptr;
    if (has_shared) {
        rc = lin_stack(f, pre + "shared_expert.gate_proj", 2, sg);
        if (!rc) rc = lin_stack(f, pre + "shared_expert.up_proj", 2, su);
        if (!rc) rc = lin_stack(f, pre + "shared_expert.down_proj", 2, sd);
        if (rc) return rc;
        Is = sg.O;
        if (sg.K != H || su.O != Is || su.K != H || sd.O != H || sd.K != Is)
            return set_error(QGMOE_ERR_INVALID_ARG, "shared expert shapes do not fit H=%lld",
                             (long long)H);
        if (su.bits != sg.bits || sd.bits != sg.bits || su.sdt != sg.sdt || sd.sdt != sg.sdt)
            return set_error(QGMOE_ERR_INVALID_ARG,
                             "shared expert projections differ in format or scale dtype");
        const std::string gname = pre + "shared_expert_gate.weight";
        const auto *gate = find(f, gname);
        if (!gate || (gate->dtype != QGMOE_DT_F32 && gate->dtype != QGMOE_DT_BF16) ||
            (gate->rank == 1 ? gate->shape[0] != H
                             : (gate->rank != 2 || gate->shape[0] != 1 || gate->shape[1] != H)))
            return set_error(QGMOE_ERR_INVALID_ARG,
                             "%s: F32 or BF16 [1, H] expected", gname.c_str());
        gate_vec = f32_view(f, gname, gate);
    }
    // one scale dtype for every quantised group of the layer
    int sdt = -1;
    for (int g : {gu.sdt, has_shared ? sg.sdt : -1, router_quant ? rq.sdt : -1}) {
        if (g < 0) continue;
        if (sdt >= 0 && g != sdt)
            return set_error(QGMOE_ERR_INVALID_ARG,
                             "the layer's quantised groups mix F16 and F32 scales");
        sdt = g;
    }
    if (E > INT32_MAX || H > INT32_MAX || I > INT32_MAX || Is > INT32_MAX)
        return set_error(QGMOE_ERR_INVALID_ARG, "dimensions beyond int32");
    memset(d, 0, sizeof(*d));
    d->n_embed = (int32_t)H;
    d->n_experts = (int32_t)E;
    d->top_k = top_k;
    d->n_moe_mlp = (int32_t)I;
    d->n_shared_mlp = (int32_t)Is;
    d->bits = gu.bits;
    d->shared_bits = has_shared ? sg.bits : 0;
    d->router_mode = router_mode;
    d->scale_dtype = sdt >= 0 ? sdt : QGMOE_SCALE_F16;
    d->weights_on_device = 0;
    d->device = device;
    if (router_quant) {
        d->router_bits = rq.bits;
        d->router_q = rq.w;
        d->router_scale = rq.s;
    } else {
        d->router = f32_view(f, pre + "gate.weight", router);
    }
    d->shared_gate = gate_vec;
    auto put = [&](const LinStack &l, const float **w32, const uint8_t **q, const void **sc) {
        if (l.bits == 32) {
            *w32 = static_cast<const float *>(l.w);
        } else {
            *q = static_cast<const uint8_t *>(l.w);  // codes, or bf16 bit patterns (bits 16)
            *sc = l.s;
        }
    };
    put(gu, &d->gate_up, &d->gate_up_q, &d->gate_up_scale);
    put(dn, &d->down, &d->down_q, &d->down_scale);
    if (has_shared) {
        put(sg, &d->shared_gate_proj, &d->shared_gate_q, &d->shared_gate_scale);
        put(su, &d->shared_up_proj, &d->shared_up_q, &d->shared_up_scale);
        put(sd, &d->shared_down_proj, &d->shared_down_q, &d->shared_down_scale);
    }
    return QGMOE_OK;
}

}  // extern "C"
