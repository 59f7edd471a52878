// obs_safetensors.cu -- the per-layer expert files of the reference's splitter
// into the context's HBM store.
//
// tools/split_experts.py:63-75 writes one safetensors file per layer,
// layer_{il}_experts.safetensors, holding for every expert e and projection p in
// {gate_proj, up_proj, down_proj} the tensors e{e}.{p}.weight (U32 [out, in/8],
// packed 4-bit codes), e{e}.{p}.scales and e{e}.{p}.biases (F16 [out, in/64];
// cast from the checkpoint's bf16).  The reference indexes these names in
// ExpertIndex::open (src/disk_io.rs:36-63: exactly three dot-separated parts, the
// expert id after the leading 'e') and preads the routed experts per token.  Here
// a layer is read once, its tensors are stacked into the [E, out, ...] arrays
// obs_load_layer takes, scales and biases are rounded to bf16 (exactly: every f16
// value the splitter writes came from a bf16 value), and the layer is re-tiled
// into HBM by the ordinary loader.  The router gate (mlp.gate.*) is not in these
// files (it is a non-expert tensor, src/weight_loader.rs:19-71) and is passed in.
//
// The safetensors format: an 8-byte little-endian header length N, N bytes of
// JSON {"name": {"dtype": "...", "shape": [...], "data_offsets": [begin, end]},
// ..., "__metadata__": {...}}, then the data; offsets are relative to the data.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/obs_moe.h"

namespace obs {
void set_thread_error(const char* msg);
// the context's shape and its error message (obs_api.cu)
void ctx_shape(const obs_ctx* ctx, int* E, int* H, int* I);
int ctx_fail(obs_ctx* ctx, int code, const char* msg);
}  // namespace obs

namespace {

// ------------------------------------------------------ a small JSON reader
struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* end;
    std::string err;
    int depth = 0;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool string(std::string& out) {
        if (p >= end || *p != '"') return fail("expected a string");
        ++p;
        while (p < end && *p != '"') {
            if (*p == '\\') {
                if (++p >= end) return fail("bad escape");
                switch (*p) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u':  // names here are ASCII; keep the code point's low byte
                        if (end - p < 5) return fail("bad \\u escape");
                        out += (char)strtol(std::string(p + 1, p + 5).c_str(), nullptr, 16);
                        p += 4;
                        break;
                    default: return fail("bad escape");
                }
                ++p;
            } else {
                out += *p++;
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JVal& v) {
        if (++depth > 16) return fail("JSON nested too deeply");
        ws();
        if (p >= end) return fail("unexpected end of header");
        bool ok = true;
        if (*p == '{') {
            v.kind = JVal::Obj;
            ++p;
            ws();
            if (p < end && *p == '}') {
                ++p;
            } else {
                for (;;) {
                    ws();
                    std::string k;
                    JVal x;
                    if (!string(k)) { ok = false; break; }
                    ws();
                    if (p >= end || *p != ':') { ok = fail("expected ':'"); break; }
                    ++p;
                    if (!value(x)) { ok = false; break; }
                    v.obj.emplace_back(std::move(k), std::move(x));
                    ws();
                    if (p < end && *p == ',') { ++p; continue; }
                    if (p < end && *p == '}') { ++p; break; }
                    ok = fail("expected ',' or '}'");
                    break;
                }
            }
        } else if (*p == '[') {
            v.kind = JVal::Arr;
            ++p;
            ws();
            if (p < end && *p == ']') {
                ++p;
            } else {
                for (;;) {
                    JVal x;
                    if (!value(x)) { ok = false; break; }
                    v.arr.push_back(std::move(x));
                    ws();
                    if (p < end && *p == ',') { ++p; continue; }
                    if (p < end && *p == ']') { ++p; break; }
                    ok = fail("expected ',' or ']'");
                    break;
                }
            }
        } else if (*p == '"') {
            v.kind = JVal::Str;
            ok = string(v.str);
        } else if (*p == '-' || (*p >= '0' && *p <= '9')) {
            v.kind = JVal::Num;
            char* e = nullptr;
            v.num = strtod(std::string(p, end - p < 64 ? end - p : 64).c_str(), &e);
            const char* q = p;
            while (q < end && (*q == '-' || *q == '+' || *q == '.' || *q == 'e' || *q == 'E' || (*q >= '0' && *q <= '9')))
                ++q;
            p = q;
        } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
            v.kind = JVal::Bool, v.b = true, p += 4;
        } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
            v.kind = JVal::Bool, p += 5;
        } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
            p += 4;
        } else {
            ok = fail("unexpected character in header");
        }
        --depth;
        return ok;
    }
};

// ------------------------------------------------------------ the file
struct Tensor {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

struct ExpertFile {
    std::vector<uint8_t> bytes;  // the whole file
    uint64_t data0 = 0;          // start of the data section
    std::map<std::string, Tensor> tensors;
    int E = 0, H = 0, I = 0;
    std::string err;

    bool fail(const std::string& m) {
        err = m;
        return false;
    }

    bool read(const char* path, bool header_only) {
        FILE* f = fopen(path, "rb");
        if (!f) return fail(std::string("cannot open ") + path);
        uint8_t lenb[8];
        if (fread(lenb, 1, 8, f) != 8) {
            fclose(f);
            return fail("file shorter than the 8-byte header length");
        }
        uint64_t n = 0;
        for (int i = 7; i >= 0; --i) n = (n << 8) | lenb[i];
        if (n == 0 || n > (100ull << 20)) {
            fclose(f);
            return fail("implausible safetensors header length");
        }
        fseek(f, 0, SEEK_END);
        const long long size = ftell(f);
        if (size < (long long)(8 + n)) {
            fclose(f);
            return fail("file shorter than its header");
        }
        const size_t want = header_only ? (size_t)(8 + n) : (size_t)size;
        bytes.resize(want);
        fseek(f, 0, SEEK_SET);
        const size_t got = fread(bytes.data(), 1, want, f);
        fclose(f);
        if (got != want) return fail("short read");
        data0 = 8 + n;
        JParser jp{reinterpret_cast<const char*>(bytes.data()) + 8, reinterpret_cast<const char*>(bytes.data()) + 8 + n};
        JVal root;
        if (!jp.value(root) || root.kind != JVal::Obj) return fail("bad safetensors header: " + jp.err);
        const uint64_t data_size = (uint64_t)size - data0;
        for (const auto& kv : root.obj) {
            if (kv.first == "__metadata__") continue;
            const JVal& t = kv.second;
            const JVal *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
            if (!dt || dt->kind != JVal::Str || !sh || sh->kind != JVal::Arr || !off || off->kind != JVal::Arr ||
                off->arr.size() != 2)
                return fail("tensor entry without dtype, shape or data_offsets: " + kv.first);
            Tensor x;
            x.dtype = dt->str;
            for (const auto& d : sh->arr) x.shape.push_back((int64_t)d.num);
            x.begin = (uint64_t)off->arr[0].num, x.end = (uint64_t)off->arr[1].num;
            if (x.end < x.begin || x.end > data_size) return fail("data_offsets outside the file: " + kv.first);
            tensors[kv.first] = x;
        }
        return index();
    }

    // shapes of the e{N}.{proj}.{kind} tensors: E experts, H, I consistent throughout
    bool index() {
        int max_e = -1;
        for (const auto& kv : tensors) {
            const std::string& name = kv.first;
            const size_t d1 = name.find('.'), d2 = name.find('.', d1 == std::string::npos ? 0 : d1 + 1);
            if (name.size() < 2 || name[0] != 'e' || d1 == std::string::npos || d2 == std::string::npos ||
                name.find('.', d2 + 1) != std::string::npos)
                continue;  // not an expert tensor (disk_io.rs:45-47 skips these too)
            int e = 0;
            for (size_t i = 1; i < d1; ++i) {
                if (name[i] < '0' || name[i] > '9') return fail("bad expert id in " + name);
                e = e * 10 + (name[i] - '0');
            }
            if (e > max_e) max_e = e;
        }
        if (max_e < 0) return fail("no e{N}.{proj}.{kind} tensors in the file");
        E = max_e + 1;
        const Tensor* g = find(0, "gate_proj", "weight");
        const Tensor* d = find(0, "down_proj", "weight");
        if (!g || !d || g->shape.size() != 2 || d->shape.size() != 2) return fail("expert 0 lacks 2-D gate/down weights");
        I = (int)g->shape[0], H = (int)g->shape[1] * 8;
        if (d->shape[0] != H || d->shape[1] * 8 != I) return fail("gate_proj and down_proj shapes disagree");
        for (int e = 0; e < E; ++e)
            for (const char* p : {"gate_proj", "up_proj", "down_proj"}) {
                const int out_f = strcmp(p, "down_proj") ? I : H, in_f = strcmp(p, "down_proj") ? H : I;
                const Tensor* w = find(e, p, "weight");
                const Tensor* s = find(e, p, "scales");
                const Tensor* b = find(e, p, "biases");
                const std::string nm = "e" + std::to_string(e) + "." + p;
                if (!w || !s || !b) return fail("missing tensor of " + nm);
                if (w->dtype != "U32" && w->dtype != "I32") return fail(nm + ".weight is not U32");
                if (w->shape != std::vector<int64_t>{out_f, in_f / 8}) return fail(nm + ".weight has the wrong shape");
                for (const Tensor* q : {s, b}) {
                    if (q->dtype != "F16" && q->dtype != "BF16") return fail(nm + " scales/biases are not F16 or BF16");
                    if (q->shape != std::vector<int64_t>{out_f, in_f / 64}) return fail(nm + " scales/biases have the wrong shape");
                }
                if (w->end - w->begin != (uint64_t)out_f * in_f / 2 || s->end - s->begin != (uint64_t)out_f * (in_f / 64) * 2 ||
                    b->end - b->begin != (uint64_t)out_f * (in_f / 64) * 2)
                    return fail(nm + ": data size does not match the shape");
            }
        return true;
    }

    const Tensor* find(int e, const char* proj, const char* kind) const {
        auto it = tensors.find("e" + std::to_string(e) + "." + proj + "." + kind);
        return it == tensors.end() ? nullptr : &it->second;
    }
    const uint8_t* data(const Tensor* t) const { return bytes.data() + data0 + t->begin; }
};

// f16 -> bf16, round to nearest even (exact for every f16 that came from a bf16)
uint16_t f16_to_bf16(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1F, man = h & 0x3FF;
    uint32_t f;
    if (ex == 0x1F) {
        f = sign | 0x7F800000u | (man << 13);  // inf / NaN
    } else if (ex == 0) {
        if (man == 0) {
            f = sign;
        } else {  // subnormal: normalise
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while (!(man & 0x400u));
            f = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else {
        f = sign | ((ex + 127 - 15) << 23) | (man << 13);
    }
    if ((f & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((f >> 16) | 0x40u);
    f += 0x7FFFu + ((f >> 16) & 1u);
    return (uint16_t)(f >> 16);
}

int fail_thread(int code, const std::string& m) {
    obs::set_thread_error(m.c_str());
    return code;
}

}  // namespace

extern "C" int obs_expert_file_info(const char* path, int32_t* n_experts, int32_t* hidden, int32_t* inter) {
    if (!path) return fail_thread(OBS_ERR_INVALID, "null path");
    ExpertFile f;
    if (!f.read(path, true)) return fail_thread(OBS_ERR_INVALID, f.err);
    if (n_experts) *n_experts = f.E;
    if (hidden) *hidden = f.H;
    if (inter) *inter = f.I;
    return OBS_OK;
}

extern "C" int obs_load_layer_safetensors(obs_ctx* ctx, int layer, const char* path, const uint32_t* router_w,
                                          const uint16_t* router_s, const uint16_t* router_b) {
    if (!ctx) return OBS_ERR_INVALID;
    if (!path || !router_w || !router_s || !router_b) return obs::ctx_fail(ctx, OBS_ERR_INVALID, "null argument");
    ExpertFile f;
    if (!f.read(path, false)) return obs::ctx_fail(ctx, OBS_ERR_INVALID, f.err.c_str());
    int E = 0, H = 0, I = 0;
    obs::ctx_shape(ctx, &E, &H, &I);
    if (E != f.E || H != f.H || I != f.I) {
        char m[160];
        snprintf(m, sizeof m, "expert file shape (E=%d, H=%d, I=%d) differs from the context's (E=%d, H=%d, I=%d)", f.E,
                 f.H, f.I, E, H, I);
        return obs::ctx_fail(ctx, OBS_ERR_INVALID, m);
    }
    // stack the per-expert tensors into the [E, out, ...] arrays obs_load_layer takes
    std::vector<uint32_t> w[3];
    std::vector<uint16_t> s[3], b[3];
    const char* projs[3] = {"gate_proj", "up_proj", "down_proj"};
    for (int p = 0; p < 3; ++p) {
        const int out_f = p == 2 ? f.H : f.I, in_f = p == 2 ? f.I : f.H;
        const size_t nw = (size_t)out_f * in_f / 8, ng = (size_t)out_f * (in_f / 64);
        w[p].resize(nw * f.E), s[p].resize(ng * f.E), b[p].resize(ng * f.E);
        for (int e = 0; e < f.E; ++e) {
            const Tensor* tw = f.find(e, projs[p], "weight");
            const Tensor* ts = f.find(e, projs[p], "scales");
            const Tensor* tb = f.find(e, projs[p], "biases");
            memcpy(w[p].data() + nw * e, f.data(tw), nw * 4);
            const uint16_t* ps = reinterpret_cast<const uint16_t*>(f.data(ts));
            const uint16_t* pb = reinterpret_cast<const uint16_t*>(f.data(tb));
            for (size_t i = 0; i < ng; ++i) {
                s[p][ng * e + i] = ts->dtype == "F16" ? f16_to_bf16(ps[i]) : ps[i];
                b[p][ng * e + i] = tb->dtype == "F16" ? f16_to_bf16(pb[i]) : pb[i];
            }
        }
    }
    obs_layer_weights lw{router_w, router_s, router_b, w[0].data(), s[0].data(), b[0].data(),
                         w[1].data(), s[1].data(), b[1].data(), w[2].data(), s[2].data(), b[2].data()};
    return obs_load_layer(ctx, layer, &lw, 0);
}
