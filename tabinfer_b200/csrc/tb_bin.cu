// tb_bin.cu -- the `.cpu.bin` ternary model container loaded onto the device.
//
// Format (native/docs/FORMAT.md:10-45): u32 le header_len, header_len bytes of
// UTF-8 JSON {"G": 64, "tensors": {name: {kind, ...}}}, then the blob; every
// offset in the header is blob-relative and every entry 16-byte aligned.  Kinds:
// `tern` (N, K, codesOff/Len, scalesOff/Len: Q2_0_g64 codes u8 [N][K/4] and
// f32 scales [N][K/64]), `embed_f16` and `f32` (shape, off, len).
//
// The checks are the reference reader's (Container::assemble / validate,
// native/crates/n2-core/src/binfmt.rs:155-257): G must equal the kernels' 64
// (absent means 64), K % G == 0, codesLen == N*K/4, scalesLen == N*(K/G)*4,
// known kinds only, every range inside the blob, header inside the file.
//
// B200 design: the blob is streamed from the file through two pinned staging
// buffers into ONE device allocation (copies on the context's stream overlap
// the next read), so every tensor is a device pointer `blob + off` already in
// the layout the Q2_0_g64 GEMV, the embedding gather and the norms read --
// no repacking.
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <vector>

#include "tb_common.cuh"

namespace {

// ---- a small JSON reader (objects, arrays, strings, numbers, literals) -------
struct JVal {
    enum Type { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
    double num = 0.0;
    bool integral = false;
    long long ival = 0;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal* get(const char* k) const
    {
        if (t != OBJ) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* end;
    std::string err;
    void ws()
    {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool fail(const char* m)
    {
        if (err.empty()) err = m;
        return false;
    }
    bool string(std::string& out)
    {
        if (p >= end || *p != '"') return fail("expected a string");
        p++;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c != '\\') { out.push_back(c); continue; }
            if (p >= end) return fail("unterminated escape");
            char e = *p++;
            switch (e) {
            case '"': out.push_back('"'); break;
            case '\\': out.push_back('\\'); break;
            case '/': out.push_back('/'); break;
            case 'b': out.push_back('\b'); break;
            case 'f': out.push_back('\f'); break;
            case 'n': out.push_back('\n'); break;
            case 'r': out.push_back('\r'); break;
            case 't': out.push_back('\t'); break;
            case 'u': {
                if (end - p < 4) return fail("short \\u escape");
                unsigned cp = 0;
                for (int i = 0; i < 4; i++) {
                    char h = *p++;
                    cp <<= 4;
                    if (h >= '0' && h <= '9') cp |= h - '0';
                    else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
                    else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
                    else return fail("bad \\u escape");
                }
                if (cp < 0x80) out.push_back((char)cp);
                else if (cp < 0x800) { out.push_back((char)(0xC0 | (cp >> 6))); out.push_back((char)(0x80 | (cp & 0x3F))); }
                else {
                    out.push_back((char)(0xE0 | (cp >> 12)));
                    out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
                    out.push_back((char)(0x80 | (cp & 0x3F)));
                }
                break;
            }
            default: return fail("bad escape");
            }
        }
        if (p >= end) return fail("unterminated string");
        p++;
        return true;
    }
    bool value(JVal& v, int depth)
    {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end of JSON");
        if (*p == '{') {
            v.t = JVal::OBJ;
            p++;
            ws();
            if (p < end && *p == '}') { p++; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (p >= end || *p != ':') return fail("expected ':'");
                p++;
                JVal child;
                if (!value(child, depth + 1)) return false;
                v.obj.emplace_back(std::move(k), std::move(child));
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == '}') { p++; return true; }
                return fail("expected ',' or '}'");
            }
        }
        if (*p == '[') {
            v.t = JVal::ARR;
            p++;
            ws();
            if (p < end && *p == ']') { p++; return true; }
            for (;;) {
                JVal child;
                if (!value(child, depth + 1)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == ']') { p++; return true; }
                return fail("expected ',' or ']'");
            }
        }
        if (*p == '"') { v.t = JVal::STR; return string(v.str); }
        if (end - p >= 4 && !strncmp(p, "true", 4)) { v.t = JVal::BOOL; v.num = 1; p += 4; return true; }
        if (end - p >= 5 && !strncmp(p, "false", 5)) { v.t = JVal::BOOL; p += 5; return true; }
        if (end - p >= 4 && !strncmp(p, "null", 4)) { v.t = JVal::NUL; p += 4; return true; }
        // number
        const char* s = p;
        bool frac = false;
        if (p < end && (*p == '-' || *p == '+')) p++;
        while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) {
            if (*p == '.' || *p == 'e' || *p == 'E') frac = true;
            p++;
        }
        if (p == s) return fail("unexpected character");
        std::string tok(s, p);
        char* e2 = nullptr;
        v.t = JVal::NUM;
        v.num = strtod(tok.c_str(), &e2);
        if (!e2 || *e2) return fail("bad number");
        if (!frac) {
            v.integral = true;
            v.ival = strtoll(tok.c_str(), nullptr, 10);
        }
        return true;
    }
};

// ---- the container ----------------------------------------------------------
struct TensorRec {
    int kind = 0;                 // TB_BIN_*
    int64_t N = 0, K = 0;
    std::vector<int64_t> shape;
    int64_t off = 0, len = 0;     // codes (tern) or data
    int64_t soff = 0, slen = 0;   // scales (tern)
};

// Non-negative integer field, with the reference's messages ("missing field",
// "not a non-negative integer").
bool usize_field(const JVal& t, const char* k, int64_t& out, std::string& err)
{
    const JVal* v = t.get(k);
    if (!v) { err = std::string("missing field `") + k + "`"; return false; }
    if (v->t != JVal::NUM || !v->integral || v->ival < 0) {
        err = std::string("field `") + k + "` is not a non-negative integer";
        return false;
    }
    out = v->ival;
    return true;
}

bool usize_array(const JVal& t, const char* k, std::vector<int64_t>& out, std::string& err)
{
    const JVal* v = t.get(k);
    if (!v) { err = std::string("missing field `") + k + "`"; return false; }
    if (v->t != JVal::ARR) { err = std::string("field `") + k + "` is not an array"; return false; }
    for (const auto& e : v->arr) {
        if (e.t != JVal::NUM || !e.integral || e.ival < 0) {
            err = std::string("field `") + k + "` holds a non-integer";
            return false;
        }
        out.push_back(e.ival);
    }
    return true;
}

constexpr int64_t KERNEL_G = 64;

// Container::assemble + validate (binfmt.rs:155-257) on a header and a blob length.
bool parse_header(const char* hdr, size_t n, int64_t blob_len, int64_t& G,
                  std::map<std::string, TensorRec>& out, std::string& err)
{
    JParser jp{hdr, hdr + n, {}};
    JVal root;
    if (!jp.value(root, 0)) { err = "header JSON: " + jp.err; return false; }
    jp.ws();
    if (jp.p != jp.end) { err = "header JSON: trailing characters"; return false; }
    if (root.t != JVal::OBJ) { err = "header JSON: not an object"; return false; }
    G = KERNEL_G;
    if (const JVal* g = root.get("G")) {
        if (g->t != JVal::NUM || !g->integral || g->ival < 0) { err = "header field `G` is not an integer"; return false; }
        G = g->ival;
    }
    if (G != KERNEL_G) {
        char b[160];
        snprintf(b, sizeof b, "container group size G=%lld but the kernels are built for G=%lld", (long long)G,
                 (long long)KERNEL_G);
        err = b;
        return false;
    }
    const JVal* tensors = root.get("tensors");
    if (!tensors || tensors->t != JVal::OBJ) { err = "header has no `tensors` object"; return false; }
    for (const auto& kv : tensors->obj) {
        const std::string& name = kv.first;
        const JVal& t = kv.second;
        const JVal* kind = t.get("kind");
        if (!kind || kind->t != JVal::STR) { err = name + ": missing `kind`"; return false; }
        TensorRec r;
        std::string e;
        char b[256];
        if (kind->str == "tern") {
            r.kind = TB_BIN_TERN;
            if (!usize_field(t, "N", r.N, e) || !usize_field(t, "K", r.K, e)) { err = name + ": " + e; return false; }
            if (r.N > (1LL << 31) || r.K > (1LL << 31)) { err = name + ": shape too large"; return false; }
            if (r.K % G != 0) {
                snprintf(b, sizeof b, ": K=%lld is not a multiple of G=%lld", (long long)r.K, (long long)G);
                err = name + b;
                return false;
            }
            if (!usize_field(t, "codesLen", r.len, e) || !usize_field(t, "scalesLen", r.slen, e)) {
                err = name + ": " + e;
                return false;
            }
            const int64_t want_codes = r.N * r.K / 4, want_scales = r.N * (r.K / G) * 4;
            if (r.len != want_codes) {
                snprintf(b, sizeof b, ": codesLen=%lld but N*K/4=%lld", (long long)r.len, (long long)want_codes);
                err = name + b;
                return false;
            }
            if (r.slen != want_scales) {
                snprintf(b, sizeof b, ": scalesLen=%lld but N*(K/G)*4=%lld", (long long)r.slen, (long long)want_scales);
                err = name + b;
                return false;
            }
            if (!usize_field(t, "codesOff", r.off, e) || !usize_field(t, "scalesOff", r.soff, e)) {
                err = name + ": " + e;
                return false;
            }
            r.shape = {r.N, r.K};
        } else if (kind->str == "embed_f16" || kind->str == "f32") {
            r.kind = kind->str == "f32" ? TB_BIN_F32 : TB_BIN_EMBED_F16;
            if (!usize_array(t, "shape", r.shape, e) || !usize_field(t, "off", r.off, e) ||
                !usize_field(t, "len", r.len, e)) {
                err = name + ": " + e;
                return false;
            }
        } else {
            err = name + ": unknown kind `" + kind->str + "`";
            return false;
        }
        out[name] = std::move(r);
    }
    // every declared byte range must lie inside the blob (validate, binfmt.rs:234-257)
    for (const auto& kv : out) {
        const TensorRec& r = kv.second;
        const int64_t offs[2] = {r.off, r.soff}, lens[2] = {r.len, r.slen};
        for (int i = 0; i < (r.kind == TB_BIN_TERN ? 2 : 1); i++) {
            if (offs[i] > blob_len || lens[i] > blob_len - offs[i]) {
                char b[200];
                snprintf(b, sizeof b, ": range %lld..%lld overruns the %lld-byte blob", (long long)offs[i],
                         (long long)(offs[i] + lens[i]), (long long)blob_len);
                err = kv.first + b;
                return false;
            }
        }
    }
    return true;
}

struct FileCloser {
    void operator()(FILE* f) const { if (f) fclose(f); }
};

// header of a file: header bytes and blob length (Container::open, binfmt.rs:104-131)
bool read_header(const char* path, FILE*& fout, std::string& hdr, int64_t& blob_len, std::string& err)
{
    FILE* f = fopen(path, "rb");
    if (!f) { err = std::string(path) + ": cannot open"; return false; }
    std::unique_ptr<FILE, FileCloser> guard(f);
    if (fseeko(f, 0, SEEK_END) != 0) { err = std::string(path) + ": cannot seek"; return false; }
    const int64_t total = (int64_t)ftello(f);
    fseeko(f, 0, SEEK_SET);
    unsigned char lb[4];
    if (total < 4 || fread(lb, 1, 4, f) != 4) { err = "file is too short to contain a header length"; return false; }
    const int64_t hl = (int64_t)lb[0] | ((int64_t)lb[1] << 8) | ((int64_t)lb[2] << 16) | ((int64_t)lb[3] << 24);
    if (4 + hl > total) {
        char b[160];
        snprintf(b, sizeof b, "header length %lld overruns the file (%lld bytes)", (long long)hl, (long long)total);
        err = b;
        return false;
    }
    hdr.resize((size_t)hl);
    if (hl && fread(&hdr[0], 1, (size_t)hl, f) != (size_t)hl) { err = std::string(path) + ": short read"; return false; }
    blob_len = total - 4 - hl;
    fout = guard.release();
    return true;
}

}  // namespace

struct tb_bin {
    tb_ctx* ctx = nullptr;
    int64_t G = KERNEL_G;
    int64_t blob_len = 0;
    unsigned char* blob = nullptr;            // device
    std::map<std::string, TensorRec> tensors; // sorted by name (the reference's BTreeMap order)
    std::vector<const std::string*> order;
};

namespace {

int fill_info(const tb_bin* b, const std::string& name, const TensorRec& r, tb_bin_tensor* info)
{
    memset(info, 0, sizeof *info);
    info->name = name.c_str();
    info->kind = r.kind;
    info->N = r.N;
    info->K = r.K;
    info->ndim = (int)std::min<size_t>(r.shape.size(), 4);
    for (int i = 0; i < info->ndim; i++) info->shape[i] = r.shape[i];
    info->data = b->blob + r.off;
    info->bytes = r.len;
    if (r.kind == TB_BIN_TERN) {
        info->scales = b->blob + r.soff;
        info->scales_bytes = r.slen;
    }
    info->blob_offset = r.off;
    return TB_OK;
}

// stream `n` bytes of f (at its current position) into device memory dst
int upload_stream(tb_ctx* ctx, FILE* f, unsigned char* dst, int64_t n)
{
    constexpr size_t CHUNK = 32u << 20;
    void* pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    int rc = TB_OK;
    for (int i = 0; i < 2 && rc == TB_OK; i++) {
        if (cudaHostAlloc(&pin[i], CHUNK, cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess)
            rc = tb_fail(ctx, TB_ERR_NOMEM, "bin: pinned staging allocation failed");
    }
    int64_t done = 0;
    for (int it = 0; rc == TB_OK && done < n; it++) {
        const int s = it & 1;
        const size_t m = (size_t)std::min<int64_t>((int64_t)CHUNK, n - done);
        if (it >= 2) cudaEventSynchronize(ev[s]);   // the copy that last used this buffer has finished
        if (fread(pin[s], 1, m, f) != m) { rc = tb_fail(ctx, TB_ERR_INVALID, "bin: short read of the blob"); break; }
        cudaError_t e = cudaMemcpyAsync(dst + done, pin[s], m, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaEventRecord(ev[s], ctx->stream);
        if (e != cudaSuccess) { rc = tb_fail(ctx, TB_ERR_CUDA, "bin: blob copy: %s", cudaGetErrorString(e)); break; }
        done += (int64_t)m;
    }
    cudaStreamSynchronize(ctx->stream);   // staging buffers are freed below
    for (int i = 0; i < 2; i++) {
        if (ev[i]) cudaEventDestroy(ev[i]);
        if (pin[i]) cudaFreeHost(pin[i]);
    }
    return rc;
}

}  // namespace

extern "C" {

TB_API int tb_bin_check(const char* path, char* err, size_t err_len)
{
    auto put = [&](const std::string& m) {
        if (err && err_len) { strncpy(err, m.c_str(), err_len - 1); err[err_len - 1] = 0; }
    };
    if (!path) { put("null path"); return TB_ERR_INVALID; }
    FILE* f = nullptr;
    std::string hdr, e;
    int64_t blob_len = 0, G = 0;
    if (!read_header(path, f, hdr, blob_len, e)) { put(e); return TB_ERR_INVALID; }
    fclose(f);
    std::map<std::string, TensorRec> t;
    if (!parse_header(hdr.data(), hdr.size(), blob_len, G, t, e)) { put(e); return TB_ERR_INVALID; }
    put("");
    return TB_OK;
}

TB_API int tb_bin_open(tb_ctx* ctx, const char* path, tb_bin** out)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, path && out, "null pointer");
    *out = nullptr;
    FILE* f = nullptr;
    std::string hdr, e;
    int64_t blob_len = 0;
    if (!read_header(path, f, hdr, blob_len, e)) return tb_fail(ctx, TB_ERR_INVALID, "%s", e.c_str());
    std::unique_ptr<FILE, FileCloser> guard(f);
    std::unique_ptr<tb_bin> b(new tb_bin);
    b->ctx = ctx;
    b->blob_len = blob_len;
    if (!parse_header(hdr.data(), hdr.size(), blob_len, b->G, b->tensors, e))
        return tb_fail(ctx, TB_ERR_INVALID, "%s", e.c_str());
    cudaError_t ce = cudaSetDevice(ctx->device);
    if (ce == cudaSuccess) ce = cudaMalloc(&b->blob, (size_t)std::max<int64_t>(blob_len, 256));
    if (ce != cudaSuccess) {
        cudaGetLastError();
        return tb_fail(ctx, TB_ERR_NOMEM, "bin: cudaMalloc of the %lld-byte blob failed", (long long)blob_len);
    }
    int rc = upload_stream(ctx, f, b->blob, blob_len);
    if (rc) { cudaFree(b->blob); return rc; }
    for (const auto& kv : b->tensors) b->order.push_back(&kv.first);
    *out = b.release();
    return TB_OK;
}

TB_API int tb_bin_close(tb_bin* b)
{
    if (!b) return TB_OK;
    if (b->blob) cudaFree(b->blob);
    delete b;
    return TB_OK;
}

TB_API int64_t tb_bin_blob_bytes(const tb_bin* b) { return b ? b->blob_len : -1; }

TB_API int tb_bin_count(const tb_bin* b) { return b ? (int)b->order.size() : -1; }

TB_API int tb_bin_info(const tb_bin* b, int index, tb_bin_tensor* info)
{
    if (!b || !info) return TB_ERR_INVALID;
    TB_REQUIRE(b->ctx, index >= 0 && index < (int)b->order.size(), "bin: tensor index %d out of range", index);
    const std::string& name = *b->order[index];
    return fill_info(b, name, b->tensors.at(name), info);
}

TB_API int tb_bin_find(const tb_bin* b, const char* name, tb_bin_tensor* info)
{
    if (!b || !name || !info) return TB_ERR_INVALID;
    auto it = b->tensors.find(name);
    if (it == b->tensors.end()) return tb_fail(b->ctx, TB_ERR_INVALID, "%s: not in container", name);
    return fill_info(b, it->first, it->second, info);
}

}  // extern "C"
