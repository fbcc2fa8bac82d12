// `.gturbo` bundle loader (include/gtmoe_bundle.h): manifest and layout JSON, the resident
// index, and blocking file -> HBM loads through pinned staging buffers.
//
// Format (the reference's v1, restated here in this library's own code):
//   manifest.json               src/manifest.cpp:24-49 (validate), :157-240 (fields)
//   packed_experts/layout.json  src/packed_experts.cpp:15-58 (validate), :60-83 (cross-check),
//                               :115-166 (fields)
//   resident.bin index          src/resident_index.cpp:40-97; the converter's writer
//                               tools/convert_hf_to_gturbo.py:293-376 (names, 16 KB alignment)
//   tensor names                src/runner.cpp:319-353 ("model.layers.<L>.<suffix>")
#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <stdexcept>
#include <string>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

#include "gtm_internal.h"
#include "gtmoe_bundle.h"

namespace gtm {
namespace bundle {

struct FormatError : std::runtime_error {
    explicit FormatError(const std::string& m) : std::runtime_error(m) {}
};

// ---- a small JSON reader (objects, arrays, strings, numbers, true/false/null) -------------------
struct Json {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    bool integral = false;
    int64_t i = 0;
    double d = 0.0;
    std::string s;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* find(const char* key) const {
        if (kind != OBJ) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonReader {
public:
    JsonReader(const std::string& text, const std::string& what) : p_(text.data()), e_(text.data() + text.size()), what_(what) {}
    Json parse() {
        Json v = value(0);
        ws();
        if (p_ != e_) fail("trailing characters");
        return v;
    }

private:
    const char* p_;
    const char* e_;
    std::string what_;

    [[noreturn]] void fail(const char* why) { throw FormatError(what_ + ": malformed JSON (" + why + ")"); }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if ((size_t)(e_ - p_) >= n && memcmp(p_, w, n) == 0) { p_ += n; return true; }
        return false;
    }
    static void put_utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) out += (char)cp;
        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
        else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (e_ - p_ < 4) fail("short \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else fail("bad \\u escape");
        }
        return v;
    }
    std::string str() {
        if (p_ >= e_ || *p_ != '"') fail("expected a string");
        ++p_;
        std::string out;
        for (;;) {
            if (p_ >= e_) fail("unterminated string");
            const char c = *p_++;
            if (c == '"') break;
            if ((unsigned char)c < 0x20) fail("control character in string");
            if (c != '\\') { out += c; continue; }
            if (p_ >= e_) fail("unterminated escape");
            const char x = *p_++;
            switch (x) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    put_utf8(out, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
        return out;
    }
    Json number() {
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') ++p_;
        if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) fail("bad number");
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        bool integral = true;
        if (p_ < e_ && *p_ == '.') {
            integral = false;
            ++p_;
            if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) fail("bad fraction");
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            ++p_;
            if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= e_ || !(*p_ >= '0' && *p_ <= '9')) fail("bad exponent");
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        const std::string t(s, p_);
        Json v;
        v.kind = Json::NUM;
        v.d = strtod(t.c_str(), nullptr);
        v.integral = integral;
        if (integral) {
            errno = 0;
            v.i = strtoll(t.c_str(), nullptr, 10);
            if (errno == ERANGE) fail("integer out of range");
        } else {
            v.i = (int64_t)v.d;
        }
        return v;
    }
    Json value(int depth) {
        if (depth > 64) fail("nested too deeply");
        ws();
        if (p_ >= e_) fail("unexpected end");
        Json v;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = Json::OBJ;
            ws();
            if (p_ < e_ && *p_ == '}') { ++p_; return v; }
            for (;;) {
                ws();
                std::string k = str();
                ws();
                if (p_ >= e_ || *p_ != ':') fail("expected ':'");
                ++p_;
                v.obj.emplace_back(std::move(k), value(depth + 1));
                ws();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == '}') { ++p_; break; }
                fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            ++p_;
            v.kind = Json::ARR;
            ws();
            if (p_ < e_ && *p_ == ']') { ++p_; return v; }
            for (;;) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == ']') { ++p_; break; }
                fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = Json::STR;
            v.s = str();
        } else if (lit("true")) {
            v.kind = Json::BOOL; v.b = true;
        } else if (lit("false")) {
            v.kind = Json::BOOL; v.b = false;
        } else if (lit("null")) {
            v.kind = Json::NUL;
        } else {
            v = number();
        }
        return v;
    }
};

const Json& need(const Json& o, const char* key, const std::string& ctx) {
    const Json* v = o.find(key);
    if (!v) throw FormatError(ctx + ": missing '" + key + "'");
    return *v;
}
int64_t as_int(const Json& v, const std::string& ctx) {
    if (v.kind != Json::NUM || !v.integral) throw FormatError(ctx + ": expected an integer");
    return v.i;
}
int64_t int_or(const Json& o, const char* key, int64_t dflt, const std::string& ctx) {
    const Json* v = o.find(key);
    return v ? as_int(*v, ctx + "." + key) : dflt;
}
double num_or(const Json& o, const char* key, double dflt, const std::string& ctx) {
    const Json* v = o.find(key);
    if (!v) return dflt;
    if (v->kind != Json::NUM) throw FormatError(ctx + "." + key + ": expected a number");
    return v->d;
}
const std::string& as_str(const Json& v, const std::string& ctx) {
    if (v.kind != Json::STR) throw FormatError(ctx + ": expected a string");
    return v.s;
}

// ---- files ----------------------------------------------------------------------------------------
std::string read_text(const std::string& path) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) throw FormatError("cannot open " + path);
    std::string out;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out.append(buf, n);
    fclose(f);
    return out;
}

uint64_t file_size(const std::string& path) {
    struct stat st;
    if (stat(path.c_str(), &st) != 0 || !S_ISREG(st.st_mode)) throw FormatError("missing file " + path);
    return (uint64_t)st.st_size;
}

uint64_t add_checked(uint64_t a, uint64_t b, const std::string& what) {
    if (a + b < a) throw FormatError(what + ": arithmetic overflow");
    return a + b;
}

// src/format.hpp PathValidator: a plain file name, no separators, no "..", not empty
void check_basename(const std::string& s, const std::string& ctx) {
    if (s.empty() || s.find('/') != std::string::npos || s.find('\\') != std::string::npos ||
        s.find("..") != std::string::npos || s.find('\0') != std::string::npos)
        throw FormatError(ctx + ": expected a plain file name, got '" + s + "'");
}

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

constexpr uint64_t kAlign = 16384;               // GTurboFormatV1::ALIGNMENT_BYTES
constexpr uint64_t kIndexMax = 16ull << 20;      // RESIDENT_INDEX_MAX_BYTES
constexpr uint64_t kHeader = 24, kEntry = 72;    // RESIDENT_HEADER_BYTES, RESIDENT_ENTRY_BYTES
enum : uint8_t { DT_U32 = 0, DT_BF16 = 1, DT_FP16 = 2, DT_FP32 = 3 };

struct Entry {
    uint8_t dtype;
    uint64_t offset, size;
    uint32_t shape[4];
    uint64_t scale_offset, scale_size, bias_offset, bias_size;
};

struct Sub {
    uint64_t offset, size;
    uint8_t dtype;
};

// Staging kept for the bundle's lifetime (pinned allocations are slow): per reader thread two
// pinned chunk buffers, a stream and two events, created on the first load.
constexpr int kReaders = 4;
constexpr uint64_t kChunk = 16ull << 20;
struct Reader {
    cudaStream_t st = nullptr;
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
};
struct Stager {
    int device = -1;
    Reader r[kReaders];
    cudaError_t init(int dev) {
        if (device == dev) return cudaSuccess;
        release();
        cudaError_t e = cudaSuccess;
        for (int k = 0; k < kReaders && e == cudaSuccess; ++k) {
            e = cudaStreamCreateWithFlags(&r[k].st, cudaStreamNonBlocking);
            for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
                e = cudaHostAlloc(&r[k].stage[b], kChunk, cudaHostAllocDefault);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r[k].done[b], cudaEventDisableTiming);
            }
        }
        if (e != cudaSuccess) release();
        else device = dev;
        return e;
    }
    void release() {
        for (Reader& x : r) {
            for (int b = 0; b < 2; ++b) {
                if (x.done[b]) cudaEventDestroy(x.done[b]);
                if (x.stage[b]) cudaFreeHost(x.stage[b]);
                x.done[b] = nullptr;
                x.stage[b] = nullptr;
            }
            if (x.st) cudaStreamDestroy(x.st);
            x.st = nullptr;
        }
        device = -1;
    }
};

}  // namespace bundle
}  // namespace gtm

struct GtmBundle {
    std::string dir;
    GtmBundleInfo info;
    std::map<std::string, gtm::bundle::Entry> entries;
    std::map<std::string, gtm::bundle::Sub> block;
    std::vector<std::string> layer_files;   // by layer id
    gtm::bundle::Stager stager;
    ~GtmBundle() { stager.release(); }
};

namespace gtm {
namespace bundle {

void parse_manifest(GtmBundle& B) {
    const std::string path = B.dir + "/manifest.json";
    const std::string text = read_text(path);
    if (text.empty()) throw FormatError("manifest: empty JSON");
    const Json root = JsonReader(text, "manifest").parse();
    if (root.kind != Json::OBJ) throw FormatError("manifest: top level must be an object");
    if (as_str(need(root, "magic", "manifest"), "manifest.magic") != "GTURBO")
        throw FormatError("manifest.magic: expected GTURBO");
    const int64_t vmaj = as_int(need(root, "versionMajor", "manifest"), "manifest.versionMajor");
    const int64_t vmin = as_int(need(root, "versionMinor", "manifest"), "manifest.versionMinor");
    if (vmaj != 1 || vmin < 0) throw FormatError("manifest.version: unsupported version");
    if (const Json* f = root.find("flags")) {
        if (f->kind != Json::OBJ) throw FormatError("manifest.flags: expected an object");
        for (const auto& kv : f->obj) {
            if (kv.first != "streamingPresent" && kv.first != "turboQuantKV" && kv.first != "aneSharedExpert")
                throw FormatError("manifest.flags: unknown v1 flag: " + kv.first);
            if (kv.second.kind != Json::BOOL) throw FormatError("manifest.flags." + kv.first + ": expected a bool");
        }
    }
    const int64_t layers = as_int(need(root, "numLayers", "manifest"), "manifest.numLayers");
    const int64_t experts = as_int(need(root, "expertsPerLayer", "manifest"), "manifest.expertsPerLayer");
    const int64_t stride = as_int(need(root, "expertStride", "manifest"), "manifest.expertStride");
    if (layers <= 0 || experts <= 0 || stride <= 0 || stride % 4096 != 0)
        throw FormatError("manifest: invalid dimensions or stride");
    const Json& a = need(root, "arch", "manifest");
    if (a.kind != Json::OBJ) throw FormatError("manifest.arch: expected an object");
    const std::string ca = "manifest.arch";
    const int64_t hidden = int_or(a, "hiddenSize", 2816, ca), ffn = int_or(a, "ffnIntermediate", 2112, ca);
    const int64_t moe = int_or(a, "moeIntermediateSize", 704, ca), topk = int_or(a, "topKExperts", 8, ca);
    const int64_t an_layers = int_or(a, "numLayers", layers, ca), an_experts = int_or(a, "numExperts", experts, ca);
    if (an_layers != layers || an_experts != experts)
        throw FormatError("manifest.arch: dimensions disagree with streaming metadata");
    if (hidden <= 0 || ffn <= 0 || moe <= 0 || topk <= 0 || topk > experts)
        throw FormatError("manifest.arch: invalid architecture values");
    B.info.num_layers = (uint32_t)layers;
    B.info.experts_per_layer = (uint32_t)experts;
    B.info.expert_stride = (uint64_t)stride;
    B.info.hidden = (uint32_t)hidden;
    B.info.ffn_inter = (uint32_t)ffn;
    B.info.moe_inter = (uint32_t)moe;
    B.info.top_k = (uint32_t)topk;
    B.info.rms_norm_eps = (float)num_or(a, "rmsNormEps", 1e-6, ca);
}

void parse_layout(GtmBundle& B) {
    const std::string text = read_text(B.dir + "/packed_experts/layout.json");
    if (text.empty()) throw FormatError("layout: empty JSON");
    const Json root = JsonReader(text, "layout").parse();
    if (root.kind != Json::OBJ) throw FormatError("layout: top level must be an object");
    const int64_t stride = as_int(need(root, "expertStride", "layout"), "layout.expertStride");
    const int64_t layers = as_int(need(root, "numLayers", "layout"), "layout.numLayers");
    const int64_t experts = as_int(need(root, "expertsPerLayer", "layout"), "layout.expertsPerLayer");
    if (layers <= 0 || experts <= 0 || stride <= 0 || (uint64_t)stride % kAlign != 0)
        throw FormatError("layout: invalid dimensions, or stride not a multiple of 16384");
    if ((uint64_t)stride != B.info.expert_stride || (uint64_t)layers != B.info.num_layers ||
        (uint64_t)experts != B.info.experts_per_layer)
        throw FormatError("manifest/layout: numLayers, expertsPerLayer or expertStride disagree");
    const Json& blk = need(root, "expertBlock", "layout");
    if (blk.kind != Json::OBJ) throw FormatError("layout.expertBlock: expected an object");
    std::vector<std::pair<uint64_t, uint64_t>> spans;
    for (const auto& kv : blk.obj) {
        const std::string ctx = "layout.expertBlock." + kv.first;
        Sub t;
        t.offset = (uint64_t)as_int(need(kv.second, "offset", ctx), ctx + ".offset");
        t.size = (uint64_t)as_int(need(kv.second, "size", ctx), ctx + ".size");
        t.dtype = (uint8_t)int_or(kv.second, "dtype", 0, ctx);
        const uint64_t end = add_checked(t.offset, t.size, ctx);
        if (end > (uint64_t)stride) throw FormatError(ctx + ": extends past expert_stride");
        spans.emplace_back(t.offset, end);
        B.block[kv.first] = t;
    }
    static const char* const kRequired[] = {"gate_proj.weight", "gate_proj.scales", "gate_proj.biases",
                                            "up_proj.weight",   "up_proj.scales",   "up_proj.biases",
                                            "down_proj.weight", "down_proj.scales", "down_proj.biases"};
    for (const char* n : kRequired)
        if (!B.block.count(n)) throw FormatError(std::string("layout.expertBlock: missing required sub-tensor '") + n + "'");
    std::sort(spans.begin(), spans.end());
    for (size_t i = 1; i < spans.size(); ++i)
        if (spans[i].first < spans[i - 1].second) throw FormatError("layout.expertBlock: sub-tensors overlap");
    const Json& ls = need(root, "layers", "layout");
    if (ls.kind != Json::ARR) throw FormatError("layout.layers: expected an array");
    if ((int64_t)ls.arr.size() != layers)
        throw FormatError("layout.layers: expected " + std::to_string(layers) + " entries, got " + std::to_string(ls.arr.size()));
    B.layer_files.assign((size_t)layers, std::string());
    for (const Json& e : ls.arr) {
        const int64_t id = as_int(need(e, "layer", "layout.layers"), "layout.layers.layer");
        if (id < 0 || id >= layers || !B.layer_files[(size_t)id].empty())
            throw FormatError("layout.layers: duplicate or out-of-range layer ID " + std::to_string(id));
        const std::string& f = as_str(need(e, "file", "layout.layers"), "layout.layers.file");
        check_basename(f, "layout.layers.file");
        B.layer_files[(size_t)id] = f;
    }
    B.info.layer_file_bytes = (uint64_t)experts * (uint64_t)stride;
    for (size_t l = 0; l < B.layer_files.size(); ++l) {
        const std::string p = B.dir + "/packed_experts/" + B.layer_files[l];
        if (file_size(p) < B.info.layer_file_bytes)
            throw FormatError("packed_experts/" + B.layer_files[l] + ": shorter than expertsPerLayer x expertStride");
    }
}

void parse_resident(GtmBundle& B) {
    const std::string path = B.dir + "/resident.bin";
    const uint64_t fsize = file_size(path);
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) throw FormatError("cannot open " + path);
    uint8_t hdr[kHeader];
    if (fread(hdr, 1, kHeader, f) != kHeader) { fclose(f); throw FormatError("resident.header: truncated header"); }
    const uint64_t index_size = rd64(hdr), resident_size = rd64(hdr + 8), count = rd64(hdr + 16);
    if (index_size > kIndexMax) { fclose(f); throw FormatError("resident.indexSize: exceeds max cap"); }
    if (index_size > fsize || index_size < kHeader || index_size % kAlign != 0) {
        fclose(f);
        throw FormatError("resident.index: truncated or unaligned index");
    }
    std::vector<uint8_t> idx(index_size);
    memcpy(idx.data(), hdr, kHeader);
    if (fread(idx.data() + kHeader, 1, index_size - kHeader, f) != index_size - kHeader) {
        fclose(f);
        throw FormatError("resident.index: short read");
    }
    fclose(f);
    if (count > (kIndexMax - kHeader) / kEntry) throw FormatError("resident.entryTable: outside index range");
    const uint64_t table_end = kHeader + count * kEntry;
    if (table_end > index_size) throw FormatError("resident.entryTable: outside index range");
    if (resident_size > fsize) throw FormatError("resident.bin: shorter than the header's residentSize");
    for (uint64_t i = 0; i < count; ++i) {
        const uint8_t* e = idx.data() + kHeader + i * kEntry;
        const uint32_t name_off = rd32(e);
        const uint16_t name_len = rd16(e + 4);
        if (e[7] != 0) throw FormatError("resident.entry: reserved byte must be zero");
        if (name_off < table_end || (uint64_t)name_off + name_len > index_size)
            throw FormatError("resident.entry.name: range outside string table");
        Entry t;
        t.dtype = e[6];
        t.offset = rd64(e + 8);
        t.size = rd64(e + 16);
        for (int k = 0; k < 4; ++k) t.shape[k] = rd32(e + 24 + 4 * k);
        t.scale_offset = rd64(e + 40);
        t.scale_size = rd64(e + 48);
        t.bias_offset = rd64(e + 56);
        t.bias_size = rd64(e + 64);
        const std::string name(reinterpret_cast<const char*>(idx.data() + name_off), name_len);
        if (add_checked(t.offset, t.size, name) > fsize || add_checked(t.scale_offset, t.scale_size, name) > fsize ||
            add_checked(t.bias_offset, t.bias_size, name) > fsize)
            throw FormatError("resident." + name + ": data range past the end of resident.bin");
        B.entries[name] = t;
    }
    B.info.resident_bytes = fsize;
    B.info.resident_index_bytes = index_size;
    B.info.resident_entries = (uint32_t)count;
}

// ---- file -> device ---------------------------------------------------------------------------
// Chunks of the byte range go round-robin to the reader threads; each reads a chunk with pread
// into one of its two pinned buffers while the copy of its previous chunk runs on its stream.
int load_range(Stager& S, const std::string& path, uint64_t offset, uint64_t bytes, void* dst, const char* what) {
    if (bytes == 0) return GTM_OK;
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 == cudaSuccess) e0 = S.init(dev);
    if (e0 != cudaSuccess) return set_cuda_error(what, e0);
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) return set_error(GTM_ERR_INVALID, "%s: cannot open %s", what, path.c_str());
    const uint64_t nchunks = (bytes + kChunk - 1) / kChunk;
    const int nthreads = (int)std::min<uint64_t>(nchunks, kReaders);
    std::vector<int> status(nthreads, GTM_OK);
    std::vector<std::string> msg(nthreads);
    auto worker = [&](int k) {
        cudaSetDevice(dev);
        Reader& R = S.r[k];
        cudaError_t e = cudaSuccess;
        int used = 0;
        for (uint64_t c = (uint64_t)k; c < nchunks; c += (uint64_t)nthreads, ++used) {
            const int b = used & 1;
            if (used >= 2) e = cudaEventSynchronize(R.done[b]);   // the copy that last used this buffer
            if (e != cudaSuccess) break;
            const uint64_t off = c * kChunk, n = std::min(kChunk, bytes - off);
            uint64_t got = 0;
            while (got < n) {
                const ssize_t r = pread(fd, static_cast<uint8_t*>(R.stage[b]) + got, n - got, (off_t)(offset + off + got));
                if (r <= 0) {
                    if (r < 0 && errno == EINTR) continue;
                    status[k] = GTM_ERR_INVALID;
                    msg[k] = "short read of " + path;
                    break;
                }
                got += (uint64_t)r;
            }
            if (status[k] != GTM_OK) break;
            e = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, R.stage[b], n, cudaMemcpyHostToDevice, R.st);
            if (e == cudaSuccess) e = cudaEventRecord(R.done[b], R.st);
            if (e != cudaSuccess) break;
        }
        const cudaError_t e2 = cudaStreamSynchronize(R.st);
        if (e == cudaSuccess) e = e2;
        if (e != cudaSuccess && status[k] == GTM_OK) {
            status[k] = GTM_ERR_CUDA;
            msg[k] = cudaGetErrorString(e);
        }
    };
    std::vector<std::thread> th;
    for (int k = 0; k < nthreads; ++k) th.emplace_back(worker, k);
    for (auto& t : th) t.join();
    close(fd);
    for (int k = 0; k < nthreads; ++k)
        if (status[k] != GTM_OK) return set_error(status[k], "%s: %s", what, msg[k].c_str());
    return GTM_OK;
}

// A quantized resident tensor of `rows` x `in_dim` at `bits` (the runner derives in_dim from the
// scale table the same way, src/runner.cpp:334-347).
GtmQuant quant(const GtmBundle& B, const std::string& name, uint32_t rows, uint32_t in_dim, int bits) {
    auto it = B.entries.find(name);
    if (it == B.entries.end()) throw FormatError("resident index has no tensor '" + name + "'");
    const Entry& t = it->second;
    const uint64_t groups = in_dim / 64;
    if (t.shape[0] != rows || t.size != (uint64_t)rows * in_dim * bits / 8 || t.scale_size != (uint64_t)rows * groups * 2 ||
        t.bias_size != (uint64_t)rows * groups * 2)
        throw FormatError(name + ": expected " + std::to_string(rows) + " x " + std::to_string(in_dim) + " at " +
                          std::to_string(bits) + " bits with bf16 scales and biases per 64 inputs");
    return GtmQuant{t.offset, t.scale_offset, t.bias_offset};
}

uint64_t vec_bf16(const GtmBundle& B, const std::string& name, uint32_t n) {
    auto it = B.entries.find(name);
    if (it == B.entries.end()) throw FormatError("resident index has no tensor '" + name + "'");
    const Entry& t = it->second;
    if (t.dtype != DT_BF16 || t.size != 2ull * n)
        throw FormatError(name + ": expected bf16[" + std::to_string(n) + "]");
    return t.offset;
}

GtmQuant expert_quant(const GtmBundle& B, const char* proj, uint32_t rows, uint32_t in_dim) {
    const std::string p(proj);
    const Sub& w = B.block.at(p + ".weight");
    const Sub& s = B.block.at(p + ".scales");
    const Sub& b = B.block.at(p + ".biases");
    const uint64_t groups = in_dim / 64;
    if (w.size != (uint64_t)rows * in_dim / 2 || s.size != (uint64_t)rows * groups * 2 || b.size != (uint64_t)rows * groups * 2)
        throw FormatError("layout.expertBlock." + p + ": expected " + std::to_string(rows) + " x " + std::to_string(in_dim) +
                          " at 4 bits with bf16 scales and biases per 64 inputs");
    return GtmQuant{w.offset, s.offset, b.offset};
}

}  // namespace bundle
}  // namespace gtm

using gtm::bundle::FormatError;

extern "C" {

GTM_API int gtm_bundle_open(const char* dir, GtmBundle** out) {
    if (!dir || !out) return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_open: null argument");
    *out = nullptr;
    GtmBundle* B = new GtmBundle();
    memset(&B->info, 0, sizeof(B->info));
    B->dir = dir;
    try {
        gtm::bundle::parse_manifest(*B);
        gtm::bundle::parse_layout(*B);
        gtm::bundle::parse_resident(*B);
    } catch (const std::exception& e) {
        delete B;
        return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_open: %s", e.what());
    }
    *out = B;
    gtm::clear_error();
    return GTM_OK;
}

GTM_API int gtm_bundle_close(GtmBundle* B) {
    delete B;
    gtm::clear_error();
    return GTM_OK;
}

GTM_API int gtm_bundle_info(const GtmBundle* B, GtmBundleInfo* out) {
    if (!B || !out) return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_info: null argument");
    *out = B->info;
    gtm::clear_error();
    return GTM_OK;
}

GTM_API int gtm_bundle_load_resident(GtmBundle* B, void* dst, uint64_t dst_bytes) {
    if (!B || !dst) return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_load_resident: null argument");
    if (dst_bytes < B->info.resident_bytes)
        return gtm::set_error(GTM_ERR_WORKSPACE, "gtm_bundle_load_resident: needs %llu bytes",
                              (unsigned long long)B->info.resident_bytes);
    const int rc = gtm::bundle::load_range(B->stager, B->dir + "/resident.bin", 0, B->info.resident_bytes, dst,
                                           "gtm_bundle_load_resident");
    if (rc == GTM_OK) gtm::clear_error();
    return rc;
}

GTM_API int gtm_bundle_load_experts(GtmBundle* B, uint32_t layer, uint32_t first, uint32_t count, void* dst,
                                    uint64_t dst_bytes) {
    if (!B || !dst) return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_load_experts: null argument");
    if (layer >= B->info.num_layers || (uint64_t)first + count > B->info.experts_per_layer)
        return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_load_experts: layer %u / experts [%u, %u) out of range", layer,
                              first, first + count);
    const uint64_t bytes = (uint64_t)count * B->info.expert_stride;
    if (dst_bytes < bytes)
        return gtm::set_error(GTM_ERR_WORKSPACE, "gtm_bundle_load_experts: needs %llu bytes", (unsigned long long)bytes);
    const int rc = gtm::bundle::load_range(B->stager, B->dir + "/packed_experts/" + B->layer_files[layer],
                                           (uint64_t)first * B->info.expert_stride, bytes, dst, "gtm_bundle_load_experts");
    if (rc == GTM_OK) gtm::clear_error();
    return rc;
}

GTM_API int gtm_bundle_layer_desc(const GtmBundle* B, uint32_t layer, const void* resident_dev, const void* experts_dev,
                                  GtmLayer* out) {
    if (!B || !out) return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_layer_desc: null argument");
    if (layer >= B->info.num_layers)
        return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_layer_desc: layer %u >= %u", layer, B->info.num_layers);
    const uint32_t D = B->info.hidden, F = B->info.ffn_inter, M = B->info.moe_inter, E = B->info.experts_per_layer;
    const std::string P = "model.layers." + std::to_string(layer) + ".";
    GtmLayer L;
    memset(&L, 0, sizeof(L));
    try {
        using namespace gtm::bundle;
        L.resident_dev = resident_dev;
        L.router = quant(*B, P + "router.proj.weight", E, D, 8);
        L.router_scale = vec_bf16(*B, P + "router.scale", D);
        L.per_expert_scale = vec_bf16(*B, P + "router.per_expert_scale", E);
        L.shared_gate = quant(*B, P + "mlp.gate_proj.weight", F, D, 4);
        L.shared_up = quant(*B, P + "mlp.up_proj.weight", F, D, 4);
        L.shared_down = quant(*B, P + "mlp.down_proj.weight", D, F, 4);
        L.pre_ffn_norm = vec_bf16(*B, P + "pre_feedforward_layernorm.weight", D);
        L.pre_ffn_norm_2 = vec_bf16(*B, P + "pre_feedforward_layernorm_2.weight", D);
        L.post_ffn_norm_1 = vec_bf16(*B, P + "post_feedforward_layernorm_1.weight", D);
        L.post_ffn_norm_2 = vec_bf16(*B, P + "post_feedforward_layernorm_2.weight", D);
        L.post_ffn_norm = vec_bf16(*B, P + "post_feedforward_layernorm.weight", D);
        L.layer_scalar = vec_bf16(*B, P + "layer_scalar", 1);
        L.experts_dev = experts_dev;
        L.expert_stride = B->info.expert_stride;
        L.expert_gate = expert_quant(*B, "gate_proj", M, D);
        L.expert_up = expert_quant(*B, "up_proj", M, D);
        L.expert_down = expert_quant(*B, "down_proj", D, M);
    } catch (const std::exception& e) {
        return gtm::set_error(GTM_ERR_INVALID, "gtm_bundle_layer_desc: %s", e.what());
    }
    *out = L;
    gtm::clear_error();
    return GTM_OK;
}

}  // extern "C"
