// g4s_vpk.cu -- the reference's weight archive, read on the host, and the LM
// head moved from it to the device.
//
// Format (StdApp's TVFS, src/vendor/StdApp/StdApp.VFS.pas:68-85, little endian,
// packed): a 52-byte header (magic "VPK0", version u32 = 1, entry count u32,
// data start u64, 32 reserved bytes), then per entry 544 bytes: the entry path
// as 260 UTF-16 code units (NUL-padded), offset u64 (from the start of the
// archive), size u64, CRC-32 u32 (IEEE polynomial, the zlib one), flags u32.
// Entry paths are looked up lower-cased with '/' separators (TVFS.NormalizePath,
// :180-183).  The model's tensors live in two entries (TWeightStore.Open,
// src/Gemma4.Tensors.pas:321-380; default paths src/Gemma4.Types.pas:79, 85):
// manifest.json = {"tensors": [{"name", "source_dtype", "output_dtype",
// "offset", "size", "shape"}, ...]} (DoParseManifest, :396-455) and
// weights.bin, into which the manifest's offsets point.
//
// The archive is mapped read-only (as the reference maps it); nothing is
// copied until a caller moves a tensor to the device.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "g4s_kernels.cuh"
#include "g4sampler.h"

extern "C" int32_t g4s_noalloc_set_error(const char *msg);  // g4s_api.cu: thread error text

namespace {

constexpr size_t HEADER_BYTES = 52;
constexpr size_t ENTRY_BYTES = 544;
constexpr int PATH_UNITS = 260;

struct Entry {
    uint64_t offset, size;
    uint32_t crc, flags;
};

uint32_t crc32_update(uint32_t crc, const uint8_t *p, size_t n)
{
    static uint32_t table[256];
    static bool init = false;
    if (!init) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int b = 0; b < 8; b++) c = (c & 1u) ? (c >> 1) ^ 0xEDB88320u : c >> 1;
            table[i] = c;
        }
        init = true;
    }
    for (size_t i = 0; i < n; i++) crc = table[(crc ^ p[i]) & 0xFFu] ^ (crc >> 8);
    return crc;
}

std::string normalize(const std::string &p)
{
    std::string r = p;
    for (char &c : r) {
        if (c == '\\') c = '/';
        c = (char)std::tolower((unsigned char)c);
    }
    return r;
}

uint32_t rd32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }
uint64_t rd64(const uint8_t *p) { uint64_t v; memcpy(&v, p, 8); return v; }

// A small JSON reader: enough for the manifest (objects, arrays, strings,
// numbers, true/false/null); values are kept as a tree.
struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    double num = 0;
    uint64_t unum = 0;  // exact value of a non-negative integer literal
    bool is_uint = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
    const JVal *get(const char *k) const
    {
        for (auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JParser {
    const char *p, *end;
    std::string err;
    void ws()
    {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool fail(const char *m)
    {
        if (err.empty()) err = m;
        return false;
    }
    bool str(std::string &out)
    {
        if (p >= end || *p != '"') return fail("string expected");
        p++;
        while (p < end && *p != '"') {
            if (*p == '\\') {
                if (++p >= end) return fail("bad escape");
                switch (*p) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {
                    if (end - p < 5) return fail("bad \\u escape");
                    unsigned cp = 0;
                    for (int i = 1; i <= 4; i++) {
                        const char h = p[i];
                        cp = cp * 16 + (unsigned)(isdigit((unsigned char)h) ? h - '0' : (tolower(h) - 'a' + 10));
                    }
                    p += 4;
                    if (cp < 0x80) out += (char)cp;
                    else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
                    else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
                    break;
                }
                default: out += *p;
                }
                p++;
            } else {
                out += *p++;
            }
        }
        if (p >= end) return fail("unterminated string");
        p++;
        return true;
    }
    bool value(JVal &v, int depth)
    {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        if (*p == '{') {
            v.kind = JVal::OBJ;
            p++;
            ws();
            if (p < end && *p == '}') { p++; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (p >= end || *p != ':') return fail("':' expected");
                p++;
                v.obj.emplace_back(k, JVal());
                if (!value(v.obj.back().second, depth + 1)) return false;
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == '}') { p++; return true; }
                return fail("',' or '}' expected");
            }
        }
        if (*p == '[') {
            v.kind = JVal::ARR;
            p++;
            ws();
            if (p < end && *p == ']') { p++; return true; }
            for (;;) {
                v.arr.emplace_back();
                if (!value(v.arr.back(), depth + 1)) return false;
                ws();
                if (p < end && *p == ',') { p++; continue; }
                if (p < end && *p == ']') { p++; return true; }
                return fail("',' or ']' expected");
            }
        }
        if (*p == '"') {
            v.kind = JVal::STR;
            return str(v.str);
        }
        if (end - p >= 4 && !strncmp(p, "true", 4)) { v.kind = JVal::BOOL; v.num = 1; p += 4; return true; }
        if (end - p >= 5 && !strncmp(p, "false", 5)) { v.kind = JVal::BOOL; p += 5; return true; }
        if (end - p >= 4 && !strncmp(p, "null", 4)) { v.kind = JVal::NUL; p += 4; return true; }
        // number
        const char *s = p;
        bool digits_only = true;
        if (p < end && (*p == '-' || *p == '+')) { digits_only = false; p++; }
        while (p < end && (isdigit((unsigned char)*p) || *p == '.' || *p == 'e' || *p == 'E' || *p == '-' || *p == '+')) {
            if (!isdigit((unsigned char)*p)) digits_only = false;
            p++;
        }
        if (p == s) return fail("value expected");
        std::string tok(s, p - s);
        v.kind = JVal::NUM;
        v.num = strtod(tok.c_str(), nullptr);
        if (digits_only) {
            v.is_uint = true;
            v.unum = strtoull(tok.c_str(), nullptr, 10);
        }
        return true;
    }
};

int32_t dtype_from(const std::string &s)
{
    // DtypeKindFromString (src/Gemma4.Types.pas:505-517)
    if (s == "BF16") return G4S_DT_BF16;
    if (s == "F16") return G4S_DT_F16;
    if (s == "F32") return G4S_DT_F32;
    if (s == "Q4_0") return G4S_DT_Q4_0;
    return G4S_DT_UNKNOWN;
}

int32_t vfail(int32_t code, const std::string &m)
{
    g4s_noalloc_set_error(m.c_str());
    return code;
}

}  // namespace

struct g4s_vpk {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t len = 0;
    std::map<std::string, Entry> entries;
    Entry weights{};
    std::vector<g4s_tensor_info> tensors;
    std::map<std::string, size_t> lookup;
    ~g4s_vpk()
    {
        if (map) munmap((void *)map, len);
        if (fd >= 0) close(fd);
    }
};

extern "C" {

int32_t g4s_vpk_open(const char *path, const char *manifest_path, const char *weights_path, g4s_vpk **out)
{
    g4s_noalloc_set_error("");
    if (!path || !out) return vfail(G4S_ERR_ARG, "g4s_vpk_open: path and out must be non-NULL");
    *out = nullptr;
    const std::string mpath = normalize(manifest_path ? manifest_path : "E4B/manifest.json");
    const std::string wpath = normalize(weights_path ? weights_path : "E4B/weights.bin");
    g4s_vpk *v = new g4s_vpk();
    v->fd = open(path, O_RDONLY);
    if (v->fd < 0) {
        delete v;
        return vfail(G4S_ERR_ARG, std::string("g4s_vpk_open: cannot open ") + path);
    }
    struct stat st;
    if (fstat(v->fd, &st) != 0 || st.st_size < (off_t)HEADER_BYTES) {
        delete v;
        return vfail(G4S_ERR_ARG, std::string("g4s_vpk_open: archive shorter than its header: ") + path);
    }
    v->len = (size_t)st.st_size;
    void *m = mmap(nullptr, v->len, PROT_READ, MAP_PRIVATE, v->fd, 0);
    if (m == MAP_FAILED) {
        delete v;
        return vfail(G4S_ERR_ARG, std::string("g4s_vpk_open: cannot map ") + path);
    }
    v->map = (const uint8_t *)m;
    if (memcmp(v->map, "VPK0", 4) != 0) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: not a VPK archive (magic)");
    }
    const uint32_t version = rd32(v->map + 4);
    if (version != 1) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: unsupported VPK version " + std::to_string(version));
    }
    const uint32_t count = rd32(v->map + 8);
    if ((uint64_t)HEADER_BYTES + (uint64_t)count * ENTRY_BYTES > v->len) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: directory truncated");
    }
    for (uint32_t i = 0; i < count; i++) {
        const uint8_t *e = v->map + HEADER_BYTES + (size_t)i * ENTRY_BYTES;
        std::string name;
        for (int k = 0; k < PATH_UNITS; k++) {
            uint16_t u;
            memcpy(&u, e + 2 * k, 2);
            if (!u) break;
            if (u < 0x80) name += (char)u;
            else if (u < 0x800) { name += (char)(0xC0 | (u >> 6)); name += (char)(0x80 | (u & 0x3F)); }
            else { name += (char)(0xE0 | (u >> 12)); name += (char)(0x80 | ((u >> 6) & 0x3F)); name += (char)(0x80 | (u & 0x3F)); }
        }
        Entry en{rd64(e + 520), rd64(e + 528), rd32(e + 536), rd32(e + 540)};
        if (en.offset > v->len || en.size > v->len - en.offset) {
            delete v;
            return vfail(G4S_ERR_ARG, "g4s_vpk_open: entry '" + name + "' lies outside the archive");
        }
        v->entries[normalize(name)] = en;
    }
    auto mi = v->entries.find(mpath);
    if (mi == v->entries.end()) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: manifest not found in the archive: " + mpath);
    }
    auto wi = v->entries.find(wpath);
    if (wi == v->entries.end()) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: weights not found in the archive: " + wpath);
    }
    v->weights = wi->second;
    JParser jp{(const char *)v->map + mi->second.offset, (const char *)v->map + mi->second.offset + mi->second.size, ""};
    JVal root;
    if (!jp.value(root, 0) || root.kind != JVal::OBJ) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: cannot parse the manifest: " + (jp.err.empty() ? "not an object" : jp.err));
    }
    const JVal *ts = root.get("tensors");
    if (!ts || ts->kind != JVal::ARR || ts->arr.empty()) {
        delete v;
        return vfail(G4S_ERR_ARG, "g4s_vpk_open: the manifest has no tensors array");
    }
    for (const JVal &t : ts->arr) {
        g4s_tensor_info ti;
        memset(&ti, 0, sizeof(ti));
        const JVal *nm = t.get("name"), *sd = t.get("source_dtype"), *od = t.get("output_dtype"), *of = t.get("offset"),
                   *sz = t.get("size"), *sh = t.get("shape");
        std::string name = nm && nm->kind == JVal::STR ? nm->str : "";
        strncpy(ti.name, name.c_str(), sizeof(ti.name) - 1);
        ti.source_dtype = sd && sd->kind == JVal::STR ? dtype_from(sd->str) : G4S_DT_UNKNOWN;
        ti.output_dtype = od && od->kind == JVal::STR ? dtype_from(od->str) : G4S_DT_UNKNOWN;
        ti.offset = of && of->is_uint ? of->unum : 0;
        ti.size = sz && sz->is_uint ? sz->unum : 0;
        if (sh && sh->kind == JVal::ARR)
            for (const JVal &d : sh->arr)
                if (ti.ndim < G4S_MAX_DIMS) ti.shape[ti.ndim++] = d.kind == JVal::NUM ? (int64_t)d.num : 0;
        if (ti.offset > v->weights.size || ti.size > v->weights.size - ti.offset) {
            delete v;
            return vfail(G4S_ERR_ARG, "g4s_vpk_open: tensor '" + name + "' lies outside weights.bin");
        }
        v->lookup[name] = v->tensors.size();  // a later duplicate wins, as AddOrSetValue does
        v->tensors.push_back(ti);
    }
    *out = v;
    return G4S_OK;
}

int32_t g4s_vpk_close(g4s_vpk *vpk)
{
    delete vpk;
    return G4S_OK;
}

int32_t g4s_vpk_tensor_count(const g4s_vpk *vpk) { return vpk ? (int32_t)vpk->tensors.size() : 0; }

int32_t g4s_vpk_tensor_at(const g4s_vpk *vpk, int32_t index, g4s_tensor_info *info)
{
    if (!vpk || !info || index < 0 || index >= (int32_t)vpk->tensors.size())
        return vfail(G4S_ERR_ARG, "g4s_vpk_tensor_at: bad archive, index or info");
    *info = vpk->tensors[(size_t)index];
    return G4S_OK;
}

int32_t g4s_vpk_find(const g4s_vpk *vpk, const char *name, g4s_tensor_info *info)
{
    if (!vpk || !name || !info) return vfail(G4S_ERR_ARG, "g4s_vpk_find: NULL argument");
    auto it = vpk->lookup.find(name);
    if (it == vpk->lookup.end()) return vfail(G4S_ERR_ARG, std::string("g4s_vpk_find: tensor not found: ") + name);
    *info = vpk->tensors[it->second];
    return G4S_OK;
}

const void *g4s_vpk_data(const g4s_vpk *vpk, const g4s_tensor_info *info)
{
    if (!vpk || !info || info->offset > vpk->weights.size || info->size > vpk->weights.size - info->offset) return nullptr;
    return vpk->map + vpk->weights.offset + info->offset;
}

int32_t g4s_vpk_verify(const g4s_vpk *vpk, const char *entry_path)
{
    if (!vpk || !entry_path) return vfail(G4S_ERR_ARG, "g4s_vpk_verify: NULL argument");
    auto it = vpk->entries.find(normalize(entry_path));
    if (it == vpk->entries.end()) return vfail(G4S_ERR_ARG, std::string("g4s_vpk_verify: no entry ") + entry_path);
    const uint32_t crc = crc32_update(0xFFFFFFFFu, vpk->map + it->second.offset, it->second.size) ^ 0xFFFFFFFFu;
    if (crc != it->second.crc)
        return vfail(G4S_ERR_STATE, std::string("g4s_vpk_verify: checksum mismatch in ") + entry_path);
    return G4S_OK;
}

int32_t g4s_vpk_load_lmhead(const g4s_vpk *vpk, int32_t device, uint8_t *nibbles, uint16_t *scales, int32_t max_vocab,
                            int32_t *out_vocab, int32_t *out_hidden, void *stream)
{
    if (!vpk || !nibbles || !scales || !out_vocab || !out_hidden)
        return vfail(G4S_ERR_ARG, "g4s_vpk_load_lmhead: NULL argument");
    // the projection DoRecordFinalGpu uses (src/Gemma4.Model.pas:1293-1299): an
    // lm_head tensor when the archive has one, else the tied embed_tokens
    g4s_tensor_info ti;
    auto it = vpk->lookup.find("model.language_model.lm_head.weight");
    if (it == vpk->lookup.end()) it = vpk->lookup.find("model.language_model.embed_tokens.weight");
    if (it == vpk->lookup.end())
        return vfail(G4S_ERR_ARG, "g4s_vpk_load_lmhead: neither lm_head nor embed_tokens is in the manifest");
    ti = vpk->tensors[it->second];
    if (ti.output_dtype != G4S_DT_Q4_0 || ti.ndim != 2)
        return vfail(G4S_ERR_ARG, std::string("g4s_vpk_load_lmhead: ") + ti.name + " is not a 2-D Q4_0 tensor");
    const int64_t vocab = ti.shape[0], hidden = ti.shape[1];
    if (vocab < 1 || hidden < 32 || hidden % 32 || vocab > max_vocab || vocab > INT32_MAX ||
        (uint64_t)vocab * (uint64_t)(hidden / 32) * 18u != ti.size)
        return vfail(G4S_ERR_ARG, std::string("g4s_vpk_load_lmhead: ") + ti.name + " has shape/size " +
                                      std::to_string(vocab) + "x" + std::to_string(hidden) + "/" +
                                      std::to_string(ti.size) + " (want vocab <= " + std::to_string(max_vocab) +
                                      ", hidden a multiple of 32, 18 bytes per 32 values)");
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return vfail(G4S_ERR_CUDA, "g4s_vpk_load_lmhead: cannot select device " + std::to_string(device));
    }
    cudaStream_t s = (cudaStream_t)stream;
    void *staging = nullptr;
    cudaError_t e = cudaMalloc(&staging, ti.size);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(staging, vpk->map + vpk->weights.offset + ti.offset, ti.size, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = g4s::launch_q4_repack((const uint8_t *)staging, (int)vocab, (int)hidden, nibbles, scales, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (staging) cudaFree(staging);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return vfail(G4S_ERR_CUDA, std::string("g4s_vpk_load_lmhead: ") + cudaGetErrorString(e));
    }
    *out_vocab = (int32_t)vocab;
    *out_hidden = (int32_t)hidden;
    return G4S_OK;
}

}  // extern "C"
