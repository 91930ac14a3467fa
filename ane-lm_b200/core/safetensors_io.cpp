// safetensors_io.cpp -- safetensors header parsing, shard discovery, blob
// header and path (see safetensors_io.h).
#include "safetensors_io.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <set>
#include <sstream>

namespace ane_lm {
namespace cuda {

namespace fs = std::filesystem;

int64_t TensorInfo::numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
}

// ---------------------------------------------------------------------------
// A small JSON reader: enough for safetensors headers and shard indexes
// (objects, arrays, strings with escapes, integers, numbers, literals).
// ---------------------------------------------------------------------------
namespace {

struct Json {
    enum Kind { Null, Bool, Int, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    int64_t i = 0;
    double d = 0;
    std::string s;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* get(const std::string& k) const {
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class JsonReader {
public:
    JsonReader(const char* p, size_t n) : base_(p), p_(p), end_(p + n) {}
    bool parse(Json* out, std::string* err) {
        if (!value(out, 0)) {
            if (err) *err = "JSON parse error at byte " + std::to_string(p_ - base_);
            return false;
        }
        return true;
    }

private:
    const char* base_;
    const char* p_;
    const char* end_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) p_++;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if ((size_t)(end_ - p_) < n || memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    bool str(std::string* s) {
        if (p_ >= end_ || *p_ != '"') return false;
        p_++;
        while (p_ < end_ && *p_ != '"') {
            if (*p_ == '\\') {
                if (++p_ >= end_) return false;
                switch (*p_) {
                    case 'n': s->push_back('\n'); break;
                    case 't': s->push_back('\t'); break;
                    case 'r': s->push_back('\r'); break;
                    case 'b': s->push_back('\b'); break;
                    case 'f': s->push_back('\f'); break;
                    case 'u': {  // kept as UTF-8 for the BMP
                        if (end_ - p_ < 5) return false;
                        unsigned cp = (unsigned)strtoul(std::string(p_ + 1, 4).c_str(), nullptr, 16);
                        p_ += 4;
                        if (cp < 0x80) s->push_back((char)cp);
                        else if (cp < 0x800) {
                            s->push_back((char)(0xC0 | (cp >> 6)));
                            s->push_back((char)(0x80 | (cp & 0x3F)));
                        } else {
                            s->push_back((char)(0xE0 | (cp >> 12)));
                            s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
                            s->push_back((char)(0x80 | (cp & 0x3F)));
                        }
                        break;
                    }
                    default: s->push_back(*p_); break;  // \" \\ \/
                }
                p_++;
            } else {
                s->push_back(*p_++);
            }
        }
        if (p_ >= end_) return false;
        p_++;
        return true;
    }
    bool value(Json* v, int depth) {
        if (depth > 64) return false;
        ws();
        if (p_ >= end_) return false;
        const char c = *p_;
        if (c == '{') {
            v->kind = Json::Obj;
            p_++;
            ws();
            if (p_ < end_ && *p_ == '}') { p_++; return true; }
            while (true) {
                ws();
                std::string k;
                if (!str(&k)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                p_++;
                Json item;
                if (!value(&item, depth + 1)) return false;
                v->obj.emplace_back(std::move(k), std::move(item));
                ws();
                if (p_ < end_ && *p_ == ',') { p_++; continue; }
                if (p_ < end_ && *p_ == '}') { p_++; return true; }
                return false;
            }
        }
        if (c == '[') {
            v->kind = Json::Arr;
            p_++;
            ws();
            if (p_ < end_ && *p_ == ']') { p_++; return true; }
            while (true) {
                Json item;
                if (!value(&item, depth + 1)) return false;
                v->arr.push_back(std::move(item));
                ws();
                if (p_ < end_ && *p_ == ',') { p_++; continue; }
                if (p_ < end_ && *p_ == ']') { p_++; return true; }
                return false;
            }
        }
        if (c == '"') { v->kind = Json::Str; return str(&v->s); }
        if (lit("true")) { v->kind = Json::Bool; v->b = true; return true; }
        if (lit("false")) { v->kind = Json::Bool; v->b = false; return true; }
        if (lit("null")) { v->kind = Json::Null; return true; }
        // number
        const char* q = p_;
        bool integral = true;
        if (q < end_ && (*q == '-' || *q == '+')) q++;
        const char* digits = q;
        while (q < end_ && ((*q >= '0' && *q <= '9') || *q == '.' || *q == 'e' || *q == 'E' ||
                            *q == '-' || *q == '+')) {
            if (*q == '.' || *q == 'e' || *q == 'E') integral = false;
            q++;
        }
        if (q == digits) return false;
        const std::string num(p_, q);
        p_ = q;
        if (integral) {
            v->kind = Json::Int;
            v->i = strtoll(num.c_str(), nullptr, 10);
            v->d = (double)v->i;
        } else {
            v->kind = Json::Num;
            v->d = strtod(num.c_str(), nullptr);
        }
        return true;
    }
};

TensorDtype dtype_of(const std::string& s) {
    if (s == "BF16") return TensorDtype::BF16;
    if (s == "F16") return TensorDtype::F16;
    if (s == "F32") return TensorDtype::F32;
    if (s == "F64") return TensorDtype::F64;
    if (s == "I32") return TensorDtype::I32;
    if (s == "I64") return TensorDtype::I64;
    if (s == "U8") return TensorDtype::U8;
    return TensorDtype::Unknown;
}

}  // namespace

// ---------------------------------------------------------------------------
SafetensorsFile::~SafetensorsFile() {
    if (map_) munmap(map_, map_size_);
}

bool SafetensorsFile::open(const std::string& path, std::string* err) {
    path_ = path;
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { *err = "cannot open " + path; return false; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) {
        ::close(fd);
        *err = "not a safetensors file: " + path;
        return false;
    }
    map_size_ = (size_t)st.st_size;
    map_ = mmap(nullptr, map_size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) { map_ = nullptr; *err = "mmap failed: " + path; return false; }
    uint64_t hsize = 0;
    memcpy(&hsize, map_, 8);  // little-endian u64 header length
    if (hsize > map_size_ - 8) { *err = "invalid safetensors header size: " + path; return false; }
    data_ = (const uint8_t*)map_ + 8 + hsize;
    data_bytes_ = map_size_ - 8 - (size_t)hsize;
    Json root;
    JsonReader rd((const char*)map_ + 8, (size_t)hsize);
    std::string perr;
    if (!rd.parse(&root, &perr) || root.kind != Json::Obj) {
        *err = "failed to parse safetensors header of " + path + (perr.empty() ? "" : ": " + perr);
        return false;
    }
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const Json& o = kv.second;
        const Json* dt = o.get("dtype");
        const Json* sh = o.get("shape");
        const Json* off = o.get("data_offsets");
        if (o.kind != Json::Obj || !dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !off ||
            off->kind != Json::Arr || off->arr.size() != 2) {
            *err = "malformed tensor entry '" + kv.first + "' in " + path;
            return false;
        }
        TensorInfo t;
        t.name = kv.first;
        t.dtype = dtype_of(dt->s);
        for (const Json& d : sh->arr) {
            if (d.kind != Json::Int || d.i < 0) { *err = "bad shape of '" + kv.first + "'"; return false; }
            t.shape.push_back(d.i);
        }
        if (off->arr[0].kind != Json::Int || off->arr[1].kind != Json::Int || off->arr[0].i < 0 ||
            off->arr[1].i < off->arr[0].i || (uint64_t)off->arr[1].i > data_bytes_) {
            *err = "bad data_offsets of '" + kv.first + "' in " + path;
            return false;
        }
        t.begin = (uint64_t)off->arr[0].i;
        t.end = (uint64_t)off->arr[1].i;
        tensors_.push_back(std::move(t));
    }
    return true;
}

bool discover_shards(const std::string& model_dir, std::vector<std::string>* files,
                     std::string* err) {
    files->clear();
    std::error_code ec;
    const fs::path dir(model_dir);
    if (!fs::is_directory(dir, ec)) { *err = "model directory not found: " + model_dir; return false; }
    const fs::path index = dir / "model.safetensors.index.json";
    if (fs::is_regular_file(index, ec)) {
        std::ifstream f(index);
        std::stringstream ss;
        ss << f.rdbuf();
        const std::string text = ss.str();
        Json root;
        JsonReader rd(text.data(), text.size());
        std::string perr;
        const Json* wm = nullptr;
        if (!rd.parse(&root, &perr) || !(wm = root.get("weight_map")) || wm->kind != Json::Obj) {
            *err = "invalid shard index JSON: " + index.string();
            return false;
        }
        std::set<std::string> uniq;
        for (const auto& kv : wm->obj)
            if (kv.second.kind == Json::Str) uniq.insert(kv.second.s);
        if (uniq.empty()) { *err = "no shard files listed in " + index.string(); return false; }
        for (const std::string& rel : uniq) {  // std::set iterates sorted
            const fs::path p = dir / rel;
            if (!fs::is_regular_file(p, ec)) { *err = "missing shard file: " + p.string(); return false; }
            files->push_back(p.string());
        }
        return true;
    }
    std::vector<fs::path> found;
    for (const auto& e : fs::recursive_directory_iterator(dir, ec)) {
        if (e.is_regular_file() && e.path().extension() == ".safetensors") found.push_back(e.path());
    }
    if (ec) { *err = "failed to enumerate files in " + model_dir; return false; }
    std::sort(found.begin(), found.end());
    for (const auto& p : found) files->push_back(p.string());
    if (files->empty()) { *err = "no .safetensors files found in " + model_dir; return false; }
    return true;
}

void ane_blob_header(uint8_t h[128], uint64_t data_bytes) {
    memset(h, 0, 128);
    h[0] = 0x01;  // global header
    h[4] = 0x02;
    uint8_t* c = h + 64;  // chunk header
    c[0] = 0xEF; c[1] = 0xBE; c[2] = 0xAD; c[3] = 0xDE;
    c[4] = 0x01;
    const uint32_t size = (uint32_t)data_bytes;  // 32-bit field, as written by ANE-LM
    const uint32_t offset = 128;
    memcpy(c + 8, &size, 4);
    memcpy(c + 16, &offset, 4);
}

std::string ane_blob_path(const std::string& output_dir, const std::string& name) {
    std::string rel = name;
    std::replace(rel.begin(), rel.end(), '.', '/');
    return output_dir + "/" + rel + ".bin";
}

}  // namespace cuda
}  // namespace ane_lm
