// Hugging Face checkpoint directory reader: a small JSON parser, the
// safetensors header format (8-byte little-endian header length, a JSON object
// of name -> {dtype, shape, data_offsets}, then the payload), the sharded
// index (weight_map: name -> shard file) and the Llama config fields.
#include "runtime/hf_checkpoint.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstring>
#include <fstream>
#include <set>
#include <sstream>

namespace aethermind {
namespace hf {

// ---------------------------------------------------------------- JSON
namespace {

struct Json {
    enum Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = kNull;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* Find(const std::string& k) const {
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
public:
    explicit JsonParser(const std::string& s) : s_(s) {}
    StatusOr<Json> Parse() {
        Json v;
        AM_RETURN_IF_ERROR(Value(v, 0));
        Ws();
        if (i_ != s_.size()) return Err("trailing characters");
        return v;
    }

private:
    Status Err(const std::string& what) const {
        return Status::InvalidArgument("malformed JSON at byte " + std::to_string(i_) + ": " + what);
    }
    void Ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    bool Lit(const char* w) {
        const size_t n = std::strlen(w);
        if (s_.compare(i_, n, w) != 0) return false;
        i_ += n;
        return true;
    }
    Status String(std::string& out) {
        if (i_ >= s_.size() || s_[i_] != '"') return Err("expected a string");
        ++i_;
        while (i_ < s_.size() && s_[i_] != '"') {
            char c = s_[i_++];
            if (c == '\\') {
                if (i_ >= s_.size()) return Err("unterminated escape");
                const char e = s_[i_++];
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
                        if (i_ + 4 > s_.size()) return Err("short \\u escape");
                        const unsigned cp = (unsigned)std::stoul(s_.substr(i_, 4), nullptr, 16);
                        i_ += 4;
                        // names and config keys are ASCII; keep other code points as UTF-8
                        if (cp < 0x80) out += (char)cp;
                        else if (cp < 0x800) {
                            out += (char)(0xC0 | (cp >> 6));
                            out += (char)(0x80 | (cp & 0x3F));
                        } else {
                            out += (char)(0xE0 | (cp >> 12));
                            out += (char)(0x80 | ((cp >> 6) & 0x3F));
                            out += (char)(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: return Err("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (i_ >= s_.size()) return Err("unterminated string");
        ++i_;
        return Status::Ok();
    }
    Status Value(Json& v, int depth) {
        if (depth > 64) return Err("nesting too deep");
        Ws();
        if (i_ >= s_.size()) return Err("unexpected end");
        const char c = s_[i_];
        if (c == '{') {
            v.kind = Json::kObject;
            ++i_;
            Ws();
            if (i_ < s_.size() && s_[i_] == '}') {
                ++i_;
                return Status::Ok();
            }
            for (;;) {
                Ws();
                std::string k;
                AM_RETURN_IF_ERROR(String(k));
                Ws();
                if (i_ >= s_.size() || s_[i_] != ':') return Err("expected ':'");
                ++i_;
                Json e;
                AM_RETURN_IF_ERROR(Value(e, depth + 1));
                v.obj.emplace_back(std::move(k), std::move(e));
                Ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == '}') {
                    ++i_;
                    return Status::Ok();
                }
                return Err("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::kArray;
            ++i_;
            Ws();
            if (i_ < s_.size() && s_[i_] == ']') {
                ++i_;
                return Status::Ok();
            }
            for (;;) {
                Json e;
                AM_RETURN_IF_ERROR(Value(e, depth + 1));
                v.arr.push_back(std::move(e));
                Ws();
                if (i_ < s_.size() && s_[i_] == ',') {
                    ++i_;
                    continue;
                }
                if (i_ < s_.size() && s_[i_] == ']') {
                    ++i_;
                    return Status::Ok();
                }
                return Err("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::kString;
            return String(v.str);
        }
        if (Lit("true")) {
            v.kind = Json::kBool;
            v.b = true;
            return Status::Ok();
        }
        if (Lit("false")) {
            v.kind = Json::kBool;
            return Status::Ok();
        }
        if (Lit("null")) return Status::Ok();
        // number
        const size_t b = i_;
        while (i_ < s_.size() && (std::isdigit((unsigned char)s_[i_]) || s_[i_] == '-' || s_[i_] == '+' ||
                                  s_[i_] == '.' || s_[i_] == 'e' || s_[i_] == 'E'))
            ++i_;
        if (b == i_) return Err("unexpected character");
        try {
            v.num = std::stod(s_.substr(b, i_ - b));
        } catch (...) {
            return Err("bad number");
        }
        v.kind = Json::kNumber;
        return Status::Ok();
    }

    const std::string& s_;
    size_t i_ = 0;
};

StatusOr<std::string> ReadText(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return Status::NotFound("cannot open " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

bool FileExists(const std::string& p) {
    struct stat st {};
    return ::stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}
bool DirExists(const std::string& p) {
    struct stat st {};
    return ::stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}

}  // namespace

// ---------------------------------------------------------------- files
class MappedFile {
public:
    ~MappedFile() {
        if (base_ && base_ != MAP_FAILED) ::munmap(base_, size_);
    }
    static StatusOr<std::unique_ptr<MappedFile>> Open(const std::string& path) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) return Status::NotFound("cannot open " + path + ": " + std::strerror(errno));
        struct stat st {};
        if (::fstat(fd, &st) != 0) {
            ::close(fd);
            return Status::Internal("cannot stat " + path);
        }
        auto f = std::unique_ptr<MappedFile>(new MappedFile());
        f->size_ = (size_t)st.st_size;
        f->path_ = path;
        if (f->size_ > 0) {
            f->base_ = ::mmap(nullptr, f->size_, PROT_READ, MAP_PRIVATE, fd, 0);
            if (f->base_ == MAP_FAILED) {
                ::close(fd);
                return Status::Internal("cannot map " + path);
            }
        }
        ::close(fd);
        return f;
    }
    const uint8_t* data() const { return static_cast<const uint8_t*>(base_); }
    size_t size() const { return size_; }
    const std::string& path() const { return path_; }

private:
    MappedFile() = default;
    void* base_ = nullptr;
    size_t size_ = 0;
    std::string path_;
};

Checkpoint::~Checkpoint() = default;

Status Checkpoint::AddFile(const std::string& path) {
    auto mf = MappedFile::Open(path);
    if (!mf.ok()) return mf.status();
    const MappedFile& f = *mf.value();
    if (f.size() < 8) return Status::InvalidArgument(path + ": too short for a safetensors header");
    uint64_t hlen = 0;
    std::memcpy(&hlen, f.data(), 8);  // little-endian on the hosts this runs on
    if (hlen > f.size() - 8) return Status::InvalidArgument(path + ": header length beyond the file");
    const std::string header(reinterpret_cast<const char*>(f.data()) + 8, hlen);
    auto js = JsonParser(header).Parse();
    if (!js.ok()) return Status::InvalidArgument(path + ": " + js.status().message());
    const Json& h = js.value();
    if (h.kind != Json::kObject) return Status::InvalidArgument(path + ": header is not a JSON object");
    const uint8_t* payload = f.data() + 8 + hlen;
    const size_t payload_bytes = f.size() - 8 - hlen;
    for (const auto& kv : h.obj) {
        if (kv.first == "__metadata__") continue;
        const Json& t = kv.second;
        const Json* dt = t.Find("dtype");
        const Json* shp = t.Find("shape");
        const Json* off = t.Find("data_offsets");
        if (!dt || dt->kind != Json::kString || !shp || shp->kind != Json::kArray || !off ||
            off->kind != Json::kArray || off->arr.size() != 2)
            return Status::InvalidArgument(path + ": tensor '" + kv.first + "' lacks dtype/shape/data_offsets");
        TensorInfo ti;
        size_t esize = 0;
        if (dt->str == "F32") ti.dtype = TensorDtype::kF32, esize = 4;
        else if (dt->str == "BF16") ti.dtype = TensorDtype::kBF16, esize = 2;
        else if (dt->str == "F16") ti.dtype = TensorDtype::kF16, esize = 2;
        else return Status::InvalidArgument(path + ": tensor '" + kv.first + "' has dtype " + dt->str +
                                            " (F32, BF16 and F16 are supported)");
        for (const Json& d : shp->arr) {
            if (d.kind != Json::kNumber || d.num < 0) return Status::InvalidArgument(path + ": bad shape of " + kv.first);
            ti.shape.push_back((int64_t)d.num);
        }
        const double b0 = off->arr[0].num, b1 = off->arr[1].num;
        if (b0 < 0 || b1 < b0 || (size_t)b1 > payload_bytes)
            return Status::InvalidArgument(path + ": data_offsets of '" + kv.first + "' out of the file");
        ti.bytes = (size_t)(b1 - b0);
        if (ti.bytes != (size_t)ti.numel() * esize)
            return Status::InvalidArgument(path + ": '" + kv.first + "' byte size does not match its shape");
        ti.data = payload + (size_t)b0;
        if (tensors_.count(kv.first)) return Status::InvalidArgument("tensor '" + kv.first + "' appears twice");
        tensors_[kv.first] = std::move(ti);
    }
    files_.push_back(std::move(mf.value()));
    return Status::Ok();
}

StatusOr<const TensorInfo*> Checkpoint::Get(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) return Status::InvalidArgument("checkpoint is missing required tensor '" + name + "'");
    return &it->second;
}

StatusOr<std::unique_ptr<Checkpoint>> Checkpoint::Open(const std::string& dir) {
    if (dir.empty()) return Status::InvalidArgument("checkpoint directory path is empty");
    if (!DirExists(dir)) return Status::NotFound("checkpoint directory not found: " + dir);
    auto ck = std::unique_ptr<Checkpoint>(new Checkpoint());
    // config.json: the Llama fields the engine needs
    auto text = ReadText(dir + "/config.json");
    if (!text.ok()) return Status::NotFound("checkpoint has no config.json: " + dir);
    auto js = JsonParser(text.value()).Parse();
    if (!js.ok()) return Status::InvalidArgument("config.json: " + js.status().message());
    const Json& cj = js.value();
    auto num = [&](const char* k, bool required, double def) -> StatusOr<double> {
        const Json* v = cj.Find(k);
        if (!v || v->kind == Json::kNull) {
            if (required) return Status::InvalidArgument(std::string("config.json lacks '") + k + "'");
            return def;
        }
        if (v->kind != Json::kNumber) return Status::InvalidArgument(std::string("config.json '") + k + "' is not a number");
        return v->num;
    };
    LlamaConfig& c = ck->config_;
    auto need = [&](const char* k, int64_t& dst) -> Status {
        auto v = num(k, true, 0);
        if (!v.ok()) return v.status();
        if (v.value() <= 0 || v.value() != std::floor(v.value()))
            return Status::InvalidArgument(std::string("config.json '") + k + "' must be a positive integer");
        dst = (int64_t)v.value();
        return Status::Ok();
    };
    AM_RETURN_IF_ERROR(need("vocab_size", c.vocab));
    AM_RETURN_IF_ERROR(need("hidden_size", c.hidden));
    AM_RETURN_IF_ERROR(need("num_hidden_layers", c.layers));
    AM_RETURN_IF_ERROR(need("num_attention_heads", c.n_q_heads));
    AM_RETURN_IF_ERROR(need("intermediate_size", c.inter));
    auto kv = num("num_key_value_heads", false, (double)c.n_q_heads);
    if (!kv.ok()) return kv.status();
    c.n_kv_heads = (int64_t)kv.value();
    auto hd = num("head_dim", false, (double)(c.hidden / c.n_q_heads));
    if (!hd.ok()) return hd.status();
    c.head_dim = (int64_t)hd.value();
    auto mp = num("max_position_embeddings", false, 4096.0);
    if (!mp.ok()) return mp.status();
    c.max_position_embeddings = (int64_t)mp.value();
    auto th = num("rope_theta", false, 10000.0);
    if (!th.ok()) return th.status();
    c.rope_theta = th.value();
    auto eps = num("rms_norm_eps", false, 1e-5);
    if (!eps.ok()) return eps.status();
    c.rms_eps = (float)eps.value();
    if (const Json* t = cj.Find("tie_word_embeddings"); t && t->kind == Json::kBool) c.tied_embeddings = t->b;
    if (const Json* rs = cj.Find("rope_scaling"); rs && rs->kind == Json::kObject) {
        const Json* ty = rs->Find("rope_type");
        if (!ty) ty = rs->Find("type");
        if (ty && ty->kind == Json::kString && ty->str != "default")
            return Status::Unimplemented("config.json rope_scaling '" + ty->str + "' is not supported (plain RoPE only)");
    }
    if (c.n_kv_heads <= 0 || c.n_q_heads % c.n_kv_heads != 0)
        return Status::InvalidArgument("config.json: num_attention_heads must be a multiple of num_key_value_heads");
    // payload files
    const std::string single = dir + "/model.safetensors", index = dir + "/model.safetensors.index.json";
    if (FileExists(single)) {
        AM_RETURN_IF_ERROR(ck->AddFile(single));
    } else if (FileExists(index)) {
        auto it = ReadText(index);
        if (!it.ok()) return it.status();
        auto ij = JsonParser(it.value()).Parse();
        if (!ij.ok()) return Status::InvalidArgument("model.safetensors.index.json: " + ij.status().message());
        const Json* wm = ij.value().Find("weight_map");
        if (!wm || wm->kind != Json::kObject)
            return Status::InvalidArgument("model.safetensors.index.json has no weight_map object");
        std::set<std::string> shards;
        for (const auto& e : wm->obj) {
            if (e.second.kind != Json::kString || e.second.str.find('/') != std::string::npos)
                return Status::InvalidArgument("weight_map entry '" + e.first + "' must name a shard file in the directory");
            shards.insert(e.second.str);
        }
        for (const auto& f : shards) AM_RETURN_IF_ERROR(ck->AddFile(dir + "/" + f));
        for (const auto& e : wm->obj)
            if (!ck->Has(e.first))
                return Status::InvalidArgument("weight_map lists '" + e.first + "' but " + e.second.str + " lacks it");
    } else {
        return Status::NotFound("checkpoint has neither model.safetensors nor model.safetensors.index.json: " + dir);
    }
    return ck;
}

}  // namespace hf
}  // namespace aethermind
