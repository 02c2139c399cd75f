// gguf.cpp -- GGUF v3 reader (public GGUF format: header, typed key/values, tensor infos,
// aligned data section). Validates every tensor against the file size like gf_load's
// truncation check (src/gguf-weights.h:132-150).
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "../../include/acb.h"

namespace acb {

namespace {
enum {
    GT_U8 = 0, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STR, GT_ARR, GT_U64, GT_I64, GT_F64,
};

size_t scalar_size(int t) {
    switch (t) {
        case GT_U8: case GT_I8: case GT_BOOL: return 1;
        case GT_U16: case GT_I16: return 2;
        case GT_U32: case GT_I32: case GT_F32: return 4;
        case GT_U64: case GT_I64: case GT_F64: return 8;
        default: return 0;
    }
}

struct Cursor {
    const uint8_t * p;
    const uint8_t * end;
    bool            ok = true;

    bool need(size_t n) {
        if (!ok || (size_t) (end - p) < n) {
            ok = false;
        }
        return ok;
    }
    template <typename T> T rd() {
        T v{};
        if (need(sizeof(T))) {
            memcpy(&v, p, sizeof(T));
            p += sizeof(T);
        }
        return v;
    }
    std::string str() {
        uint64_t n = rd<uint64_t>();
        if (!need(n)) {
            return {};
        }
        std::string s((const char *) p, (size_t) n);
        p += n;
        return s;
    }
};
}  // namespace

int64_t gguf_nbytes(int type, const int64_t * ne, int n_dims) {
    int64_t n = 1;
    for (int i = 1; i < n_dims; i++) {
        n *= ne[i];
    }
    int64_t rb = acb_row_bytes(type, ne[0]);
    if (rb < 0) {
        return -1;
    }
    return rb * n;
}

GGUFFile::~GGUFFile() {
    close();
}

void GGUFFile::close() {
    if (map_) {
        munmap(map_, size_);
        map_ = nullptr;
    }
    if (fd_ >= 0) {
        ::close(fd_);
        fd_ = -1;
    }
    tensors_.clear();
    index_.clear();
    kv_.clear();
}

bool GGUFFile::fail(const std::string & m) {
    err_ = m;
    close();
    return false;
}

bool GGUFFile::open(const char * path) {
    close();
    fd_ = ::open(path, O_RDONLY);
    if (fd_ < 0) {
        return fail(std::string("cannot open ") + path);
    }
    struct stat sb;
    if (fstat(fd_, &sb) != 0) {
        return fail("fstat failed");
    }
    size_ = (size_t) sb.st_size;
    if (size_ < 24) {
        return fail("file too small for a GGUF header");
    }
    void * m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) {
        return fail("mmap failed");
    }
    map_ = (uint8_t *) m;
    Cursor c{ map_, map_ + size_ };
    if (memcmp(map_, "GGUF", 4) != 0) {
        return fail("bad magic (not a GGUF file)");
    }
    c.p += 4;
    const uint32_t version = c.rd<uint32_t>();
    if (version < 2 || version > 3) {
        return fail("unsupported GGUF version " + std::to_string(version));
    }
    const uint64_t n_tensors = c.rd<uint64_t>();
    const uint64_t n_kv      = c.rd<uint64_t>();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) {
        return fail("implausible tensor / key counts");
    }
    for (uint64_t i = 0; i < n_kv && c.ok; i++) {
        std::string key = c.str();
        GGUFValue   v;
        v.type          = (int) c.rd<uint32_t>();
        auto rd_scalar  = [&](int t, GGUFValue & out) {
            switch (t) {
                case GT_U8: out.u = c.rd<uint8_t>(); out.i = (int64_t) out.u; break;
                case GT_I8: out.i = c.rd<int8_t>(); out.u = (uint64_t) out.i; break;
                case GT_U16: out.u = c.rd<uint16_t>(); out.i = (int64_t) out.u; break;
                case GT_I16: out.i = c.rd<int16_t>(); out.u = (uint64_t) out.i; break;
                case GT_U32: out.u = c.rd<uint32_t>(); out.i = (int64_t) out.u; break;
                case GT_I32: out.i = c.rd<int32_t>(); out.u = (uint64_t) out.i; break;
                case GT_U64: out.u = c.rd<uint64_t>(); out.i = (int64_t) out.u; break;
                case GT_I64: out.i = c.rd<int64_t>(); out.u = (uint64_t) out.i; break;
                case GT_F32: out.f = c.rd<float>(); break;
                case GT_F64: out.f = c.rd<double>(); break;
                case GT_BOOL: out.b = c.rd<uint8_t>() != 0; out.u = out.b; break;
                case GT_STR: out.s = c.str(); break;
                default: c.ok = false;
            }
        };
        if (v.type == GT_ARR) {
            v.arr_type = (int) c.rd<uint32_t>();
            v.arr_n    = c.rd<uint64_t>();
            if (v.arr_type == GT_STR) {
                for (uint64_t k = 0; k < v.arr_n && c.ok; k++) {
                    v.arr_s.push_back(c.str());
                }
            } else {
                const size_t es = scalar_size(v.arr_type);
                if (es == 0 || !c.need(es * v.arr_n)) {
                    return fail("bad array in key " + key);
                }
                c.p += es * v.arr_n;
            }
        } else {
            rd_scalar(v.type, v);
        }
        if (!c.ok) {
            return fail("truncated key/value section at " + key);
        }
        kv_[key] = std::move(v);
    }
    tensors_.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors && c.ok; i++) {
        GGUFTensor & t = tensors_[i];
        t.name         = c.str();
        t.n_dims       = (int) c.rd<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) {
            return fail("bad n_dims for " + t.name);
        }
        for (int d = 0; d < t.n_dims; d++) {
            t.ne[d] = (int64_t) c.rd<uint64_t>();
        }
        t.type   = (int) c.rd<uint32_t>();
        t.offset = c.rd<uint64_t>();
    }
    if (!c.ok) {
        return fail("truncated tensor-info section");
    }
    uint64_t     align = 32;
    const auto * a     = kv("general.alignment");
    if (a && a->u > 0) {
        align = a->u;
    }
    const size_t hdr = (size_t) (c.p - map_);
    data_off_        = (hdr + align - 1) / align * align;
    for (size_t i = 0; i < tensors_.size(); i++) {
        GGUFTensor &  t  = tensors_[i];
        const int64_t nb = gguf_nbytes(t.type, t.ne, t.n_dims);
        if (nb < 0) {
            return fail("unsupported tensor type " + std::to_string(t.type) + " for " + t.name);
        }
        t.nbytes         = (size_t) nb;
        const size_t end = data_off_ + t.offset + t.nbytes;
        if (end > size_) {
            return fail("'" + t.name + "' is truncated or corrupt: needs bytes up to " + std::to_string(end) +
                        " but the file has " + std::to_string(size_));
        }
        t.data = map_ + data_off_ + t.offset;
        index_[t.name] = i;
    }
    return true;
}

const GGUFTensor * GGUFFile::find(const std::string & name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

const GGUFValue * GGUFFile::kv(const std::string & key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
}

uint32_t GGUFFile::get_u32(const char * key) const {
    const GGUFValue * v = kv(key);
    return v ? (uint32_t) v->u : 0;
}

float GGUFFile::get_f32(const char * key) const {
    const GGUFValue * v = kv(key);
    return v ? (float) v->f : 0.0f;
}

const char * GGUFFile::get_str(const char * key) const {
    const GGUFValue * v = kv(key);
    return v && v->type == GT_STR ? v->s.c_str() : "";
}

bool GGUFFile::get_bool(const char * key) const {
    const GGUFValue * v = kv(key);
    return v ? v->b : false;
}

}  // namespace acb
