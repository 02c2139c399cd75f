// weights.cpp -- device weight arena (see weights.h).
#include "weights.h"

#include <algorithm>

#include <cstring>

#include "host_common.h"

namespace acb {

WeightArena::~WeightArena() {
    if (base_) {
        cudaFree(base_);
    }
}

DevTensor * WeightArena::reserve(int type, int64_t K, int64_t N, size_t nbytes) {
    tensors_.emplace_back();
    DevTensor & t = tensors_.back();
    t.type        = type;
    t.K           = K;
    t.N           = N;
    t.nbytes      = nbytes;
    t.offset      = total_;
    total_        = (total_ + nbytes + 256 + 255) / 256 * 256;
    return &t;
}

static void dims_kn(const GGUFTensor * s, int64_t & K, int64_t & N) {
    K = s->ne[0];
    N = 1;
    for (int i = 1; i < s->n_dims; i++) {
        N *= s->ne[i];
    }
}

DevTensor * WeightArena::try_load(const GGUFFile & gf, const std::string & name) {
    const GGUFTensor * s = gf.find(name);
    if (!s) {
        return nullptr;
    }
    int64_t K, N;
    dims_kn(s, K, N);
    DevTensor * t = reserve(s->type, K, N, s->nbytes);
    pending_.push_back({ t, s->data, s->nbytes, 0 });
    by_name_[name] = t;
    return t;
}

DevTensor * WeightArena::get(const std::string & name) const {
    const auto it = by_name_.find(name);
    return it == by_name_.end() ? nullptr : it->second;
}

std::vector<std::string> WeightArena::names() const {
    std::vector<std::string> out;
    out.reserve(by_name_.size());
    for (const auto & kv : by_name_) {
        out.push_back(kv.first);
    }
    std::sort(out.begin(), out.end());
    return out;
}

DevTensor * WeightArena::load(const GGUFFile & gf, const std::string & name) {
    DevTensor * t = try_load(gf, name);
    if (!t) {
        error = "tensor '" + name + "' not found";
    }
    return t;
}

DevTensor * WeightArena::load_f32(const GGUFFile & gf, const std::string & name) {
    const GGUFTensor * s = gf.find(name);
    if (!s) {
        error = "tensor '" + name + "' not found";
        return nullptr;
    }
    if (s->type == ACB_TYPE_F32) {
        return load(gf, name);
    }
    if (s->type != ACB_TYPE_BF16 && s->type != ACB_TYPE_F16) {
        return load(gf, name);  // loaded as-is, like gf_load_tensor_f32's fallback
    }
    int64_t K, N;
    dims_kn(s, K, N);
    const size_t             n = (size_t) (K * N);
    std::unique_ptr<float[]> buf(new float[n]);
    const uint16_t *         p = (const uint16_t *) s->data;
    for (size_t i = 0; i < n; i++) {
        buf[i] = s->type == ACB_TYPE_BF16 ? host_bf16_to_f32(p[i]) : host_f16_to_f32(p[i]);
    }
    DevTensor * t = reserve(ACB_TYPE_F32, K, N, n * 4);
    pending_.push_back({ t, buf.get(), n * 4, 0 });
    staging_.push_back(std::move(buf));
    by_name_[name] = t;
    return t;
}

DevTensor * WeightArena::load_fused(const GGUFFile & gf, const std::vector<std::string> & names) {
    std::vector<const GGUFTensor *> src;
    for (const auto & n : names) {
        const GGUFTensor * s = gf.find(n);
        if (!s) {
            return nullptr;
        }
        src.push_back(s);
    }
    int64_t K0, N0;
    dims_kn(src[0], K0, N0);
    int64_t Ntot = 0;
    size_t  nb   = 0;
    for (const auto * s : src) {
        int64_t K, N;
        dims_kn(s, K, N);
        if (K != K0 || s->type != src[0]->type) {
            return nullptr;  // caller falls back to separate loads
        }
        Ntot += N;
        nb += s->nbytes;
    }
    DevTensor * t   = reserve(src[0]->type, K0, Ntot, nb);
    size_t      off = 0;
    for (const auto * s : src) {
        pending_.push_back({ t, s->data, s->nbytes, off });
        off += s->nbytes;
    }
    return t;
}

DevTensor * WeightArena::add_host(int type, int64_t K, int64_t N, const void * src, size_t nbytes) {
    std::unique_ptr<float[]> buf(new float[(nbytes + 3) / 4]);
    memcpy(buf.get(), src, nbytes);
    DevTensor * t = reserve(type, K, N, nbytes);
    pending_.push_back({ t, buf.get(), nbytes, 0 });
    staging_.push_back(std::move(buf));
    return t;
}

acb_status WeightArena::upload(cudaStream_t st) {
    if (total_ == 0) {
        return ACB_OK;
    }
    cudaError_t e = cudaMalloc(&base_, total_);
    if (e != cudaSuccess) {
        base_ = nullptr;
        error = "cudaMalloc of the weight arena failed";
        return ACB_ERR_OOM;
    }
    cudaMemsetAsync(base_, 0, total_, st);
    for (auto & t : tensors_) {
        t.data = (uint8_t *) base_ + t.offset;
    }
    for (const auto & pc : pending_) {
        e = cudaMemcpyAsync((uint8_t *) pc.t->data + pc.dst_off, pc.src, pc.nbytes, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) {
            error = "weight upload failed";
            return ACB_ERR_CUDA;
        }
    }
    e = cudaStreamSynchronize(st);
    pending_.clear();
    staging_.clear();
    return e == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

acb_status DevBuf::alloc(size_t n, bool zero) {
    release();
    if (n == 0) {
        return ACB_OK;
    }
    if (cudaMalloc(&p, n) != cudaSuccess) {
        p = nullptr;
        return ACB_ERR_OOM;
    }
    bytes = n;
    if (zero && cudaMemset(p, 0, n) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

void DevBuf::release() {
    if (p) {
        cudaFree(p);
        p = nullptr;
    }
    bytes = 0;
}

}  // namespace acb
