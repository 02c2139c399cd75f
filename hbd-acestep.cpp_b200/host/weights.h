// weights.h -- device weight arena: the WeightCtx + gf_load_* replacement
// (src/weight-ctx.h:21-86, src/gguf-weights.h:159-354). Tensors are registered first (pending
// host copies straight from the GGUF mapping, or from converted staging buffers), then one
// device allocation is made and every piece is uploaded. Each tensor starts on a 256-byte
// boundary and is followed by >= 256 bytes of padding, so whole-16-byte bulk copies of the
// last rows never leave the allocation.
#pragma once

#include <cuda_runtime.h>

#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/acb.h"
#include "gguf.h"

namespace acb {

struct DevTensor {
    int     type   = -1;
    void *  data   = nullptr;
    int64_t K      = 0;  // ne0 (elements per row)
    int64_t N      = 0;  // rows (product of ne1..)
    size_t  nbytes = 0;
    size_t  offset = 0;  // in the arena

    bool valid() const { return type >= 0; }
    int64_t row_bytes() const { return acb_row_bytes(type, K); }
};

class WeightArena {
  public:
    ~WeightArena();

    // gf_load_tensor: native type. Returns nullptr (and sets error) if missing.
    DevTensor * load(const GGUFFile & gf, const std::string & name);
    DevTensor * try_load(const GGUFFile & gf, const std::string & name);
    // gf_load_tensor_f32: BF16/F16 converted to F32 on the host.
    DevTensor * load_f32(const GGUFFile & gf, const std::string & name);
    // gf_load_qkv_fused / gf_load_pair_fused: row concatenation when all types match, else nullptr.
    DevTensor * load_fused(const GGUFFile & gf, const std::vector<std::string> & names);
    // A host-provided tensor (e.g. a constant).
    DevTensor * add_host(int type, int64_t K, int64_t N, const void * src, size_t nbytes);
    // The tensor loaded under a GGUF name (load / try_load / load_f32), or nullptr.
    DevTensor * get(const std::string & name) const;
    // names of the tensors loaded one by one (not the fused ones), sorted
    std::vector<std::string> names() const;

    // wctx_alloc: one cudaMalloc and every pending upload.
    acb_status upload(cudaStream_t st);
    size_t     bytes() const { return total_; }

    std::string error;

  private:
    struct Pending {
        DevTensor *  t;
        const void * src;
        size_t       nbytes;
        size_t       dst_off;
    };

    DevTensor * reserve(int type, int64_t K, int64_t N, size_t nbytes);

    std::deque<DevTensor>                 tensors_;
    std::unordered_map<std::string, DevTensor *> by_name_;
    std::vector<Pending>                  pending_;
    std::vector<std::unique_ptr<float[]>> staging_;
    size_t                                total_ = 0;
    void *                                base_  = nullptr;
};

// a device buffer owned by a model (scratch, caches)
struct DevBuf {
    void * p     = nullptr;
    size_t bytes = 0;
    ~DevBuf() { release(); }
    acb_status alloc(size_t n, bool zero = true);
    void       release();
    template <typename T> T * as() const { return reinterpret_cast<T *>(p); }
};

}  // namespace acb
