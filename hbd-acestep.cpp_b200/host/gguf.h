// gguf.h -- GGUF v3 reader (mmap), the replacement for gguf-weights.h's gf_load / gf_get_*
// (src/gguf-weights.h:74-155, 357-390) without ggml. Tensor data stays in the mapping until it
// is uploaded to the device.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace acb {

struct GGUFTensor {
    std::string name;
    int         type    = 0;
    int         n_dims  = 0;
    int64_t     ne[4]   = { 1, 1, 1, 1 };
    uint64_t    offset  = 0;  // relative to the data section
    size_t      nbytes  = 0;
    const uint8_t * data = nullptr;
};

struct GGUFValue {
    int                      type = -1;  // gguf value type
    uint64_t                 u    = 0;
    int64_t                  i    = 0;
    double                   f    = 0.0;
    bool                     b    = false;
    std::string              s;
    int                      arr_type = -1;
    uint64_t                 arr_n    = 0;
    std::vector<std::string> arr_s;      // string arrays only
};

class GGUFFile {
  public:
    ~GGUFFile();
    // Opens and validates the file; on failure returns false and sets error().
    bool open(const char * path);
    void close();

    const std::string & error() const { return err_; }
    size_t              n_tensors() const { return tensors_.size(); }
    const GGUFTensor *  tensor(size_t i) const { return i < tensors_.size() ? &tensors_[i] : nullptr; }
    const GGUFTensor *  find(const std::string & name) const;
    const GGUFValue *   kv(const std::string & key) const;

    uint32_t     get_u32(const char * key) const;  // 0 if missing (gf_get_u32)
    float        get_f32(const char * key) const;  // 0 if missing (gf_get_f32)
    const char * get_str(const char * key) const;  // "" if missing (gf_get_str)
    bool         get_bool(const char * key) const;  // false if missing (gf_get_bool)

  private:
    bool fail(const std::string & m);

    std::string                             err_;
    int                                     fd_      = -1;
    uint8_t *                               map_     = nullptr;
    size_t                                  size_    = 0;
    size_t                                  data_off_ = 0;
    std::vector<GGUFTensor>                 tensors_;
    std::unordered_map<std::string, size_t> index_;
    std::unordered_map<std::string, GGUFValue> kv_;
};

// bytes of a tensor of `ne` elements along ne0 rows (GGUF block sizes); -1 if invalid
int64_t gguf_nbytes(int type, const int64_t * ne, int n_dims);

}  // namespace acb
