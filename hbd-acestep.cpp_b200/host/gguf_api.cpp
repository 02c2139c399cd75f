// gguf_api.cpp -- C ABI over the GGUF reader (acb_models.h).
#include <string>

#include "../../include/acb_models.h"
#include "gguf.h"

struct acb_gguf {
    acb::GGUFFile f;
};

namespace acb {
thread_local std::string g_last_error;

void set_last_error(const std::string & e) {
    g_last_error = e;
}
}  // namespace acb

extern "C" const char * acb_last_error(void) {
    return acb::g_last_error.c_str();
}

extern "C" acb_status acb_gguf_open(const char * path, acb_gguf ** out) {
    if (!path || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    *out       = nullptr;
    acb_gguf * g = new acb_gguf();
    if (!g->f.open(path)) {
        acb::set_last_error(g->f.error());
        const bool io = g->f.error().rfind("cannot open", 0) == 0;
        delete g;
        return io ? ACB_ERR_IO : ACB_ERR_FORMAT;
    }
    *out = g;
    return ACB_OK;
}

extern "C" void acb_gguf_close(acb_gguf * g) {
    delete g;
}

extern "C" int64_t acb_gguf_n_tensors(const acb_gguf * g) {
    return g ? (int64_t) g->f.n_tensors() : 0;
}

extern "C" int64_t acb_gguf_find_tensor(const acb_gguf * g, const char * name) {
    if (!g || !name) {
        return -1;
    }
    const acb::GGUFTensor * t = g->f.find(name);
    if (!t) {
        return -1;
    }
    for (size_t i = 0; i < g->f.n_tensors(); i++) {
        if (g->f.tensor(i) == t) {
            return (int64_t) i;
        }
    }
    return -1;
}

extern "C" acb_status acb_gguf_tensor_info(const acb_gguf * g, int64_t idx, const char ** name, int * type,
                                           int * n_dims, int64_t * ne4, const void ** data, size_t * nbytes) {
    if (!g || idx < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const acb::GGUFTensor * t = g->f.tensor((size_t) idx);
    if (!t) {
        return ACB_ERR_OUT_OF_RANGE;
    }
    if (name) {
        *name = t->name.c_str();
    }
    if (type) {
        *type = t->type;
    }
    if (n_dims) {
        *n_dims = t->n_dims;
    }
    if (ne4) {
        for (int i = 0; i < 4; i++) {
            ne4[i] = t->ne[i];
        }
    }
    if (data) {
        *data = t->data;
    }
    if (nbytes) {
        *nbytes = t->nbytes;
    }
    return ACB_OK;
}

extern "C" uint32_t acb_gguf_get_u32(const acb_gguf * g, const char * key) {
    return g && key ? g->f.get_u32(key) : 0;
}

extern "C" float acb_gguf_get_f32(const acb_gguf * g, const char * key) {
    return g && key ? g->f.get_f32(key) : 0.0f;
}

extern "C" const char * acb_gguf_get_str(const acb_gguf * g, const char * key) {
    return g && key ? g->f.get_str(key) : "";
}

extern "C" int acb_gguf_get_bool(const acb_gguf * g, const char * key) {
    return g && key ? (int) g->f.get_bool(key) : 0;
}
