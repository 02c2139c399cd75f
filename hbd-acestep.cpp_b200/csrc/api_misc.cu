// api_misc.cu -- library-level entry points: version, status strings, row sizes, RoPE table.
#include <math.h>

#include <atomic>

#include "common.cuh"

namespace acb {
static std::atomic<int> g_last_cuda_error{ 0 };

void set_last_cuda_error(cudaError_t e) {
    g_last_cuda_error.store((int) e);
}
}  // namespace acb

extern "C" int acb_version(void) {
    return (0 << 16) | (1 << 8) | 0;
}

extern "C" const char * acb_status_string(int status) {
    switch (status) {
        case ACB_OK:
            return "ok";
        case ACB_ERR_INVALID_ARG:
            return "invalid argument";
        case ACB_ERR_UNSUPPORTED:
            return "unsupported type or shape";
        case ACB_ERR_CUDA:
            return "CUDA error";
        case ACB_ERR_OUT_OF_RANGE:
            return "index out of range";
        case ACB_ERR_OOM:
            return "out of memory";
        case ACB_ERR_IO:
            return "I/O error";
        case ACB_ERR_FORMAT:
            return "malformed GGUF or missing tensor";
        case ACB_ERR_DEVICE:
            return "device-side error flag set";
        default:
            return "unknown status";
    }
}

extern "C" int acb_last_cuda_error(void) {
    return acb::g_last_cuda_error.load();
}

extern "C" int64_t acb_row_bytes(int type, int64_t n) {
    int be = 0, bb = 0;
    switch (type) {
        case ACB_TYPE_F32:
            be = 1, bb = 4;
            break;
        case ACB_TYPE_F16:
        case ACB_TYPE_BF16:
            be = 1, bb = 2;
            break;
        case ACB_TYPE_Q8_0:
        case ACB_TYPE_Q8_0_TILES:
            be = 32, bb = 34;
            break;
        case ACB_TYPE_Q4_K:
            be = 256, bb = 144;
            break;
        case ACB_TYPE_Q6_K:
            be = 256, bb = 210;
            break;
        case ACB_TYPE_Q8_K:
            be = 256, bb = 292;
            break;
        case ACB_TYPE_I32:
            be = 1, bb = 4;
            break;
        default:
            return -1;
    }
    if (n < 0 || n % be != 0) {
        return -1;
    }
    return n / be * bb;
}

// The rope cache of ggml's NEOX mode with freq_scale 1 and ext_factor 0: the angle of pair i
// at position p is built by repeated float multiplication theta <- theta * base^(-2/D),
// starting from theta = p, and cos/sin are taken in float. Sharing this table between the
// CPU and GPU paths makes the rotation bit-identical at every position.
extern "C" acb_status acb_rope_table_host(float * table, int max_pos, int head_dim, float base) {
    if (!table || max_pos <= 0 || head_dim <= 0 || head_dim % 2 != 0 || !(base > 0.0f)) {
        return ACB_ERR_INVALID_ARG;
    }
    const float theta_scale = powf(base, -2.0f / (float) head_dim);
    for (int p = 0; p < max_pos; p++) {
        float   theta = (float) p;
        float * row   = table + (int64_t) p * head_dim;
        for (int i = 0; i < head_dim / 2; i++) {
            row[2 * i]     = cosf(theta);
            row[2 * i + 1] = sinf(theta);
            theta          = theta * theta_scale;
        }
    }
    return ACB_OK;
}
