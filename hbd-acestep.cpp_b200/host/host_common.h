// host_common.h -- helpers shared by the host model drivers.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/acb.h"

namespace acb {

void set_last_error(const std::string & e);

#define ACB_TRY(x)                 \
    do {                           \
        const acb_status s_ = (x); \
        if (s_ != ACB_OK) {        \
            return s_;             \
        }                          \
    } while (0)

// IEEE binary16 / bfloat16 storage to float (exact).
inline float host_bf16_to_f32(uint16_t h) {
    const uint32_t u = (uint32_t) h << 16;
    float          f;
    memcpy(&f, &u, 4);
    return f;
}

// float to bfloat16, round to nearest even (NaN kept a quiet NaN), as ggml_fp32_to_bf16 does
inline uint16_t host_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        return (uint16_t) ((u >> 16) | 64);
    }
    return (uint16_t) ((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
}

inline float host_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000) << 16;
    const uint32_t exp  = (h >> 10) & 0x1f;
    const uint32_t man  = h & 0x3ff;
    uint32_t       u;
    if (exp == 0) {
        const float v = (float) man * 5.9604644775390625e-8f;  // subnormal: man * 2^-24
        return sign ? -v : v;
    }
    if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// Value text of "key": in a flat JSON object (the lookup of qw3lm_json_int / _float / _bool,
// src/qwen3-lm.h:60-121), or nullptr.
inline const char * json_value(const char * j, const char * key) {
    char needle[128];
    snprintf(needle, sizeof(needle), "\"%s\"", key);
    const char * p = strstr(j, needle);
    if (!p) {
        return nullptr;
    }
    p = strchr(p + strlen(needle), ':');
    if (!p) {
        return nullptr;
    }
    p++;
    while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') {
        p++;
    }
    return p;
}

inline int json_int(const char * j, const char * key, int fb) {
    const char * v = json_value(j, key);
    return v ? atoi(v) : fb;
}

inline float json_float(const char * j, const char * key, float fb) {
    const char * v = json_value(j, key);
    return v ? (float) atof(v) : fb;
}

inline bool json_bool(const char * j, const char * key, bool fb) {
    const char * v = json_value(j, key);
    return v ? strncmp(v, "true", 4) == 0 : fb;
}

// kernel nodes of a captured graph (the library's own launches; copies and memsets not counted)
inline int graph_kernel_nodes(cudaGraph_t g) {
    size_t n = 0;
    if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess || n == 0) {
        return 0;
    }
    cudaGraphNode_t * nodes = (cudaGraphNode_t *) malloc(n * sizeof(cudaGraphNode_t));
    if (!nodes) {
        return 0;
    }
    int k = 0;
    if (cudaGraphGetNodes(g, nodes, &n) == cudaSuccess) {
        for (size_t i = 0; i < n; i++) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) {
                k++;
            }
        }
    }
    free(nodes);
    return k;
}

}  // namespace acb
